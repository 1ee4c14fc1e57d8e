// fused.cuh — the single-launch sampling pass (k_fused), included by sampler.cu inside its
// anonymous namespace after the shared helpers (row configuration, penalties, keys, the
// finishing arithmetic and the exact search).
//
// One persistent CTA per SM, ten warps, each with one job and no CTA-wide barrier while
// streaming. The batch is a row-major list of tiles (6 KiB of one row each); CTA b streams the
// contiguous tiles [b * ntt / G, (b + 1) * ntt / G), so every CTA moves the same bytes. A CTA's
// range meets a few rows; its piece of one row is a "part".
//
//   * Warp 8, the producer: before the first tile of each part it prepares the part's slot
//     (one of two, alternating): the row's parameters, the part's history entries copied into
//     shared memory by bulk copies, and the first entry of each tile in them. Then it copies the
//     tiles into a 16-stage shared-memory ring with cp.async.bulk (TMA, no multicast), each
//     stage's mbarrier counting the bytes. Up to 96 KiB per SM are in flight, about 2 us of
//     the SM's share of HBM bandwidth.
//   * Warps 0-7, the consumers: tile i of the range goes to warp i % 8 (stage i % 16, so each
//     warp has one tile landing while it works on another). Per tile the warp first handles the
//     penalised tokens inside it (raw logit read from the stage, penalised exactly, kept as a
//     scalar candidate, overwritten with -inf in the stage), then takes the maximum of each
//     16-byte vector and compares it with the part's filter; a vector that reaches it is noted
//     as a delegate (its maximum and position) in the warp's list. Rows without top-k also keep
//     an online softmax maximum and sum. The filter is the smallest logit whose processed value
//     reaches the part's bound: the K-th largest of K distinct elements' values (first from a
//     warp's first tile, then from its list when it fills), raised CTA-wide with atomicMax.
//   * Warp 9, the finisher: once the eight consumers have handed in a part (an mbarrier), it
//     expands the delegates that still reach the final bound (re-read from L2: the part was just
//     streamed), keeps the K largest with the ties of the K-th, sorts them and writes the part's
//     record with its completeness key (every element of the part at or above it is listed).
//     The record is counted on the row's counter (release); the CTA completing the row merges
//     the row's records, checks that the row's K-th reaches every part's completeness key,
//     applies top-p / min-p and draws (or writes this rank's shard record). Rows the records
//     cannot decide are queued; the consumers search them exactly once streaming is over.

constexpr int FW = 8;                          // consumer warps
constexpr int FPROD = FW;                      // the producer warp
constexpr int FFIN = FW + 1;                   // the finisher warps: part p goes to
constexpr int FNFIN = 2;                       //   FFIN + p % FNFIN
constexpr int FPREP = FFIN + FNFIN;            // the warp that prepares the parts' slots
constexpr int FNT = (FPREP + 1) * 32;
constexpr int FNSLOT = 3;                      // parts in flight (prepared, streamed, finished)
constexpr int FSTAGES = 16;                    // tiles in flight per CTA
constexpr int FTILE = 6144;                    // bytes of one tile (one stage)
constexpr int FVEC = FTILE / 16;               // 16-byte vectors of a tile
constexpr int FVPL = FVEC / 32;                // ... per lane of its warp
constexpr int FHCAP = 2048;                    // history entries of a part staged in shared memory
constexpr int FWB = 192;                       // candidate list of one consumer warp
constexpr int FKF = 96;                        // largest top-k the candidate lists serve
constexpr int FSUMK = 64;                      // entries kept per part for rows without top-k
constexpr int FCAP = 1024;                     // candidates a part or a row merges
constexpr int FRCAP = 128;                     // entries of a part record
constexpr int FMAXP = 16;                      // parts of one row (record slots)
constexpr int FMAXT = (int)(((int64_t)VINFER_MAX_VOCAB * 4 + FTILE - 1) / FTILE);  // longest row
constexpr size_t FREC_STRIDE = sizeof(RecHdr) + 8 * FRCAP;
constexpr int FQ_HDR = 4;                      // deferred-row queue: pushed, claimed, CTAs done
// Stage i % FSTAGES holds tile i and tile i goes to warp i % FW, so with FSTAGES a multiple of
// FW every stage belongs to one warp, which waits on its phases in order. (A stage shared by two
// warps would let one wait for a phase two ahead of the barrier's, which a one-bit phase parity
// reports as complete.)
static_assert(FSTAGES % FW == 0 && FSTAGES >= 2 * FW, "each consumer owns two stages");
static_assert(FVPL * 32 * 16 == FTILE && FVPL <= 32, "a consumer lane takes FVPL vectors");
static_assert(FKF + 64 <= FWB - 32, "a tightened list leaves room for a round of appends");
static_assert(KC <= FSUMK && FSUMK <= FRCAP && FKF <= FRCAP, "records hold the kept entries");

enum { FM_CANDS = 0, FM_SUM = 1, FM_SKIP = 2 };

// one part's shared state: written by the producer before the part's tiles, by the consumers
// during them, read by the finisher after them
struct __align__(16) FSlot {
  int hid[FHCAP + 4];                          // the part's history ids (global), from hbase ...
  int hcnt[FHCAP + 4];                         // ... and counts
  int hoff[FMAXT + 1];                         // first staged entry of each tile of the part
  float prm[8];                                // the row's parameters (load_param order)
  int hbase, nh;                               // staged entries: [hbase, hbase + nh)
  int exact;                                   // the history did not fit: exact search
  uint32_t thr_key;                            // the part's bound: processed key (atomicMax)
  uint32_t thr_raw;                            // ... and the smallest logit reaching it
  int wc[FW], wovf[FW];                        // consumer lists: length, overflow
  float wm[FW], wsum[FW];                      // consumer softmax maxima and sums
  uint32_t fmax[FW * 32];                      // each warp's 32 largest first-tile vector maxima
  int nfirst;                                  // warps that wrote theirs
};

struct __align__(128) FSmem {
  unsigned char stage[FSTAGES][FTILE];         // the ring; after streaming, Smem for exact_row
  FSlot slot[FNSLOT];
  unsigned long long wbuf[FNSLOT][FW][FWB];    // consumer candidate lists, per slot
  struct Fin {                                 // one finisher warp's scratch
    unsigned long long cand[FCAP];             // a part's candidates; a row's records
    unsigned long long srt[FCAP];              // ... sorted
    RecHdr ph[FMAXP];                          // a row's part headers
    int poff[FMAXP + 1];
  } fin[FNFIN];
  unsigned long long full[FSTAGES];            // mbarriers: tile landed
  unsigned long long empty[FSTAGES];           // ... consumer done with the stage
  unsigned long long ready[FNSLOT];            // ... slot prepared (prep warp)
  unsigned long long handed[FNSLOT];           // ... all consumers done with the part
  unsigned long long done[FNSLOT];             // ... finisher done with the part
  unsigned long long hbar;                     // ... history copy landed (producer)
  unsigned long long fin_all;                  // ... finisher done with every part
  int abort_, claim;
};
static_assert(sizeof(Smem) <= sizeof(((FSmem*)nullptr)->stage),
              "the exact search's shared memory fits the drained ring");
static_assert(sizeof(FSmem) <= 227 * 1024, "one CTA's shared memory");
static_assert(offsetof(FSlot, hcnt) % 16 == 0 && sizeof(FSlot) % 16 == 0,
              "staged history arrays are 16-byte aligned for bulk copies");

// ---- mbarriers and bulk copies ---------------------------------------------------------------
__device__ __forceinline__ uint32_t smem_addr(const void* p) {
  return (uint32_t)__cvta_generic_to_shared(p);
}
__device__ __forceinline__ void mbar_init(unsigned long long* b, uint32_t count) {
  asm volatile("mbarrier.init.shared::cta.b64 [%0], %1;" ::"r"(smem_addr(b)), "r"(count)
               : "memory");
}
// one test of a barrier phase; a waiting thread is suspended for up to about 20 us (it resumes
// as soon as the phase completes), so waiting warps do not spin on the issue slots
__device__ __forceinline__ bool mbar_try_wait(unsigned long long* b, uint32_t parity) {
  uint32_t ok;
  asm volatile(
      "{\n\t.reg .pred p;\n\t"
      "mbarrier.try_wait.parity.shared::cta.b64 p, [%1], %2, %3;\n\t"
      "selp.u32 %0, 1, 0, p;\n\t}"
      : "=r"(ok)
      : "r"(smem_addr(b)), "r"(parity), "r"(20000u)
      : "memory");
  return ok != 0u;
}
__device__ __forceinline__ void mbar_arrive(unsigned long long* b) {
  asm volatile("mbarrier.arrive.shared::cta.b64 _, [%0];" ::"r"(smem_addr(b)) : "memory");
}
__device__ __forceinline__ void mbar_arrive_tx(unsigned long long* b, uint32_t bytes) {
  asm volatile("mbarrier.arrive.expect_tx.shared::cta.b64 _, [%0], %1;" ::"r"(smem_addr(b)),
               "r"(bytes)
               : "memory");
}
// one bulk copy global -> this CTA's shared memory (no multicast); both addresses 16-byte
// aligned, bytes a multiple of 16
__device__ __forceinline__ void bulk_load(void* dst, const void* src, uint32_t bytes,
                                          unsigned long long* bar) {
  asm volatile(
      "cp.async.bulk.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1], %2, [%3];"
      ::"r"(smem_addr(dst)), "l"(src), "r"(bytes), "r"(smem_addr(bar))
      : "memory");
}
// Bounded wait for a barrier phase: gives up after about two seconds (or at once when the
// CTA has already given up), reports VINFER_ST_TIMEOUT and returns false.
__device__ bool fwait(const KParams& P, FSmem& S, unsigned long long* b, uint32_t parity) {
  if (mbar_try_wait(b, parity)) return true;
  uint64_t t0;
  asm volatile("mov.u64 %0, %%globaltimer;" : "=l"(t0));
  for (int it = 0;; ++it) {
    if (mbar_try_wait(b, parity)) return true;
    if (*reinterpret_cast<volatile int*>(&S.abort_)) return false;
    if ((it & 255) == 255) {
      uint64_t t;
      asm volatile("mov.u64 %0, %%globaltimer;" : "=l"(t));
      if (t - t0 > 2000000000ull) {
        S.abort_ = 1;
        status_or(P, VINFER_ST_TIMEOUT);
        return false;
      }
    }
  }
}

// ---- geometry ----------------------------------------------------------------------------------
__device__ __forceinline__ int64_t ftile0(const KParams& P, int b) {
  return (int64_t)b * P.ntt / P.geff;
}
// the CTA streaming global tile g (every CTA has at least one tile)
__device__ int fcta_of(const KParams& P, int64_t g) {
  int b = (int)((g * P.geff) / P.ntt);
  b = min(max(b, 0), P.geff - 1);
  while (b + 1 < P.geff && ftile0(P, b + 1) <= g) ++b;
  while (b > 0 && ftile0(P, b) > g) --b;
  return b;
}

// tile j of a row: local elements [e0, e1); the 16-byte aligned interior goes through the ring
// (nv vectors starting at element e0 + hoff); the ragged elements around it are read directly
struct FTileGeo {
  const unsigned char* src;
  uint32_t bytes;
  int e0, e1, hoff, nv;
};
template <typename TIn>
__device__ __forceinline__ FTileGeo ftile(const KParams& P, int row, int j) {
  FTileGeo t;
  const TIn* rowp = (const TIn*)P.logits + (int64_t)row * P.ld;
  t.e0 = j * P.te;
  t.e1 = (int)min((int64_t)t.e0 + P.te, P.V);
  const uintptr_t a0 = (uintptr_t)(rowp + t.e0), a1 = (uintptr_t)(rowp + t.e1);
  const uintptr_t b0 = (a0 + 15u) & ~(uintptr_t)15u, b1 = a1 & ~(uintptr_t)15u;
  if (b1 > b0) {
    t.src = (const unsigned char*)b0;
    t.bytes = (uint32_t)(b1 - b0);
    t.hoff = (int)((b0 - a0) / sizeof(TIn));
    t.nv = (int)(t.bytes / 16u);
  } else {
    t.src = nullptr;
    t.bytes = 0u;
    t.hoff = t.e1 - t.e0;
    t.nv = 0;
  }
  return t;
}


__device__ __forceinline__ int lower_bound_smem(const int* a, int n, int64_t x) {
  int lo = 0, hi = n;
  while (lo < hi) {
    const int mid = (lo + hi) >> 1;
    if ((int64_t)a[mid] < x) lo = mid + 1; else hi = mid;
  }
  return lo;
}

// ---- warp-level selection and sorting ----------------------------------------------------------
// A lower bound on the K-th largest of the warp's keys (NK per lane, 0 = absent): the largest
// 16-bit prefix p such that at least K keys are >= p << 16, built bit by bit, returned as p << 16
// (so at least K keys reach it); 0 when fewer than K keys are present. Keys of bf16 logits differ
// only in their high half, so for them the bound is the K-th largest key itself.
template <int NK>
__device__ __forceinline__ uint32_t warp_kth_hi(const uint32_t (&k)[NK], int K) {
  uint32_t v = 0u;
#pragma unroll 1
  for (int bit = 31; bit >= 16; --bit) {
    const uint32_t cand = v | (1u << bit);
    int cnt = 0;
#pragma unroll
    for (int i = 0; i < NK; ++i) cnt += k[i] >= cand ? 1 : 0;
    cnt = __reduce_add_sync(FULLMASK, cnt);
    if (cnt >= K) v = cand;
  }
  return v;
}
// the K-th largest key of entries e[0, n) in shared memory, exactly (32 rounds); 0 when n < K
__device__ uint32_t warp_kth_smem(const unsigned long long* e, int n, int K) {
  const int lane = threadIdx.x & 31;
  uint32_t v = 0u;
#pragma unroll 1
  for (int bit = 31; bit >= 0; --bit) {
    const uint32_t cand = v | (1u << bit);
    int cnt = 0;
    for (int j = lane; j < n; j += 32) cnt += comp_key(e[j]) >= cand ? 1 : 0;
    cnt = __reduce_add_sync(FULLMASK, cnt);
    if (cnt >= K) v = cand;
  }
  return v;
}
// Ascending bitonic sort of 32 * NPL entries held NPL per lane: entry e = i * 32 + lane is
// x[i] of that lane. Compare-exchanges across lanes use shuffles, within a lane registers.
template <int NPL>
__device__ __forceinline__ void warp_bitonic(unsigned long long (&x)[NPL]) {
  const int lane = threadIdx.x & 31;
  constexpr int N = 32 * NPL;
#pragma unroll
  for (int k = 2; k <= N; k <<= 1) {
#pragma unroll
    for (int j = k >> 1; j > 0; j >>= 1) {
      if (j >= 32) {
        const int r = j / 32;
#pragma unroll
        for (int i = 0; i < NPL; ++i) {
          const int p = i ^ r;
          if (p > i) {
            const int e = i * 32 + lane;
            const bool up = (e & k) == 0;
            const unsigned long long a = x[i], b = x[p];
            if ((a > b) == up) {
              x[i] = b;
              x[p] = a;
            }
          }
        }
      } else {
#pragma unroll
        for (int i = 0; i < NPL; ++i) {
          const int e = i * 32 + lane;
          const unsigned long long o = __shfl_xor_sync(FULLMASK, x[i], j);
          const bool up = (e & k) == 0;
          const bool lower = (lane & j) == 0;
          // the lower position keeps the smaller (ascending run) or the larger one
          const bool take_min = (lower == up);
          x[i] = take_min ? (o < x[i] ? o : x[i]) : (o > x[i] ? o : x[i]);
        }
      }
    }
  }
}
// sort e[0, n) (n <= 32 * NPL) in shared memory ascending, in place, by one warp
template <int NPL>
__device__ __forceinline__ void warp_sort_smem(unsigned long long* e, int n) {
  const int lane = threadIdx.x & 31;
  unsigned long long x[NPL];
#pragma unroll
  for (int i = 0; i < NPL; ++i) {
    const int j = i * 32 + lane;
    x[i] = j < n ? e[j] : ~0ull;
  }
  warp_bitonic<NPL>(x);
  __syncwarp();
#pragma unroll
  for (int i = 0; i < NPL; ++i) {
    const int j = i * 32 + lane;
    if (j < n) e[j] = x[i];
  }
  __syncwarp();
}
// warp-wide exclusive prefix sum of one int per lane; *total receives the sum
__device__ __forceinline__ int warp_excl(int v, int* total) {
  const int lane = threadIdx.x & 31;
  int inc = v;
#pragma unroll
  for (int o = 1; o < 32; o <<= 1) {
    const int t = __shfl_up_sync(FULLMASK, inc, o);
    if (lane >= o) inc += t;
  }
  *total = __shfl_sync(FULLMASK, inc, 31);
  return inc - v;
}

// ---- candidate lists -----------------------------------------------------------------------------
// Each consumer warp keeps its own list per part. An entry is comp(okey(y), id): y is an element's
// pre-temperature value (penalised where it has history), ordered like the processed values, so
// nothing is divided while streaming; the part's end converts the survivors to processed keys.
// The entries are distinct elements, so K of them bound the row's K-th largest value from below.

// The row's values the consumers use, as scalars (kept in registers: nothing on the streaming
// path takes the address of a row configuration)
struct FRow {
  float T, c2, rep, pres, freq;
  int K;
  bool greedy, pen, pen_down;
};
__device__ __forceinline__ float vf_s(float y, const FRow& r) {
  return r.greedy ? y : __fdiv_rn(y, r.T);
}
// penalties: repetition, then frequency * count, then presence; one IEEE op each (penalize)
__device__ __forceinline__ float pen_s(float x, int cnt, const FRow& r) {
  x = (x > 0.f) ? __fdiv_rn(x, r.rep) : __fmul_rn(x, r.rep);
  x = __fsub_rn(x, __fmul_rn(r.freq, (float)cnt));
  return __fsub_rn(x, r.pres);
}
// smallest y whose processed value reaches vt (ylo_for), out of line; warp-wide
__device__ __noinline__ float ylo_s(float vt, float T, bool greedy) {
  RowCfg c{};
  c.T = T;
  c.greedy = greedy;
  return ylo_for(vt, c);
}

// per-warp candidate state (uniform across the warp)
struct FWarp {
  unsigned long long* buf;
  int wc;         // entries in buf
  uint32_t tkey;  // processed-key bound this warp knows (the CTA's, or its own)
  float th;       // smallest pre-temperature value reaching it: the filter
  bool ovf;       // ties filled the list: the part cannot be decided from it
};
struct FBound {
  uint32_t tkey;
  float th;
};

// the part's bound as published by all warps, and this warp's own, whichever is higher
__device__ __forceinline__ FBound fw_merge(FBound b, FSlot* L) {
  uint32_t tk = 0u, tr = 0u;
  if ((threadIdx.x & 31) == 0) {
    tk = *reinterpret_cast<volatile uint32_t*>(&L->thr_key);
    tr = *reinterpret_cast<volatile uint32_t*>(&L->thr_raw);
  }
  tk = __shfl_sync(FULLMASK, tk, 0);
  tr = __shfl_sync(FULLMASK, tr, 0);
  b.tkey = max(b.tkey, tk);
  b.th = fmaxf(b.th, from_okey(tr));
  return b;
}
__device__ __forceinline__ void fw_refresh(FWarp& W, FSlot* L) {
  const FBound b = fw_merge(FBound{W.tkey, W.th}, L);
  W.tkey = b.tkey;
  W.th = b.th;
}
// Publish a bound (out of line, rare): yk is a pre-temperature key that at least K distinct
// elements reach. Returns the warp's new bound. Warp-wide.
__device__ __noinline__ FBound fw_publish(uint32_t yk, FBound b, float T, bool greedy, FSlot* L) {
  const float y = from_okey(yk);
  const uint32_t v = okey(greedy ? y : __fdiv_rn(y, T));
  if (v > b.tkey) {
    const float th = ylo_s(from_okey(v), T, greedy);
    if ((threadIdx.x & 31) == 0) {
      atomicMax(&L->thr_key, v);
      atomicMax(&L->thr_raw, okey(th));
    }
    __syncwarp();
  }
  return fw_merge(b, L);
}
struct FTight {
  int wc;
  uint32_t tkey;
  float th;
};
// Raise the bound to the list's K-th largest entry and keep the entries that still pass the
// filter (out of line, rare). Warp-wide.
__device__ __noinline__ FTight fw_tighten(unsigned long long* buf, int wc, FBound b, int K,
                                          float T, bool greedy, FSlot* L) {
  const int lane = threadIdx.x & 31;
  constexpr int NK = FWB / 32;
  uint32_t k[NK];
#pragma unroll
  for (int i = 0; i < NK; ++i) {
    const int j = i * 32 + lane;
    k[i] = j < wc ? comp_key(buf[j]) : 0u;
  }
  const uint32_t yk = warp_kth_hi(k, K);
  if (yk != 0u) b = fw_publish(yk, b, T, greedy, L);
  const uint32_t keep_key = okey(b.th);
  int out = 0;
#pragma unroll
  for (int i = 0; i < NK; ++i) {
    const int j = i * 32 + lane;
    const bool keep = j < wc && k[i] >= keep_key;
    const unsigned long long e = keep ? buf[j] : 0ull;
    const unsigned m = __ballot_sync(FULLMASK, keep);
    if (keep) buf[out + __popc(m & ((1u << lane) - 1u))] = e;
    out += __popc(m);
  }
  __syncwarp();
  return FTight{out, b.tkey, b.th};
}
__device__ __forceinline__ int fw_trigger(int K) { return min(FWB - 32, max(2 * K + 32, FWB / 2)); }
__device__ __forceinline__ void fw_tighten_now(FWarp& W, const FRow& r, FSlot* L) {
  const FTight t = fw_tighten(W.buf, W.wc, FBound{W.tkey, W.th}, r.K, r.T, r.greedy, L);
  W.wc = t.wc;
  W.tkey = t.tkey;
  W.th = t.th;
}
// one scalar element per lane (ok): its pre-temperature value y and id; warp-wide
template <bool SUM>
__device__ __forceinline__ void fw_scalar(FWarp& W, const FRow& r, FSlot* L, bool ok, float y,
                                          int gid, float& m_t, float& s_t) {
  ok = ok && y >= -FLT_MAX;  // -inf has no mass and is never a candidate; NaN neither
  if (SUM && ok) {
    if (y > m_t) {
      s_t *= ex2((m_t - y) * r.c2);
      m_t = y;
    }
    s_t += ex2((y - m_t) * r.c2);
  }
  bool want = ok && y >= W.th;
  unsigned m = __ballot_sync(FULLMASK, want);
  if (!m) return;
  if (W.wc + __popc(m) > fw_trigger(r.K)) {
    fw_tighten_now(W, r, L);
    want = want && y >= W.th;
    m = __ballot_sync(FULLMASK, want);
  }
  if (W.wc + __popc(m) > FWB) {
    W.ovf = true;
    return;
  }
  const int lane = threadIdx.x & 31;
  if (want) W.buf[W.wc + __popc(m & ((1u << lane) - 1u))] = comp(okey(y), gid);
  __syncwarp();
  W.wc += __popc(m);
}

// Post this warp's lane values for the part's first bound and count the warp in; with
// `wait`, wait (bounded) for all warps and raise the bound to the K-th largest posted value.
__device__ __noinline__ void fw_post(FSlot* L, uint32_t lk) {
  const int lane = threadIdx.x & 31, w = threadIdx.x >> 5;
  L->fmax[w * 32 + lane] = lk;
  __syncwarp();
  if (lane == 0) {
    __threadfence_block();
    atomicAdd(&L->nfirst, 1);
  }
  __syncwarp();
}
__device__ __noinline__ FBound fw_first_wait(FSlot* L, FBound b, int K, float T, bool greedy) {
  const int lane = threadIdx.x & 31;
  int ready = 0;
  if (lane == 0) {
    for (int it = 0; it < (1 << 16); ++it) {
      if (*reinterpret_cast<volatile int*>(&L->nfirst) >= FW) {
        ready = 1;
        break;
      }
      __nanosleep(32);
    }
    __threadfence_block();
  }
  // a warp that gave up keeps its own bound (a looser filter, never a wrong one)
  if (!__shfl_sync(FULLMASK, ready, 0)) return b;
  uint32_t ka[FW];
#pragma unroll
  for (int i = 0; i < FW; ++i) ka[i] = *reinterpret_cast<volatile uint32_t*>(&L->fmax[i * 32 + lane]);
  const uint32_t va = warp_kth_hi(ka, K);
  if (va != 0u) b = fw_publish(va, b, T, greedy, L);
  return b;
}
__device__ __forceinline__ void fw_first_bound(FWarp& W, const FRow& r, FSlot* L, uint32_t lk) {
  fw_post(L, lk);
  const FBound b = fw_first_wait(L, FBound{W.tkey, W.th}, r.K, r.T, r.greedy);
  W.tkey = b.tkey;
  W.th = b.th;
}

// ---- one tile (one consumer warp) ----------------------------------------------------------------
template <typename TIn, bool SUM>
__device__ __forceinline__ void fused_tile(const KParams& P, FSlot* L, const FRow& r, bool first,
                                           FWarp& W, float& m_t, float& s_t, unsigned char* st,
                                           const FTileGeo& t, int row, int tloc) {
  using E = Elem<TIn>;
  constexpr int A = E::A;
  const int lane = threadIdx.x & 31;
  const int ibase = t.e0 + t.hoff;  // local element of the stage's first element
  const int* hid = L->hid + L->hbase;
  const int* hcnt = L->hcnt + L->hbase;
  // 1. penalised tokens inside the tile's interior: exact values, then masked in the stage
  if (r.pen && t.nv > 0) {
    const int lo = ibase, hi = ibase + t.nv * A;
    const int kb = L->hoff[tloc], ke = L->hoff[tloc + 1];
    for (int k0 = kb; k0 < ke; k0 += 32) {
      const int k = k0 + lane;
      bool ok = false;
      float y = 0.f;
      int li = 0;
      if (k < ke) {
        li = (int)((int64_t)hid[k] - P.voff);
        const int cn = hcnt[k];
        if (li >= lo && li < hi && cn > 0) {
          const int si = li - ibase;
          const float x = E::sm(st, si);
          E::neg_inf(st, si);
          // penalties that only lower values cannot lift a token below the filter
          ok = SUM || !r.pen_down || x >= W.th;
          if (ok) y = pen_s(x, cn, r);
        }
      }
      fw_scalar<SUM>(W, r, L, ok, y, (int)(P.voff + li), m_t, s_t);
    }
    __syncwarp();
  }
  // 2. ragged elements around the interior (any alignment): direct loads, explicit lookups
  {
    const int tail0 = t.hoff + t.nv * A;
    const int nhd = t.hoff, ntl = (t.e1 - t.e0) - tail0;
    if (nhd + ntl > 0) {
      const bool ok = lane < nhd + ntl;
      const int li = t.e0 + (lane < nhd ? lane : tail0 + (lane - nhd));
      float y = 0.f;
      if (ok) {
        y = E::ld((const TIn*)P.logits + (int64_t)row * P.ld, li);
        if (r.pen) {
          const int p = lower_bound_smem(hid, L->nh, P.voff + li);
          if (p < L->nh && (int64_t)hid[p] == P.voff + li && hcnt[p] > 0)
            y = pen_s(y, hcnt[p], r);
        }
      }
      fw_scalar<SUM>(W, r, L, ok, y, (int)(P.voff + li), m_t, s_t);
    }
  }
  // 3. the vectors: FVPL per lane
  const uint4* sv = reinterpret_cast<const uint4*>(st);
  float vm[FVPL];
  float lmax = -INFINITY;
#pragma unroll
  for (int i = 0; i < FVPL; ++i) {
    const int j = i * 32 + lane;
    vm[i] = -INFINITY;
    if (j < t.nv) {
      const uint4 q = sv[j];
      vm[i] = E::vmax(q);
      if (SUM && vm[i] >= -FLT_MAX) {  // online softmax sum (masked elements add nothing)
        if (vm[i] > m_t) {
          s_t *= ex2((m_t - vm[i]) * r.c2);
          m_t = vm[i];
        }
#pragma unroll
        for (int e = 0; e < A; ++e) s_t += ex2((E::at(q, e) - m_t) * r.c2);
      }
    }
    lmax = fmaxf(lmax, vm[i]);
  }
  if (first && r.K <= FKF) {
    // The part's first bound: the K-th largest of the lanes' maxima of every warp's first tile
    // (256 values, each the largest of 128 elements, K distinct elements reach it), so the
    // first tile is filtered with a bound from eight tiles' worth of elements. Every warp
    // posts its lanes' maxima and waits for the others (warps without a tile in the part post
    // nothing and count at once), then takes the K-th itself.
    const uint32_t lk = lmax >= -FLT_MAX ? okey(lmax) : 0u;
    fw_first_bound(W, r, L, lk);
    if (W.th == -FLT_MAX) {
      // too few posted values for K (a part of one or two tiles): the K-th largest of this
      // warp's own vector maxima
      uint32_t kk[FVPL];
#pragma unroll
      for (int i = 0; i < FVPL; ++i) kk[i] = vm[i] >= -FLT_MAX ? okey(vm[i]) : 0u;
      const uint32_t vr = warp_kth_hi(kk, r.K);
      if (vr != 0u) {
        const FBound bb = fw_publish(vr, FBound{W.tkey, W.th}, r.T, r.greedy, L);
        W.tkey = bb.tkey;
        W.th = bb.th;
      }
    }
  }
  // 4. the elements of the vectors whose maximum reaches the filter (read again from the stage;
  // penalised elements are -inf there) become candidates
  if (!__any_sync(FULLMASK, lmax >= W.th)) return;
  uint32_t vbits = 0u;  // vectors that reach the filter
  int n = 0;            // their elements that do
#pragma unroll
  for (int i = 0; i < FVPL; ++i) {
    if (vm[i] >= W.th) {
      vbits |= 1u << i;
      const uint4 q = sv[i * 32 + lane];
#pragma unroll
      for (int e = 0; e < A; ++e) n += E::at(q, e) >= W.th ? 1 : 0;
    }
  }
  int tot;
  int pos = warp_excl(n, &tot);
  if (W.wc + tot > fw_trigger(r.K)) {
    fw_tighten_now(W, r, L);
    vbits = 0u;
    n = 0;
#pragma unroll
    for (int i = 0; i < FVPL; ++i) {
      if (vm[i] >= W.th) {
        vbits |= 1u << i;
        const uint4 q = sv[i * 32 + lane];
#pragma unroll
        for (int e = 0; e < A; ++e) n += E::at(q, e) >= W.th ? 1 : 0;
      }
    }
    pos = warp_excl(n, &tot);
  }
  if (W.wc + tot > FWB) {
    // the list cannot take this tile (a weak bound, and fewer than K entries to tighten on):
    // raise the bound to the K-th largest of this tile's own vector maxima
    uint32_t kk[FVPL];
#pragma unroll
    for (int i = 0; i < FVPL; ++i) kk[i] = vm[i] >= -FLT_MAX ? okey(vm[i]) : 0u;
    const uint32_t vr = warp_kth_hi(kk, r.K);
    if (vr != 0u) {
      const FBound bb = fw_publish(vr, FBound{W.tkey, W.th}, r.T, r.greedy, L);
      W.tkey = bb.tkey;
      W.th = bb.th;
      fw_tighten_now(W, r, L);  // the list's entries below the raised filter go
      vbits = 0u;
      n = 0;
#pragma unroll
      for (int i = 0; i < FVPL; ++i) {
        if (vm[i] >= W.th) {
          vbits |= 1u << i;
          const uint4 q = sv[i * 32 + lane];
#pragma unroll
          for (int e = 0; e < A; ++e) n += E::at(q, e) >= W.th ? 1 : 0;
        }
      }
      pos = warp_excl(n, &tot);
    }
    if (W.wc + tot > FWB) {
      W.ovf = true;
      return;
    }
  }
  pos += W.wc;
  const float th = W.th;
  const int gbase = (int)(P.voff + ibase) + lane * A;
  while (vbits) {  // this lane's vectors, lowest first
    const int i = __ffs(vbits) - 1;
    vbits &= vbits - 1u;
    const uint4 q = sv[i * 32 + lane];
    const int gid0 = gbase + i * 32 * A;
#pragma unroll
    for (int e = 0; e < A; ++e) {
      const float y = E::at(q, e);
      if (y >= th) W.buf[pos++] = comp(okey(y), gid0 + e);
    }
  }
  __syncwarp();
  W.wc += tot;
}

// ---- part geometry ---------------------------------------------------------------------------------
struct FPartGeo {
  int row, j0, j1;
  int64_t g1;  // the part's end (global tile)
};
__device__ __forceinline__ FPartGeo fpart(const KParams& P, int64_t g, int64_t g1) {
  FPartGeo q;
  q.row = (int)(g / P.ntr);
  q.j0 = (int)(g - (int64_t)q.row * P.ntr);
  q.j1 = (int)min((int64_t)P.ntr, (int64_t)q.j0 + (g1 - g));
  q.g1 = g + (q.j1 - q.j0);
  return q;
}
struct FPart {
  RowCfg c;
  int K, mode;
  bool pen, exact, pen_down;
};
__device__ __forceinline__ FPart fpart_cfg(const KParams& P, const FSlot& L) {
  FPart pt;
  pt.c = cfg_from(P, L.prm);
  const RowCfg& c = pt.c;
  pt.exact = c.exact || (c.topk && c.k > FKF) || L.exact;
  pt.K = c.greedy ? 1 : c.K;
  pt.mode = (c.bad || pt.exact) ? FM_SKIP : (c.need_sum ? FM_SUM : FM_CANDS);
  pt.pen = c.pen && pt.mode != FM_SKIP;
  // penalties that never raise a value (repetition >= 1, presence and frequency >= 0)
  pt.pen_down = c.rep >= 1.f && c.pres >= 0.f && c.freq >= 0.f;
  return pt;
}

// ---- the producer: a part's slot, then the part's tiles -------------------------------------------
template <typename TIn>
__device__ void fused_prepare(const KParams& P, FSmem& S, FSlot& L, const FPartGeo& q,
                              uint32_t& hphase) {
  const int lane = threadIdx.x & 31;
  __syncwarp();
  if (lane < 8) L.prm[lane] = load_param(P, q.row, lane);
  int64_t a = 0, b = 0;
  if (P.hrow) {
    a = __ldg(P.hrow + q.row);
    b = __ldg(P.hrow + q.row + 1);
  }
  if (lane == 0) {
    L.thr_key = okey(-FLT_MAX);
    L.thr_raw = okey(-FLT_MAX);
    L.exact = 0;
    L.nh = 0;
    L.hbase = 0;
    L.nfirst = 0;
  }
  __syncwarp();
  const RowCfg c = cfg_from(P, L.prm);
  const bool pen = c.pen && !c.bad && !c.exact && !(c.topk && c.k > FKF);
  if (!pen) {
    __syncwarp();
    return;
  }
  const int64_t lo = P.voff + (int64_t)q.j0 * P.te, hi = P.voff + min(P.V, (int64_t)q.j1 * P.te);
  int64_t ia = a, ib = b;
  if (b - a > FHCAP) {  // only this part's entries
    ia = warp_lower_bound(P.hids, a, b, lo, lane);
    ib = warp_lower_bound(P.hids, ia, b, hi, lane);
  }
  const int nh = (int)(ib - ia);
  if (nh > FHCAP) {  // too many to stage: the row takes the exact search
    if (lane == 0) L.exact = 1;
    __syncwarp();
    return;
  }
  // the entries [ia, ib): the 16-byte aligned middle by two bulk copies, the ragged ends (at
  // most three entries each) by plain loads; staged at hid[hbase ...] so that the middle lands
  // 16-byte aligned. Unaligned arrays, or too few entries for a middle: plain loads only.
  const int64_t m0 = (ia + 3) & ~(int64_t)3, m1 = ib & ~(int64_t)3;
  const bool bulk = m1 > m0 && ((uintptr_t)P.hids & 15u) == 0 && ((uintptr_t)P.hcnt & 15u) == 0;
  const int hbase = bulk ? (int)(4 - (m0 - ia)) & 3 : 0;
  if (bulk) {
    const uint32_t bytes = (uint32_t)((m1 - m0) * 4);
    if (lane == 0) {
      mbar_arrive_tx(&S.hbar, 2u * bytes);
      bulk_load(L.hid + hbase + (m0 - ia), P.hids + m0, bytes, &S.hbar);
      bulk_load(L.hcnt + hbase + (m0 - ia), P.hcnt + m0, bytes, &S.hbar);
    }
    const int64_t nhead = m0 - ia, ntail = ib - m1;  // each at most 3
    if (lane < nhead) {
      L.hid[hbase + lane] = __ldg(P.hids + ia + lane);
      L.hcnt[hbase + lane] = __ldg(P.hcnt + ia + lane);
    } else if (lane >= 4 && lane - 4 < ntail) {
      const int64_t k = m1 + (lane - 4);
      L.hid[hbase + (k - ia)] = __ldg(P.hids + k);
      L.hcnt[hbase + (k - ia)] = __ldg(P.hcnt + k);
    }
    fwait(P, S, &S.hbar, hphase);
    hphase ^= 1u;
  } else {
    for (int k = lane; k < nh; k += 32) {
      L.hid[k] = __ldg(P.hids + ia + k);
      L.hcnt[k] = __ldg(P.hcnt + ia + k);
    }
  }
  __syncwarp();
  // first staged entry of each tile of the part (the last slot: the part's end)
  const int nt = q.j1 - q.j0;
  for (int k = lane; k <= nt; k += 32) {
    int64_t id = hi;
    if (k < nt) {
      const FTileGeo t = ftile<TIn>(P, q.row, q.j0 + k);
      id = P.voff + t.e0;
    }
    L.hoff[k] = lower_bound_smem(L.hid + hbase, nh, id);
  }
  if (lane == 0) {
    L.hbase = hbase;
    L.nh = nh;
  }
  __syncwarp();
}

template <typename TIn>
__device__ void fused_producer(const KParams& P, FSmem& S) {
  const int64_t g0 = ftile0(P, blockIdx.x), g1 = ftile0(P, blockIdx.x + 1);
  if ((threadIdx.x & 31) != 0) return;
  int row = -1;
  int64_t rbase = 0;
  for (int64_t g = g0; g < g1; ++g) {
    const int i = (int)(g - g0);
    const int s = i % FSTAGES;
    if (!fwait(P, S, &S.empty[s], ((uint32_t)(i / FSTAGES) & 1u) ^ 1u)) return;
    if (row < 0 || g - rbase >= P.ntr) {
      row = (int)(g / P.ntr);
      rbase = (int64_t)row * P.ntr;
    }
    const FTileGeo t = ftile<TIn>(P, row, (int)(g - rbase));
    mbar_arrive_tx(&S.full[s], t.bytes);
    if (t.bytes) bulk_load(S.stage[s], t.src, t.bytes, &S.full[s]);
  }
}

// The prep warp: each part's slot, ahead of the consumers (a slot is reused once the part
// FNSLOT earlier in the range is finished).
template <typename TIn>
__device__ void fused_prep(const KParams& P, FSmem& S) {
  const int lane = threadIdx.x & 31;
  const int64_t g0 = ftile0(P, blockIdx.x), g1 = ftile0(P, blockIdx.x + 1);
  uint32_t hphase = 0u;
  int p = 0;
  int64_t g = g0;
  while (g < g1) {
    const FPartGeo q = fpart(P, g, g1);
    const int sl = p % FNSLOT;
    if (p >= FNSLOT &&
        !fwait(P, S, &S.done[sl], (uint32_t)((p - FNSLOT) / FNSLOT) & 1u))
      return;
    fused_prepare<TIn>(P, S, S.slot[sl], q, hphase);
    if (lane == 0) {
      __threadfence_block();
      mbar_arrive(&S.ready[sl]);
    }
    g = q.g1;
    ++p;
  }
}

// ---- the consumers ----------------------------------------------------------------------------------
template <typename TIn>
__device__ void fused_consume(const KParams& P, FSmem& S) {
  const int lane = threadIdx.x & 31, w = threadIdx.x >> 5;
  const int64_t g0 = ftile0(P, blockIdx.x), g1 = ftile0(P, blockIdx.x + 1);
  int p = 0;
  int64_t g = g0;
  while (g < g1) {
    const FPartGeo q = fpart(P, g, g1);
    const int sl = p % FNSLOT;
    FSlot& L = S.slot[sl];
    fwait(P, S, &S.ready[sl], (uint32_t)(p / FNSLOT) & 1u);
    const FPart pt = fpart_cfg(P, L);
    FRow r;
    r.T = pt.c.T;
    r.c2 = pt.c.c2;
    r.rep = pt.c.rep;
    r.pres = pt.c.pres;
    r.freq = pt.c.freq;
    r.K = pt.K;
    r.greedy = pt.c.greedy;
    r.pen = pt.pen;
    r.pen_down = pt.pen_down;
    FWarp W;
    W.buf = S.wbuf[sl][w];
    W.wc = 0;
    W.tkey = okey(-FLT_MAX);
    W.th = -FLT_MAX;
    W.ovf = false;
    float m_t = -FLT_MAX, s_t = 0.f;
    // this warp's tiles of the part: range index i with i % FW == w
    const int ib = (int)(g - g0), ie = (int)(q.g1 - g0);
    const int i0 = ib + ((w - ib) % FW + FW) % FW;
    // without a tile here, count in for the part's first bound at once
    if (i0 >= ie && pt.mode != FM_SKIP && pt.K <= FKF) fw_post(&L, 0u);
    bool first = true;
    for (int i = i0; i < ie; i += FW) {
      const int s = i % FSTAGES;
      const bool landed = fwait(P, S, &S.full[s], (uint32_t)(i / FSTAGES) & 1u);
      if (landed && pt.mode != FM_SKIP) {
        const int j = q.j0 + (i - ib);
        const FTileGeo t = ftile<TIn>(P, q.row, j);
        fw_refresh(W, &L);
        if (pt.mode == FM_SUM)
          fused_tile<TIn, true>(P, &L, r, first, W, m_t, s_t, S.stage[s], t, q.row, j - q.j0);
        else
          fused_tile<TIn, false>(P, &L, r, first, W, m_t, s_t, S.stage[s], t, q.row, j - q.j0);
        // the masks were generic-proxy writes; the next bulk copy into this stage is an
        // async-proxy write
        if (pt.pen) asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
        first = false;
      }
      __syncwarp();
      if (lane == 0) mbar_arrive(&S.empty[s]);
    }
    // hand the part to the finisher
    if (pt.mode == FM_SUM) {
      float m = m_t;
#pragma unroll
      for (int o = 16; o > 0; o >>= 1) m = fmaxf(m, __shfl_xor_sync(FULLMASK, m, o));
      float sm = (m_t == -FLT_MAX) ? 0.f : s_t * ex2((m_t - m) * r.c2);
#pragma unroll
      for (int o = 16; o > 0; o >>= 1) sm += __shfl_xor_sync(FULLMASK, sm, o);
      if (lane == 0) {
        L.wm[w] = m;
        L.wsum[w] = sm;
      }
    }
    if (lane == 0) {
      L.wc[w] = W.wc;
      L.wovf[w] = W.ovf ? 1 : 0;
      __threadfence_block();
      mbar_arrive(&S.handed[sl]);
    }
    g = q.g1;
    ++p;
  }
}

// push a row to the deferred queue (searched exactly once streaming is over). A slot holds
// row + 1; 0 marks a slot not yet written (or already taken).
__device__ __forceinline__ void fdefer(const KParams& P, int row) {
  const int i = atomicAdd(P.queue, 1);
  atomicExch(P.queue + FQ_HDR + i, row + 1);
}

// ---- the finishing arithmetic for up to 32 * NPL sorted entries (one warp) ---------------------
template <int NPL>
__device__ __forceinline__ float pick(const float (&a)[NPL], int i) {
  float r = a[0];
#pragma unroll
  for (int k = 1; k < NPL; ++k) r = (i == k) ? a[k] : r;
  return r;
}
// finalize_warp's decisions with NPL entries per lane (lane l holds [l * NPL, (l + 1) * NPL));
// returns false when the row needs the exact search. Whole warp; every lane returns the same.
template <int NPL>
__device__ __forceinline__ bool finalize_warp_n(const KParams& P, const RowCfg& c, int row,
                                                const MergeIn m, const unsigned long long* e) {
  const int lane = threadIdx.x & 31;
  const int n = m.n;
  const float mv = from_okey(comp_key(e[0]));
  if (!(mv > -INFINITY) || !(mv <= FLT_MAX)) {
    if (lane == 0) {
      write_state(P, row, 3, -1, 0.f, 0.f, 0u, 0);
      status_or(P, VINFER_ST_NONFINITE);
    }
    return true;
  }
  const bool more = (m.flags & REC_UNRETAINED) != 0;
  int avail;
  if (c.topk) avail = (n >= c.K) ? count_ge(e, n, comp_key(e[c.K - 1])) : n;
  else avail = more ? count_ge(e, n, m.d_key) : n;
  float v[NPL], C[NPL];
  float loc = 0.f;
#pragma unroll
  for (int i = 0; i < NPL; ++i) {
    const int j = lane * NPL + i;
    v[i] = j < n ? from_okey(comp_key(e[j])) : -INFINITY;
    loc += j < avail ? ex2((v[i] - mv) * LOG2E) : 0.f;
    C[i] = loc;  // inclusive, lane-local
  }
  float inc = loc;
#pragma unroll
  for (int o = 1; o < 32; o <<= 1) {
    const float t = __shfl_up_sync(FULLMASK, inc, o);
    if (lane >= o) inc += t;
  }
  const float pre = inc - loc;
#pragma unroll
  for (int i = 0; i < NPL; ++i) C[i] += pre;
  const float total = __shfl_sync(FULLMASK, inc, 31);
  float Ssum = c.topk ? total : m.s;
  if (!c.topk && vf(m.m_y, c) != mv) Ssum *= ex2(m.m_y * c.c2 - mv * LOG2E);
  const bool listed_all = c.topk || !more;
  // first index whose flag is set (ascending), -1 when none
  auto first = [&](const bool (&f)[NPL]) -> int {
    int mine = -1;
#pragma unroll
    for (int i = NPL - 1; i >= 0; --i)
      if (f[i]) mine = i;
    const unsigned b = __ballot_sync(FULLMASK, mine >= 0);
    if (!b) return -1;
    const int l = __ffs(b) - 1;
    return l * NPL + __shfl_sync(FULLMASK, mine, l);
  };
  int L = 0x7FFFFFFF;
  if (c.topk) L = avail;
  else if (!more) L = n;
  bool cut_beyond = false;
  if (c.p < 1.f) {  // top-p: keep tokens whose mass strictly before them is < top_p
    const float t = c.p * Ssum;
    bool f[NPL];
#pragma unroll
    for (int i = 0; i < NPL; ++i) f[i] = lane * NPL + i < avail && C[i] >= t;
    const int h = first(f);
    if (h >= 0) L = min(L, h + 1);
    else if (!listed_all) cut_beyond = true;
  }
  if (c.minp > 0.f) {  // min-p: keep tokens with exp(v - max) >= min_p
    bool f[NPL];
#pragma unroll
    for (int i = 0; i < NPL; ++i) f[i] = lane * NPL + i < avail && (v[i] - mv) * LOG2E < c.lm;
    const int h = first(f);
    if (h >= 0) L = min(L, max(h, 1));
    else if (!listed_all) cut_beyond = true;
  }
  const bool L_known = L <= avail;
  if (!L_known && cut_beyond) return false;
  float s_kept = Ssum;
  if (L_known) {
    const int last = L - 1;
    s_kept = __shfl_sync(FULLMASK, pick(C, last % NPL), last / NPL);
  }
  const int lim = L_known ? L : avail;
  const float t = c.u * s_kept;
  bool f[NPL];
#pragma unroll
  for (int i = 0; i < NPL; ++i) f[i] = lane * NPL + i < lim && C[i] > t;
  int j = first(f);
  if (j < 0) {
    if (L_known) j = L - 1;
    else return false;
  }
  if (lane == 0) {
    if (L_known)
      write_state(P, row, 0, comp_id(e[j]), mv, s_kept, comp_key(e[L - 1]), comp_id(e[L - 1]));
    else
      write_state(P, row, 1, comp_id(e[j]), mv, s_kept, 0u, 0);
  }
  return true;
}


// ---- the finisher: a part's record --------------------------------------------------------------
using FFinS = FSmem::Fin;
template <typename TIn>
__device__ __forceinline__ void row_finish(const KParams& P, FFinS& F, int row, const FPart& pt,
                                           int np);

// The part's record: its candidates at or above the final bound as processed keys, the K
// largest with the ties of the K-th (rows without top-k: the FSUMK largest), sorted; its
// completeness key; for rows without top-k the softmax maximum and sum. Counted on the row's
// counter; the CTA that completes the row finishes it. One warp.
template <typename TIn>
__device__ __forceinline__ void part_end(const KParams& P, FSmem& S, FFinS& F, FSlot& L,
                                         const unsigned long long* lists, const FPartGeo& q) {
  const int lane = threadIdx.x & 31;
  const FPart pt = fpart_cfg(P, L);
  const RowCfg& c = pt.c;
  FRow r{};
  r.T = c.T;
  r.greedy = c.greedy;
  const uint32_t tk = *reinterpret_cast<volatile uint32_t*>(&L.thr_key);
  const uint32_t rk = *reinterpret_cast<volatile uint32_t*>(&L.thr_raw);
  uint32_t flags = c.bad ? REC_BAD : 0u;
  if (pt.exact) flags |= REC_EXACT;
  uint32_t why = 0u;  // diagnostics: 1 a warp's list overflowed, 2 too many candidates, 4 ties
  for (int w = 0; w < FW; ++w)
    if (L.wovf[w]) {
      flags |= REC_OVERFLOW;
      why |= 1u;
    }
  int n = 0;  // candidates in F.srt
  uint32_t ck = tk;
  if (!(flags & (REC_BAD | REC_EXACT | REC_OVERFLOW))) {
    // 1. every list's entries at or above the final filter, as processed keys
    for (int w = 0; w < FW; ++w) {
      const unsigned long long* lst = lists + (size_t)w * FWB;
      const int wc = L.wc[w];
      for (int j0 = 0; j0 < wc; j0 += 32) {
        const int j = j0 + lane;
        const unsigned long long x = j < wc ? lst[j] : 0ull;
        const bool keep = j < wc && comp_key(x) >= rk;
        const unsigned m = __ballot_sync(FULLMASK, keep);
        const int pos = n + __popc(m & ((1u << lane) - 1u));
        if (keep && pos < FCAP) F.srt[pos] = comp(okey(vf_s(from_okey(comp_key(x)), r)), comp_id(x));
        n += __popc(m);
      }
    }
    __syncwarp();
    if (n > FCAP) {
      flags |= REC_OVERFLOW;
      why |= 2u;
    }
  }
  // 2. keep the K largest (and ties of the K-th), sorted
  int nrec = 0;
  if (!(flags & (REC_BAD | REC_EXACT | REC_OVERFLOW))) {
    const int Kk = pt.mode == FM_SUM ? FSUMK : pt.K;
    if (n > 128) {  // cut to the keys at or above the Kk-th largest, in place
      const uint32_t v = warp_kth_smem(F.srt, n, Kk);
      int o = 0;
      for (int j0 = 0; j0 < n; j0 += 32) {
        const int j = j0 + lane;
        const unsigned long long x = j < n ? F.srt[j] : 0ull;
        const bool keep = j < n && comp_key(x) >= v;
        const unsigned m = __ballot_sync(FULLMASK, keep);
        if (keep) F.srt[o + __popc(m & ((1u << lane) - 1u))] = x;
        o += __popc(m);
      }
      __syncwarp();
      n = o;
      ck = max(ck, v);
    }
    if (n > 128) {
      flags |= REC_OVERFLOW;  // ties of the Kk-th fill more than a record
      why |= 4u;
    } else {
      if (n <= 64) warp_sort_smem<2>(F.srt, n);
      else warp_sort_smem<4>(F.srt, n);
      nrec = n;
      if (n >= Kk) {
        const uint32_t kth = comp_key(F.srt[Kk - 1]);
        nrec = count_ge(F.srt, n, kth);
        ck = max(ck, kth);
      }
    }
  }
  // 3. the record; the row's counter
  const int64_t g_first = (int64_t)q.row * P.ntr;
  const int slot = (int)blockIdx.x - fcta_of(P, g_first);
  unsigned char* rec = P.recs + ((size_t)q.row * P.slots + slot) * FREC_STRIDE;
  unsigned long long* re = reinterpret_cast<unsigned long long*>(rec + sizeof(RecHdr));
  for (int j = lane; j < nrec; j += 32) re[j] = F.srt[j];
  if (lane == 0) {
    float m = -INFINITY, sm = 0.f;
    if (pt.mode == FM_SUM) {
      for (int w = 0; w < FW; ++w) m = fmaxf(m, L.wm[w]);
      if (m > -FLT_MAX)
        for (int w = 0; w < FW; ++w)
          if (L.wm[w] > -FLT_MAX) sm += L.wsum[w] * ex2((L.wm[w] - m) * c.c2);
    }
    RecHdr h;
    h.m_y = m;
    h.s = sm;
    h.t_key = ck;
    h.n = nrec;
    // elements of the part may be missing from the list below its completeness key
    h.flags = flags | ((ck > okey(-FLT_MAX)) ? REC_UNRETAINED : 0u);
    h.pad[0] = (int)why;
    h.pad[1] = n;
    h.pad[2] = 0;
    *reinterpret_cast<RecHdr*>(rec) = h;
  }
  __syncwarp();
  int np = 0;
  if (lane == 0) {
    __threadfence();
    const int nparts = fcta_of(P, g_first + P.ntr - 1) - fcta_of(P, g_first) + 1;
    const int old = atom_add_acq_rel(&P.counters[q.row], 1);
    np = (old == nparts - 1) ? nparts : 0;
  }
  np = __shfl_sync(FULLMASK, np, 0);
  if (np) {
    __threadfence();
    row_finish<TIn>(P, F, q.row, pt, np);
  }
}

// ---- a row's finish: merge its parts' records, cut and draw (or this rank's shard record) -----
// One warp (the finisher).
template <typename TIn>
__device__ __forceinline__ void row_finish(const KParams& P, FFinS& F, int row, const FPart& pt,
                                           int np) {
  const int lane = threadIdx.x & 31;
  const RowCfg& c = pt.c;
  const unsigned char* recs = P.recs + (size_t)row * P.slots * FREC_STRIDE;
  if (lane == 0) P.counters[row] = 0;  // ready for the next call (stream-ordered after this one)
  if (lane < np) {
    const RecHdr* h = reinterpret_cast<const RecHdr*>(recs + (size_t)lane * FREC_STRIDE);
    RecHdr r;
    r.m_y = __ldcg(&h->m_y);
    r.s = __ldcg(&h->s);
    r.t_key = __ldcg(&h->t_key);
    r.n = __ldcg(&h->n);
    r.flags = __ldcg(&h->flags);
    r.pad[0] = __ldcg(&h->pad[0]);
    r.pad[1] = __ldcg(&h->pad[1]);
    r.pad[2] = 0;
    F.ph[lane] = r;
  }
  __syncwarp();
  uint32_t fl = 0u, d = 0u;
  float m_y = -INFINITY;
  int tot = 0;
  for (int p = 0; p < np; ++p) {
    fl |= F.ph[p].flags;
    m_y = fmaxf(m_y, F.ph[p].m_y);
    if (F.ph[p].flags & REC_UNRETAINED) d = max(d, F.ph[p].t_key);
    if (lane == 0) F.poff[p] = tot;
    tot += F.ph[p].n;
  }
  if (lane == 0) F.poff[np] = tot;
  float s_y = 0.f;
  if (c.need_sum && m_y > -FLT_MAX)
    for (int p = 0; p < np; ++p)
      if (F.ph[p].m_y > -FLT_MAX) s_y += F.ph[p].s * ex2((F.ph[p].m_y - m_y) * c.c2);
  __syncwarp();
  const bool local = P.mode == 1;
  unsigned char* shard = local ? P.shard_out + (size_t)row * P.shard_stride : nullptr;
  if (fl & REC_BAD) {
    if (lane == 0) {
      if (local) {
        write_flag_hdr(reinterpret_cast<RecHdr*>(shard), REC_BAD, m_y, s_y);
      } else {
        write_state(P, row, 3, -1, 0.f, 0.f, 0u, 0);
        status_or(P, VINFER_ST_BAD_PARAM);
      }
    }
    return;
  }
  bool undecided = (fl & (REC_OVERFLOW | REC_EXACT)) != 0 || tot > FCAP;
  // why (diagnostics): 1 a part's lists overflowed, 2 a part needs the exact search, 4 too many
  // entries to merge, 8 the K-th misses a part's completeness key, 16 fewer than K entries
  uint32_t why = ((fl & REC_OVERFLOW) ? 1u : 0u) | ((fl & REC_EXACT) ? 2u : 0u) |
                 (tot > FCAP ? 4u : 0u);
  for (int p = 0; p < np; ++p) why |= (uint32_t)F.ph[p].pad[0] << 8;
  unsigned long long* e = F.srt;
  if (!undecided) {
    // every part's sorted entries into cand, then merged by rank into srt
    for (int idx = lane; idx < tot; idx += 32) {
      int p = 0;
      while (F.poff[p + 1] <= idx) ++p;
      const unsigned long long* src = reinterpret_cast<const unsigned long long*>(
          recs + (size_t)p * FREC_STRIDE + sizeof(RecHdr));
      F.cand[idx] = __ldcg(src + (idx - F.poff[p]));
    }
    __syncwarp();
    for (int idx = lane; idx < tot; idx += 32) {
      int p = 0;
      while (F.poff[p + 1] <= idx) ++p;
      const unsigned long long x = F.cand[idx];
      int rank = idx - F.poff[p];
      for (int o = 0; o < np; ++o)
        if (o != p) rank += lower_count(F.cand + F.poff[o], F.poff[o + 1] - F.poff[o], x);
      e[rank] = x;
    }
    __syncwarp();
  }
  const bool more = d != 0u;
  const int K = pt.K;
  // rows with top-k (and greedy rows): the K-th must reach every part's completeness key
  uint32_t kkey = 0u;
  int nk = tot;
  if (!undecided && (c.topk || c.greedy)) {
    if (tot >= K) {
      kkey = comp_key(e[K - 1]);
      nk = count_ge(e, tot, kkey);
      if (kkey < d) {
        undecided = true;
        why |= 8u;
      }
    } else if (d > okey(-FLT_MAX)) {
      undecided = true;
      why |= 16u;
    }
  }
  if (local) {  // this rank's shard record
    RecHdr* oh = reinterpret_cast<RecHdr*>(shard);
    unsigned long long* oe = reinterpret_cast<unsigned long long*>(shard + sizeof(RecHdr));
    if (undecided) {
      if (lane == 0) {
        write_flag_hdr(oh, REC_OVERFLOW, m_y, s_y);
        oh->pad[0] = (int)why;  // diagnostics only: why the shard's candidates do not decide
      }
      return;
    }
    // rows with top-k: the K largest and the ties of the K-th; rows without: as many of the
    // largest as the record holds (complete above the first one left out)
    int nr = nk;
    uint32_t tk2 = kkey;
    if (!(c.topk || c.greedy) && nr > P.shard_cap) {
      nr = P.shard_cap;
      tk2 = comp_key(e[nr]) + 1u;
    }
    const bool over = nr > P.shard_cap;
    const bool unret = more || nr < tot;
    for (int j = lane; j < min(nr, P.shard_cap); j += 32) oe[j] = e[j];
    if (lane == 0) {
      oh->m_y = m_y;
      oh->s = s_y;
      oh->n = over ? 0 : nr;
      oh->t_key = unret ? max(tk2, d) : 0u;
      oh->flags = over ? REC_OVERFLOW : (unret ? REC_UNRETAINED : 0u);
    }
    return;
  }
  if (!undecided) {
    if (tot == 0) {
      if (lane == 0) {
        write_state(P, row, 3, -1, 0.f, 0.f, 0u, 0);
        status_or(P, VINFER_ST_NONFINITE);
      }
      return;
    }
    if (c.greedy) {
      if (lane == 0) write_state(P, row, 2, comp_id(e[0]), 0.f, 0.f, 0u, 0);
      return;
    }
    MergeIn mi;
    mi.m_y = m_y;
    mi.s = s_y;
    mi.n = min(c.topk ? nk : tot, 256);
    mi.d_key = d;
    if (mi.n < tot) mi.d_key = max(mi.d_key, comp_key(e[mi.n]) + 1u);
    mi.flags = (more || mi.n < tot) ? REC_UNRETAINED : 0u;
    if (!(c.topk && nk > 256)) {
      const bool done = mi.n <= 64 ? finalize_warp_n<2>(P, c, row, mi, e)
                                   : finalize_warp_n<8>(P, c, row, mi, e);
      if (done) return;
    }
  }
  if (lane == 0) fdefer(P, row);
}

// ---- the finisher warps ---------------------------------------------------------------------------
// Finisher f takes the parts p with p % FNFIN == f, so FNFIN parts can be finished at once.
template <typename TIn>
__device__ void fused_finish(const KParams& P, FSmem& S, int f) {
  const int64_t g0 = ftile0(P, blockIdx.x), g1 = ftile0(P, blockIdx.x + 1);
  const int lane = threadIdx.x & 31;
  int p = 0;
  int64_t g = g0;
  while (g < g1) {
    const FPartGeo q = fpart(P, g, g1);
    if (p % FNFIN == f) {
      const int sl = p % FNSLOT;
      FSlot& L = S.slot[sl];
      if (fwait(P, S, &S.handed[sl], (uint32_t)(p / FNSLOT) & 1u))
        part_end<TIn>(P, S, S.fin[f], L, &S.wbuf[sl][0][0], q);
      __syncwarp();
      if (lane == 0) mbar_arrive(&S.done[sl]);
    }
    g = q.g1;
    ++p;
  }
  if (lane == 0) mbar_arrive(&S.fin_all);
}

// ---- the kernel ----------------------------------------------------------------------------------
template <typename TIn>
__global__ void __launch_bounds__(FNT, 1) k_fused(const __grid_constant__ KParams P) {
  extern __shared__ __align__(128) unsigned char smraw[];
  FSmem& S = *reinterpret_cast<FSmem*>(smraw);
  const int tid = threadIdx.x, w = tid >> 5;
  if (tid == 0) {
    for (int s = 0; s < FSTAGES; ++s) {
      mbar_init(&S.full[s], 1u);
      mbar_init(&S.empty[s], 1u);
    }
    for (int s = 0; s < FNSLOT; ++s) {
      mbar_init(&S.ready[s], 1u);
      mbar_init(&S.handed[s], (uint32_t)FW);
      mbar_init(&S.done[s], 1u);
    }
    mbar_init(&S.hbar, 1u);
    mbar_init(&S.fin_all, (uint32_t)FNFIN);
    S.abort_ = 0;
    asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
  }
  __syncthreads();
  if (w == FPROD) {
    fused_producer<TIn>(P, S);
    return;
  }
  if (w == FPREP) {
    fused_prep<TIn>(P, S);
    return;
  }
  if (w >= FFIN) {
    fused_finish<TIn>(P, S, w - FFIN);
    return;
  }
  fused_consume<TIn>(P, S);
  // ---- rows the records could not decide: the exact search, one row at a time per CTA, once
  // the finisher has queued this CTA's rows
  if (P.mode != 0) return;
  fwait(P, S, &S.fin_all, 0u);
  cbar();
  Smem& SX = *reinterpret_cast<Smem*>(S.stage[0]);
  for (;;) {
    if (tid == 0) {
      int got = -1;
      const int n = ld_acquire(P.queue);
      int cl = ld_acquire(P.queue + 1);
      while (cl < n) {
        const int prev = atomicCAS(P.queue + 1, cl, cl + 1);
        if (prev == cl) {
          // the pusher writes the slot right after counting it: a short bounded wait
          int v = 0;
          for (int spin = 0; spin < (1 << 20) && v == 0; ++spin) {
            v = ld_acquire(P.queue + FQ_HDR + cl);
            if (v == 0) __nanosleep(64);
          }
          if (v == 0) status_or(P, VINFER_ST_TIMEOUT);
          else atomicExch(P.queue + FQ_HDR + cl, 0);
          got = v - 1;
          break;
        }
        cl = prev;
      }
      S.claim = got;
    }
    cbar();
    const int row = S.claim;
    cbar();
    if (row < 0) break;
    const RowCfg c = load_row(P, row);
    exact_row<TIn>(P, c, row, SX, reinterpret_cast<unsigned char*>(SX.scratch));
    cbar();
  }
  if (tid == 0) {
    __threadfence();
    if (atom_add_acq_rel(P.queue + 2, 1) == P.geff - 1) {  // the last CTA: reset the queue
      P.queue[0] = 0;
      P.queue[1] = 0;
      P.queue[2] = 0;
    }
  }
}

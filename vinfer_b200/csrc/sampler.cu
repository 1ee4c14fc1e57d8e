// sampler.cu — fused token sampler for B200 (sm_100a).
//
// The path restated here is vinfer's reference sampler (src/vinfer/runtime/sampler.py:50-77):
// temperature, top-k (ties at the k-th value kept, :53-55), softmax (:56), top-p on the mass
// strictly before each token (:57-64), renormalisation, and one draw per row, extended with
// repetition / presence / frequency penalties, min-p and an inverse-CDF draw from a caller
// uniform. Tokens are ordered canonically: descending processed logit, ties by ascending id.
//
// Execution (one launch of k_sample per batch):
//   * Work items are (row, segment) pairs; a segment is <= 32 KiB of one row's logits. The grid
//     is persistent (two CTAs per SM): CTA b takes items b, b + grid, b + 2 grid, ...
//   * Each CTA has two producer warps and eight consumer warps. Producer warp p owns shared
//     stage p: it reads the row's parameters, finds the segment's slice of the row's sorted
//     history (warp-cooperative search), loads those entries and the unaligned edges, then
//     copies the 16-byte-aligned interior of the segment HBM -> shared memory with one TMA bulk
//     copy per 16 KiB on an mbarrier. Metadata for the next item is fetched before the stage
//     is free, so the consumers find each stage full when they get to it.
//   * Consumers take penalised tokens out of the staged copy (exact float32 side values), make
//     one pass computing per-thread maxima (plus an online softmax sum when top-k is off),
//     extract the K largest per-thread maxima per warp (K distinct elements, so their K-th
//     largest bounds the segment's K-th largest value from below), collect every element at or
//     above that bound, rank the candidates by counting and write the top K with all ties,
//     sorted, as the segment's record.
//   * The CTA that completes a row's last record (acq_rel atomic counter, result consumed one
//     item later so its latency is hidden) merges the row: sorted records -> merged by rank,
//     top-k, top-p and min-p cuts by prefix sums, and the draw. A row whose cut or draw lies
//     below what the records hold completely, or whose candidates overflowed, is finished by an
//     exact multi-pass search over the row (radix histograms of mass in 2^-44 fixed point, ties
//     resolved in id order) in the same CTA.
//
// All reductions run in a fixed order, so results are deterministic run to run.

#include <cuda_runtime.h>
#include <cuda_bf16.h>
#include <stdint.h>
#include <float.h>
#include <math.h>

#include <algorithm>
#include <mutex>

#include "vinfer_sampler.h"

namespace {

// ---------------------------------------------------------------------------------------------
// configuration
// ---------------------------------------------------------------------------------------------
constexpr int NCW = 8;                  // consumer warps
constexpr int NT = NCW * 32;            // consumer threads
constexpr int NSTAGE = 2;               // shared-memory stages
constexpr int NTHR = NT + 32;           // threads per CTA: consumers + one producer warp
constexpr int SEG_BYTES = 32768;        // largest segment held in a stage
constexpr int SBUF_BYTES = SEG_BYTES + 64;
constexpr int SIDE_CAP = 512;           // penalised tokens per segment
constexpr int SIDE_PER_LANE = SIDE_CAP / 32;
constexpr int CAND_CAP = 1024;          // entries of one record
constexpr int RUN_CAP = 2048;           // candidates held for the run being processed
constexpr int CTA_CAP = 320;            // resident CTAs assumed when sizing workspaces
constexpr int KMAX = 256;               // largest top-k served by the candidate path
constexpr int KC = 64;                  // candidates kept per segment when top-k is off
constexpr int MAX_NSEG = 64;
constexpr int MERGE_CAP = 2048;         // merged entries (input in cand, sorted copy in a stage)
constexpr int BM_WORDS = (SBUF_BYTES / 2 + 31) / 32 + 2;
constexpr float LOG2E = 1.4426950408889634f;
constexpr double FX_ONE = 17592186044416.0;      // 2^44: fixed-point unit of probability mass
constexpr long long WAIT_CYCLES = 4000000000LL;  // ~2 s at 2 GHz: bound on any wait
constexpr unsigned FULLMASK = 0xffffffffu;

static_assert(NT == 256, "block helpers assume 256 consumer threads");
static_assert(KMAX <= 8 * 32, "warp extraction covers at most 8 x 32 values");
static_assert(MERGE_CAP * 8 <= SEG_BYTES, "a stage holds the sorted merge");
static_assert((int64_t)VINFER_MAX_VOCAB * 4 <= (int64_t)MAX_NSEG * SEG_BYTES,
              "the largest float32 row fits MAX_NSEG segments");
static_assert(MERGE_CAP <= RUN_CAP, "the candidate buffer holds the merge input");
static_assert((size_t)VINFER_MAX_VOCAB / 8 <= (size_t)RUN_CAP * 8 + SEG_BYTES,
              "the exact search's row bitmap spans the candidate buffer and a stage");

// record flags
constexpr uint32_t REC_UNRETAINED = 1u;  // elements below t_key exist that are not listed
constexpr uint32_t REC_OVERFLOW = 2u;    // candidates did not fit: the row needs the exact search
constexpr uint32_t REC_BAD = 4u;         // invalid parameters
constexpr uint32_t REC_EXACT = 8u;       // the row is resolved by the exact search

struct RecHdr {
  float m_y;        // largest penalised logit of the source (pre-temperature)
  float s;          // sum of exp2((y - m_y) * log2(e) / T) over the source (top-k off only)
  uint32_t t_key;   // every element with key >= t_key is listed
  int32_t n;        // listed entries, sorted ascending by composite key (= canonical order)
  uint32_t flags;
  int32_t pad[3];
};
static_assert(sizeof(RecHdr) == 32, "record header is 32 bytes");

struct RowState {    // result description, read by the probabilities kernel
  float m_v;         // maximum processed logit
  float s_kept;      // mass of the kept set, relative to exp(v - m_v)
  uint32_t cut_key;  // kept: key > cut_key, or key == cut_key and id <= cut_id
  int32_t cut_id;
  int32_t kind;      // 0 = cut, 1 = keep all, 2 = greedy one-hot, 3 = no result
  int32_t token;
  int32_t pad[2];
};
static_assert(sizeof(RowState) == 32, "row state is 32 bytes");

constexpr size_t REC_STRIDE = sizeof(RecHdr) + 8 * CAND_CAP;

struct KParams {
  const void* logits;
  int64_t ld, V, voff, vtotal;
  int B, nseg, seg_len, mode;  // mode 0: finalize, 1: local (write shard records), 2: merge
  int total, grid;             // segments in the batch (B * nseg) and CTAs sharing them
  uint32_t flags;
  const float* temperature;
  const int* top_k;
  const float* top_p;
  const float* min_p;
  const float* rep;
  const float* pres;
  const float* freq;
  const int64_t* hrow;
  const int* hids;
  const int* hcnt;
  const float* uni;
  int* out_ids;
  float* out_probs;
  int* status;
  int* counters;
  RowState* rows;
  unsigned char* recs;
  unsigned char* shard_out;
  int shard_cap;
  size_t shard_stride;
};

struct __align__(16) Stage {
  unsigned char data[SBUF_BYTES];  // the segment; merge / exact search scratch afterwards
  int32_t side_id[SIDE_CAP];       // penalised tokens of the segment (global ids) ...
  int32_t side_cnt[SIDE_CAP];      // ... and their counts
  float prm[8];                    // T, top_p, min_p, rep, pres, freq, uniform, top_k (bits)
  int32_t ns;                      // side entries, -1 when more than SIDE_CAP
  int32_t pad[3];
};

struct __align__(16) Smem {
  Stage st[NSTAGE];
  unsigned long long cand[RUN_CAP];   // candidates of the run (composite keys); exact: bins
  float side_y[SIDE_CAP];             // penalised values of the current item
  uint32_t bitmap[BM_WORDS];          // penalised slots of the current item
  float ext[NT];                      // lane maxima extracted per warp
  unsigned long long bin_mass[256];   // exact search: radix bins
  uint32_t bin_cnt[256];
  RecHdr mh[MAX_NSEG];
  int moff[MAX_NSEG + 1];
  unsigned long long red64[NCW + 1];
  float redf[NCW + 1];
  int redi[NCW + 1];
  int sc[16];
  float sf[8];
  unsigned long long full[NSTAGE];
  unsigned long long empty[NSTAGE];
};

// scalar slots in Smem::sc / Smem::sf
enum { SC_NC = 0, SC_NRET, SC_TKEY, SC_LAST, SC_B, SC_J, SC_X0, SC_X1, SC_NQ, SC_RFL };
// run flags in Smem::sc[SC_RFL]
constexpr int RUN_OVER = 1;  // a side list or the candidate buffer overflowed
enum { SF_TH = 0, SF_YLO, SF_SK, SF_M };

// ---------------------------------------------------------------------------------------------
// small device helpers
// ---------------------------------------------------------------------------------------------
__device__ __forceinline__ uint32_t okey(float v) {
  // order-preserving key; -0 folds into +0 because they compare equal in the reference
  v = __fadd_rn(v, 0.0f);
  const uint32_t b = __float_as_uint(v);
  return (b & 0x80000000u) ? ~b : (b | 0x80000000u);
}
__device__ __forceinline__ float from_okey(uint32_t k) {
  return __uint_as_float((k & 0x80000000u) ? (k & 0x7FFFFFFFu) : ~k);
}
__device__ __forceinline__ float ex2(float x) {
  float r;
  asm("ex2.approx.ftz.f32 %0, %1;" : "=f"(r) : "f"(x));
  return r;
}
__device__ __forceinline__ unsigned long long comp(uint32_t key, int id) {
  return ((unsigned long long)(~key) << 32) | (uint32_t)id;  // ascending = canonical order
}
__device__ __forceinline__ uint32_t comp_key(unsigned long long c) { return ~(uint32_t)(c >> 32); }
__device__ __forceinline__ int comp_id(unsigned long long c) { return (int)(uint32_t)c; }

__device__ __forceinline__ uint32_t smem_u32(const void* p) {
  return (uint32_t)__cvta_generic_to_shared(p);
}
__device__ __forceinline__ void status_or(const KParams& P, uint32_t bits) {
  if (P.status) atomicOr(reinterpret_cast<unsigned int*>(P.status), bits);
}
// barrier of the consumer warps only (the producer warps run their own loop)
__device__ __forceinline__ void cbar() { asm volatile("bar.sync 1, %0;" ::"n"(NT) : "memory"); }
__device__ __forceinline__ bool cbar_or(bool p) {
  uint32_t r;
  asm volatile(
      "{\n .reg .pred a, b;\n setp.ne.u32 a, %1, 0;\n bar.red.or.pred b, 1, %2, a;\n"
      " selp.u32 %0, 1, 0, b;\n}\n"
      : "=r"(r)
      : "r"((uint32_t)p), "n"(NT)
      : "memory");
  return r != 0;
}
__device__ __forceinline__ int atom_add_acq_rel(int* p, int v) {
  int old;
  asm volatile("atom.acq_rel.gpu.global.add.s32 %0, [%1], %2;" : "=r"(old) : "l"(p), "r"(v)
               : "memory");
  return old;
}

// ---- TMA bulk copy (global -> shared) with an mbarrier, waits bounded -----------------------
__device__ __forceinline__ void mbar_init(unsigned long long* bar, uint32_t count) {
  asm volatile("mbarrier.init.shared::cta.b64 [%0], %1;" ::"r"(smem_u32(bar)), "r"(count)
               : "memory");
}
__device__ __forceinline__ void mbar_fence_init() {
  asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
}
__device__ __forceinline__ void mbar_arrive_expect_tx(unsigned long long* bar, uint32_t bytes) {
  asm volatile("mbarrier.arrive.expect_tx.shared::cta.b64 _, [%0], %1;" ::"r"(smem_u32(bar)),
               "r"(bytes)
               : "memory");
}
__device__ __forceinline__ void mbar_arrive(unsigned long long* bar) {
  asm volatile("mbarrier.arrive.shared::cta.b64 _, [%0];" ::"r"(smem_u32(bar)) : "memory");
}
__device__ __forceinline__ void tma_load_1d(void* dst, const void* src, uint32_t bytes,
                                            unsigned long long* bar) {
  asm volatile(
      "cp.async.bulk.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1], %2, [%3];" ::
          "r"(smem_u32(dst)),
      "l"(src), "r"(bytes), "r"(smem_u32(bar))
      : "memory");
}
__device__ __forceinline__ bool mbar_try_wait(unsigned long long* bar, uint32_t parity) {
  uint32_t ok;
  asm volatile(
      "{\n .reg .pred p;\n mbarrier.try_wait.parity.shared::cta.b64 p, [%1], %2;\n"
      " selp.u32 %0, 1, 0, p;\n}\n"
      : "=r"(ok)
      : "r"(smem_u32(bar)), "r"(parity)
      : "memory");
  return ok != 0;
}
// Wait for phase `parity` of `bar`, giving up after WAIT_CYCLES. Returns false on timeout.
// try_wait suspends the warp in hardware until the phase completes or a short time limit.
__device__ bool mbar_wait_bounded(unsigned long long* bar, uint32_t parity) {
  if (mbar_try_wait(bar, parity)) return true;
  const long long t0 = clock64();
  while (!mbar_try_wait(bar, parity)) {
    if (clock64() - t0 > WAIT_CYCLES) return false;
  }
  return true;
}

// ---- element access ---------------------------------------------------------------------------
template <typename T>
struct Elem;
template <>
struct Elem<float> {
  static constexpr int A = 4;  // elements per 16 bytes
  __device__ static float ld(const void* p, int64_t i) { return __ldg((const float*)p + i); }
  __device__ static uint32_t ldraw(const void* p, int64_t i) {
    return __ldg((const unsigned int*)p + i);
  }
  __device__ static void straw(void* s, int i, uint32_t v) { ((uint32_t*)s)[i] = v; }
  __device__ static float sm(const void* s, int i) { return ((const float*)s)[i]; }
  __device__ static void neg_inf(void* s, int i) { ((uint32_t*)s)[i] = 0xFF800000u; }
  __device__ static float vmax(const uint4& q) {
    return fmaxf(fmaxf(__uint_as_float(q.x), __uint_as_float(q.y)),
                 fmaxf(__uint_as_float(q.z), __uint_as_float(q.w)));
  }
  __device__ static float at(const uint4& q, int e) {
    const uint32_t w = e == 0 ? q.x : e == 1 ? q.y : e == 2 ? q.z : q.w;
    return __uint_as_float(w);
  }
};
template <>
struct Elem<__nv_bfloat16> {
  static constexpr int A = 8;
  __device__ static float ld(const void* p, int64_t i) {
    const unsigned short b = __ldg((const unsigned short*)p + i);
    return __uint_as_float((uint32_t)b << 16);
  }
  __device__ static uint32_t ldraw(const void* p, int64_t i) {
    return __ldg((const unsigned short*)p + i);
  }
  __device__ static void straw(void* s, int i, uint32_t v) {
    ((unsigned short*)s)[i] = (unsigned short)v;
  }
  __device__ static float sm(const void* s, int i) {
    return __uint_as_float((uint32_t)((const unsigned short*)s)[i] << 16);
  }
  __device__ static void neg_inf(void* s, int i) { ((unsigned short*)s)[i] = 0xFF80u; }
  __device__ static float vmax(const uint4& q) {
    const __nv_bfloat162 a = *reinterpret_cast<const __nv_bfloat162*>(&q.x);
    const __nv_bfloat162 b = *reinterpret_cast<const __nv_bfloat162*>(&q.y);
    const __nv_bfloat162 c = *reinterpret_cast<const __nv_bfloat162*>(&q.z);
    const __nv_bfloat162 d = *reinterpret_cast<const __nv_bfloat162*>(&q.w);
    const __nv_bfloat162 m = __hmax2(__hmax2(a, b), __hmax2(c, d));
    return fmaxf(__low2float(m), __high2float(m));
  }
  __device__ static float at(const uint4& q, int e) {
    const uint32_t w = (e >> 1) == 0 ? q.x : (e >> 1) == 1 ? q.y : (e >> 1) == 2 ? q.z : q.w;
    return __uint_as_float((e & 1) ? (w & 0xFFFF0000u) : (w << 16));
  }
};

// segment geometry: local index i lives at slot off + i of the stage buffer
struct Geo {
  int64_t lo, gbase;
  int n, head, inter, tail0, off, nvec, pad_end;
  const void* rowp;
};
template <typename TIn>
__device__ Geo geometry(const KParams& P, int row, int seg) {
  constexpr int A = Elem<TIn>::A;
  constexpr int ES = 16 / A;
  Geo g;
  g.lo = (int64_t)seg * P.seg_len;
  const int64_t hi = min(P.V, g.lo + (int64_t)P.seg_len);
  g.n = (int)(hi - g.lo);
  g.rowp = (const TIn*)P.logits + (int64_t)row * P.ld;
  const uintptr_t gaddr = (uintptr_t)((const TIn*)g.rowp + g.lo);
  g.head = (int)(((16u - (uint32_t)(gaddr & 15u)) & 15u) / ES);
  if (g.head > g.n) g.head = g.n;
  g.inter = (int)((((int64_t)(g.n - g.head) * ES) / 16) * 16 / ES);
  g.tail0 = g.head + g.inter;
  g.off = (A - g.head % A) % A;
  g.nvec = (g.off + g.n + A - 1) / A;
  g.pad_end = g.nvec * A - (g.off + g.n);
  g.gbase = P.voff + g.lo;
  return g;
}

// ---------------------------------------------------------------------------------------------
// per-row configuration
// ---------------------------------------------------------------------------------------------
struct RowCfg {
  float T, c2, p, minp, lm, rep, pres, freq, u;
  int k, K;
  bool greedy, topk, need_sum, pen, bad, exact;
};

__device__ RowCfg make_cfg(const KParams& P, float T, int k, float p, float minp, float rep,
                           float pres, float freq, float u) {
  RowCfg c;
  c.T = T;
  c.k = k;
  c.p = p;
  c.minp = minp;
  c.rep = rep;
  c.pres = pres;
  c.freq = freq;
  c.u = u;
  c.greedy = (T == 0.f);
  bool bad = !(T >= 0.f && T <= FLT_MAX) || !(p > 0.f && p <= 1.f) || k < 0 ||
             !(minp >= 0.f && minp <= 1.f) || !(rep > 0.f && rep <= FLT_MAX) ||
             !(fabsf(pres) <= FLT_MAX) || !(fabsf(freq) <= FLT_MAX);
  if (!c.greedy) bad = bad || P.uni == nullptr || !(u >= 0.f && u < 1.f);
  c.bad = bad;
  c.topk = !c.greedy && k > 0 && (int64_t)k < P.vtotal;
  c.K = c.greedy ? 1 : (c.topk ? k : KC);
  c.need_sum = !c.greedy && !c.topk;
  c.exact = (P.flags & VINFER_FLAG_EXACT_ALL) != 0 || (c.topk && k > KMAX);
  c.c2 = c.greedy ? 0.f : __fdiv_rn(LOG2E, T);
  c.lm = minp > 0.f ? log2f(minp) : -INFINITY;
  c.pen = P.hrow != nullptr && (rep != 1.f || pres != 0.f || freq != 0.f);
  return c;
}
// parameter `i` of a row: 0 T, 1 top_p, 2 min_p, 3 rep, 4 pres, 5 freq, 6 uniform, 7 top_k bits
__device__ float load_param(const KParams& P, int row, int i) {
  switch (i) {
    case 0: return P.temperature ? __ldg(P.temperature + row) : 1.f;
    case 1: return P.top_p ? __ldg(P.top_p + row) : 1.f;
    case 2: return P.min_p ? __ldg(P.min_p + row) : 0.f;
    case 3: return P.rep ? __ldg(P.rep + row) : 1.f;
    case 4: return P.pres ? __ldg(P.pres + row) : 0.f;
    case 5: return P.freq ? __ldg(P.freq + row) : 0.f;
    case 6: return P.uni ? __ldg(P.uni + row) : 0.f;
    default: return __int_as_float(P.top_k ? __ldg(P.top_k + row) : 0);
  }
}
__device__ RowCfg cfg_from(const KParams& P, const float* prm) {
  return make_cfg(P, prm[0], __float_as_int(prm[7]), prm[1], prm[2], prm[3], prm[4], prm[5],
                  prm[6]);
}
__device__ RowCfg load_row(const KParams& P, int row) {
  float prm[8];
#pragma unroll
  for (int i = 0; i < 8; ++i) prm[i] = load_param(P, row, i);
  return cfg_from(P, prm);
}

// penalties: repetition, then frequency * count, then presence; one IEEE op each
__device__ __forceinline__ float penalize(float x, int cnt, const RowCfg& c) {
  x = (x > 0.f) ? __fdiv_rn(x, c.rep) : __fmul_rn(x, c.rep);
  x = __fsub_rn(x, __fmul_rn(c.freq, (float)cnt));
  return __fsub_rn(x, c.pres);
}
// processed logit: true division by the temperature (the reference divides on CPU)
__device__ __forceinline__ float vf(float y, const RowCfg& c) {
  return c.greedy ? y : __fdiv_rn(y, c.T);
}
// first index >= target in the ascending ids[a, b) (one thread)
__device__ int64_t lower_bound_ids(const int* ids, int64_t a, int64_t b, int64_t target) {
  while (a < b) {
    const int64_t mid = a + (b - a) / 2;
    if ((int64_t)__ldg(ids + mid) < target) a = mid + 1; else b = mid;
  }
  return a;
}
// the same, by a whole warp: 32 probes per round, so about two dependent loads per search
__device__ int64_t warp_lower_bound(const int* ids, int64_t a, int64_t b, int64_t target,
                                    int lane) {
  while (b - a > 32) {
    const int64_t step = (b - a + 31) / 32;
    const int64_t p = a + lane * step;
    const bool lt = p < b && (int64_t)__ldg(ids + p) < target;
    const int c = __popc(__ballot_sync(FULLMASK, lt));
    if (c == 0) return a;
    const int64_t na = a + (int64_t)(c - 1) * step + 1;
    b = min(b, a + (int64_t)c * step);
    a = na;
  }
  const int64_t p = a + lane;
  const bool lt = p < b && (int64_t)__ldg(ids + p) < target;
  return a + __popc(__ballot_sync(FULLMASK, lt));
}

// ---------------------------------------------------------------------------------------------
// consumer-wide building blocks (all 256 consumer threads call them)
// ---------------------------------------------------------------------------------------------
__device__ float cta_excl_scan_f(float x, float* total, Smem& S) {
  const int lane = threadIdx.x & 31, w = threadIdx.x >> 5;
  float inc = x;
#pragma unroll
  for (int o = 1; o < 32; o <<= 1) {
    const float t = __shfl_up_sync(FULLMASK, inc, o);
    if (lane >= o) inc += t;
  }
  cbar();
  if (lane == 31) S.redf[w] = inc;
  cbar();
  if (threadIdx.x == 0) {
    float run = 0.f;
    for (int i = 0; i < NCW; ++i) {
      const float t = S.redf[i];
      S.redf[i] = run;
      run += t;
    }
    S.redf[NCW] = run;
  }
  cbar();
  *total = S.redf[NCW];
  return S.redf[w] + inc - x;
}
__device__ unsigned long long cta_excl_scan_u64(unsigned long long x, unsigned long long* total,
                                                Smem& S) {
  const int lane = threadIdx.x & 31, w = threadIdx.x >> 5;
  unsigned long long inc = x;
#pragma unroll
  for (int o = 1; o < 32; o <<= 1) {
    const unsigned long long t = __shfl_up_sync(FULLMASK, inc, o);
    if (lane >= o) inc += t;
  }
  cbar();
  if (lane == 31) S.red64[w] = inc;
  cbar();
  if (threadIdx.x == 0) {
    unsigned long long run = 0;
    for (int i = 0; i < NCW; ++i) {
      const unsigned long long t = S.red64[i];
      S.red64[i] = run;
      run += t;
    }
    S.red64[NCW] = run;
  }
  cbar();
  *total = S.red64[NCW];
  return S.red64[w] + inc - x;
}
__device__ int cta_excl_scan_i(int x, int* total, Smem& S) {
  const int lane = threadIdx.x & 31, w = threadIdx.x >> 5;
  int inc = x;
#pragma unroll
  for (int o = 1; o < 32; o <<= 1) {
    const int t = __shfl_up_sync(FULLMASK, inc, o);
    if (lane >= o) inc += t;
  }
  cbar();
  if (lane == 31) S.redi[w] = inc;
  cbar();
  if (threadIdx.x == 0) {
    int run = 0;
    for (int i = 0; i < NCW; ++i) {
      const int t = S.redi[i];
      S.redi[i] = run;
      run += t;
    }
    S.redi[NCW] = run;
  }
  cbar();
  *total = S.redi[NCW];
  return S.redi[w] + inc - x;
}
__device__ unsigned long long cta_min_u64(unsigned long long x, Smem& S) {
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) {
    const unsigned long long t = __shfl_xor_sync(FULLMASK, x, o);
    x = t < x ? t : x;
  }
  cbar();
  if ((threadIdx.x & 31) == 0) S.red64[threadIdx.x >> 5] = x;
  cbar();
  unsigned long long m = S.red64[0];
  for (int i = 1; i < NCW; ++i) m = S.red64[i] < m ? S.red64[i] : m;
  return m;
}
__device__ uint32_t cta_max_u32(uint32_t x, Smem& S) {
  return (uint32_t)~cta_min_u64(~(unsigned long long)x, S);
}
__device__ unsigned long long cta_sum_u64(unsigned long long x, Smem& S) {
  unsigned long long tot;
  cta_excl_scan_u64(x, &tot, S);
  return tot;
}

// ---------------------------------------------------------------------------------------------
// merge: records -> canonical order -> cuts and draw
// ---------------------------------------------------------------------------------------------
__device__ void write_flag_hdr(RecHdr* h, uint32_t flags, float m_y, float s) {
  h->m_y = m_y;
  h->s = s;
  h->t_key = 0;
  h->n = 0;
  h->flags = flags;
}

struct MergeIn {
  float m_y, s;
  uint32_t d_key;  // every element with key >= d_key is among the entries
  uint32_t flags;
  int n;
};

// number of entries of the ascending list e[0, n) below x
__device__ __forceinline__ int lower_count(const unsigned long long* e, int n,
                                           unsigned long long x) {
  int a = 0, b = n;
  while (a < b) {
    const int mid = (a + b) >> 1;
    if (e[mid] < x) a = mid + 1; else b = mid;
  }
  return a;
}

// Merge the sorted records of one row (nsrc sources at src0 + i * stride); the merged, sorted
// entries land in out[0, MERGE_CAP) (the record entries are staged in the candidate buffer).
__device__ MergeIn gather_sorted(const unsigned char* src0, size_t stride, int nsrc,
                                 const RowCfg& c, Smem& S, unsigned long long* out) {
  const int tid = threadIdx.x;
  unsigned long long* in = S.cand;
  if (tid < nsrc) {
    const RecHdr* h = (const RecHdr*)(src0 + (size_t)tid * stride);
    RecHdr r;
    r.m_y = __ldcg(&h->m_y);
    r.s = __ldcg(&h->s);
    r.t_key = __ldcg(&h->t_key);
    r.n = __ldcg(&h->n);
    r.flags = __ldcg(&h->flags);
    S.mh[tid] = r;
  }
  cbar();
  if (tid == 0) {
    float m_y = -INFINITY;
    for (int i = 0; i < nsrc; ++i) m_y = fmaxf(m_y, S.mh[i].m_y);
    float s = 0.f;
    uint32_t d = 0, fl = 0;
    int tot = 0;
    for (int i = 0; i < nsrc; ++i) {
      const RecHdr& h = S.mh[i];
      if (c.need_sum && h.m_y > -INFINITY) s += h.s * ex2((h.m_y - m_y) * c.c2);
      if (h.flags & REC_UNRETAINED) d = max(d, h.t_key);
      fl |= h.flags;
      S.moff[i] = tot;
      tot += h.n;
    }
    S.moff[nsrc] = tot;
    S.sf[SF_M] = m_y;
    S.sf[SF_SK] = s;
    S.sc[SC_X0] = (int)d;
    S.sc[SC_X1] = (int)fl;
  }
  cbar();
  MergeIn m;
  m.m_y = S.sf[SF_M];
  m.s = S.sf[SF_SK];
  m.d_key = (uint32_t)S.sc[SC_X0];
  m.flags = (uint32_t)S.sc[SC_X1];
  m.n = S.moff[nsrc];
  if ((m.flags & (REC_OVERFLOW | REC_BAD | REC_EXACT)) || m.n > MERGE_CAP) return m;
  for (int idx = tid; idx < m.n; idx += NT) {  // all sources at once: one round of loads
    int s = 0;
    while (S.moff[s + 1] <= idx) ++s;
    const unsigned long long* re =
        (const unsigned long long*)(src0 + (size_t)s * stride + sizeof(RecHdr));
    in[idx] = __ldcg(re + (idx - S.moff[s]));
  }
  cbar();
  for (int idx = tid; idx < m.n; idx += NT) {
    int s = 0;
    while (S.moff[s + 1] <= idx) ++s;
    const unsigned long long x = in[idx];
    int rank = idx - S.moff[s];
    for (int t = 0; t < nsrc; ++t) {
      if (t == s) continue;
      rank += lower_count(in + S.moff[t], S.moff[t + 1] - S.moff[t], x);
    }
    out[rank] = x;
  }
  cbar();
  return m;
}

// number of leading entries of the sorted e[0, n) whose key is >= key
__device__ int count_ge(const unsigned long long* e, int n, uint32_t key) {
  int a = 0, b = n;
  while (a < b) {
    const int mid = (a + b) / 2;
    if (comp_key(e[mid]) >= key) a = mid + 1; else b = mid;
  }
  return a;
}

__device__ void write_state(const KParams& P, int row, int kind, int token, float mv, float sk,
                            uint32_t ck, int cid) {
  P.out_ids[row] = token;
  RowState st = {};
  st.m_v = mv;
  st.s_kept = sk;
  st.cut_key = ck;
  st.cut_id = cid;
  st.kind = kind;
  st.token = token;
  P.rows[row] = st;
}

// Finalize one row from sorted entries e[0, m.n). Returns false when the row must take the
// exact search.
__device__ bool finalize_sorted(const KParams& P, const RowCfg& c, int row, const MergeIn& m,
                                const unsigned long long* e, Smem& S) {
  const int tid = threadIdx.x;
  if (m.n == 0) {
    if (tid == 0) {
      write_state(P, row, 3, -1, 0.f, 0.f, 0u, 0);
      status_or(P, VINFER_ST_NONFINITE);
    }
    return true;
  }
  if (c.greedy) {
    if (tid == 0) write_state(P, row, 2, comp_id(e[0]), 0.f, 0.f, 0u, 0);
    return true;
  }
  const float mv = from_okey(comp_key(e[0]));
  if (!(mv > -INFINITY) || !(mv <= FLT_MAX)) {
    if (tid == 0) {
      write_state(P, row, 3, -1, 0.f, 0.f, 0u, 0);
      status_or(P, VINFER_ST_NONFINITE);
    }
    return true;
  }
  int nk, avail;
  const bool more = (m.flags & REC_UNRETAINED) != 0;  // elements exist beyond the entries
  if (c.topk) {
    nk = (m.n >= c.K) ? count_ge(e, m.n, comp_key(e[c.K - 1])) : m.n;
    avail = nk;
  } else {
    avail = more ? count_ge(e, m.n, m.d_key) : m.n;
    nk = 0x7FFFFFFF;
  }
  // per-thread contiguous chunks of [0, avail), prefix sums of exp2((v - mv) * log2 e)
  const int chunk = (avail + NT - 1) / NT;
  const int j0 = min(avail, tid * chunk), j1 = min(avail, j0 + chunk);
  float loc = 0.f;
  for (int j = j0; j < j1; ++j) loc += ex2((from_okey(comp_key(e[j])) - mv) * LOG2E);
  float total;
  const float pre = cta_excl_scan_f(loc, &total, S);
  const float Ssum = c.topk ? total : m.s;
  const bool listed_all = c.topk || !more;  // every kept-by-top-k token is among the entries

  // first index in [0, lim) whose inclusive prefix C_j satisfies C_j >= t (ge) or C_j > t
  auto first_cross = [&](float t, bool ge, int lim) -> int {
    int hit = 0x7FFFFFFF;
    float run = pre;
    for (int j = j0; j < min(j1, lim); ++j) {
      run += ex2((from_okey(comp_key(e[j])) - mv) * LOG2E);
      if (ge ? (run >= t) : (run > t)) {
        hit = j;
        break;
      }
    }
    return (int)cta_min_u64((unsigned long long)(unsigned)hit, S);
  };

  // L = length of the kept prefix: the smallest bound known to lie within the entries
  int L = 0x7FFFFFFF;
  if (c.topk) L = nk;
  else if (!more) L = m.n;
  bool cut_beyond = false;  // an active cut lies beyond the listed entries
  if (c.p < 1.f) {  // top-p: keep tokens whose mass strictly before them is < top_p
    const int h = first_cross(c.p * Ssum, true, avail);
    if (h != 0x7FFFFFFF) L = min(L, h + 1);
    else if (!listed_all) cut_beyond = true;
  }
  if (c.minp > 0.f) {  // min-p: keep tokens with exp(v - max) >= min_p
    int hit = 0x7FFFFFFF;
    for (int j = j0; j < j1; ++j)
      if ((from_okey(comp_key(e[j])) - mv) * LOG2E < c.lm) {
        hit = j;
        break;
      }
    hit = (int)cta_min_u64((unsigned long long)(unsigned)hit, S);
    if (hit != 0x7FFFFFFF) L = min(L, max(hit, 1));
    else if (!listed_all) cut_beyond = true;
  }
  const bool L_known = L <= avail;
  if (!L_known && cut_beyond) return false;  // the cut needs elements the records do not hold
  // kept-set mass
  float s_kept;
  if (L_known) {
    const int last = L - 1;
    if (last >= j0 && last < j1) {
      float run = pre;
      for (int j = j0; j <= last; ++j) run += ex2((from_okey(comp_key(e[j])) - mv) * LOG2E);
      S.sf[SF_SK] = run;
    }
    cbar();
    s_kept = S.sf[SF_SK];
  } else {
    s_kept = Ssum;  // no cut at all: the kept set is every token
  }
  const int lim = L_known ? L : avail;
  int j = first_cross(c.u * s_kept, false, lim);
  if (j == 0x7FFFFFFF) {
    if (L_known) j = L - 1;
    else return false;
  }
  if (tid == 0) {
    if (L_known)
      write_state(P, row, 0, comp_id(e[j]), mv, s_kept, comp_key(e[L - 1]), comp_id(e[L - 1]));
    else
      write_state(P, row, 1, comp_id(e[j]), mv, s_kept, 0u, 0);
  }
  return true;
}

// ---------------------------------------------------------------------------------------------
// exact multi-pass search over one row (global memory), for rows the records cannot resolve
// ---------------------------------------------------------------------------------------------
// penalised-position bitmap of a whole row: the candidate buffer's words first, then a stage's
struct RowBits {
  uint32_t* w0;
  uint32_t* w1;
  static constexpr int N0 = RUN_CAP * 2;
  __device__ uint32_t& word(int w) const { return w < N0 ? w0[w] : w1[w - N0]; }
  __device__ bool bit(int i) const { return (word(i >> 5) >> (i & 31)) & 1u; }
};

template <typename TIn>
struct ExactRow {
  const KParams& P;
  const RowCfg& c;
  RowBits bm;  // penalised positions of the row
  const TIn* rowp;
  int64_t hist_a, hist_b;
  int V;
  float mv;

  __device__ float y_at(int i) const {
    float x = Elem<TIn>::ld(rowp, i);
    if (c.pen && bm.bit(i)) {
      const int64_t p = lower_bound_ids(P.hids, hist_a, hist_b, P.voff + i);
      x = penalize(x, __ldg(P.hcnt + p), c);
    }
    return x;
  }
  __device__ uint32_t key_at(int i) const { return okey(vf(y_at(i), c)); }
  __device__ unsigned long long wfx(uint32_t key) const {
    const float e = ex2((from_okey(key) - mv) * LOG2E);
    return (unsigned long long)__float2ull_rn(e * (float)FX_ONE);
  }
};

// Histogram update for one element per lane (`ok` lanes only). When every active lane of the
// warp falls in the same bin, which is the common case on the coarse levels of a float radix,
// the warp adds its totals once instead of contending 32 times on one address.
__device__ __forceinline__ void warp_bin_add(bool ok, uint32_t b, unsigned long long mw,
                                             uint32_t* cnt, unsigned long long* mass) {
  const unsigned act = __ballot_sync(FULLMASK, ok);
  if (!act) return;
  const int lane = threadIdx.x & 31;
  const int ldr = __ffs(act) - 1;
  const uint32_t bl = __shfl_sync(FULLMASK, b, ldr);
  if (__all_sync(FULLMASK, !ok || b == bl)) {
    unsigned long long sum = mw;
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) sum += __shfl_xor_sync(FULLMASK, sum, o);
    if (lane == ldr) {
      atomicAdd(&cnt[bl], (uint32_t)__popc(act));
      if (mass) atomicAdd(&mass[bl], sum);
    }
  } else if (ok) {
    atomicAdd(&cnt[b], 1u);
    if (mass) atomicAdd(&mass[b], mw);
  }
}

// kept-set predicate of the exact search
struct Cut {
  uint32_t tk;  // top-k: key >= tk
  int kind;     // 0: (key > ck) or (key == ck and i <= cid); 1: all
  uint32_t ck;
  int cid;
  uint32_t mk;  // min-p: key >= mk
  __device__ bool keep(uint32_t key, int i) const {
    if (key < tk || key < mk) return false;
    if (kind == 1) return true;
    return key > ck || (key == ck && i <= cid);
  }
};

struct Found {
  uint32_t w;                // key of the tie group reached
  unsigned long long above;  // fixed-point mass strictly above w (kept elements)
  int j;                     // 1-based rank inside the tie group, ascending id
  int n_w;
};

// Canonical position where the cumulative kept mass first reaches (>=) or passes (>) target:
// four levels of 8-bit radix histograms of count and fixed-point mass over the keys.
template <typename TIn>
__device__ Found exact_search(const ExactRow<TIn>& X, const Cut& cut, unsigned long long target,
                              bool strict, Smem& S) {
  uint32_t* cnt = S.bin_cnt;
  unsigned long long* mass = S.bin_mass;
  const int tid = threadIdx.x;
  uint32_t prefix = 0;
  unsigned long long above = 0;
  int last_cnt = 0;
#pragma unroll 1
  for (int lv = 0; lv < 4; ++lv) {
    const int sh = 24 - 8 * lv;
    cnt[tid] = 0;
    mass[tid] = 0ull;
    cbar();
    for (int base = 0; base < X.V; base += NT) {
      const int i = base + tid;
      bool ok = i < X.V;
      uint32_t key = 0;
      if (ok) {
        key = X.key_at(i);
        ok = cut.keep(key, i) && (lv == 0 || (key >> (sh + 8)) == prefix);
      }
      warp_bin_add(ok, (key >> sh) & 255u, ok ? X.wfx(key) : 0ull, cnt, mass);
    }
    cbar();
    // thread t owns bin 255 - t, so thread order is descending key order
    const int b = 255 - tid;
    const unsigned long long mb = mass[b];
    const uint32_t cb = cnt[b];
    unsigned long long tot;
    const unsigned long long ex = cta_excl_scan_u64(mb, &tot, S);
    const unsigned long long before = above + ex, after = before + mb;
    const bool cross_after = strict ? (after > target) : (after >= target);
    const bool cross_before = strict ? (before > target) : (before >= target);
    unsigned long long pick = ~0ull;
    if (cb > 0 && cross_after && !cross_before) pick = (unsigned long long)tid;
    pick = cta_min_u64(pick, S);
    if (pick == ~0ull) {  // target at or beyond the total (rounding): the lowest non-empty bin
      pick = cta_min_u64(cb > 0 ? (unsigned long long)(NT - 1 - tid) : ~0ull, S);
      if (pick == ~0ull) {
        Found f = {0u, 0ull, 0, 0};
        return f;
      }
      pick = (unsigned long long)(NT - 1 - (int)pick);
    }
    if ((int)pick == tid) {
      S.sc[SC_B] = b;
      S.red64[NCW] = before;
      S.sc[SC_J] = (int)cb;
    }
    cbar();
    prefix = (prefix << 8) | (uint32_t)S.sc[SC_B];
    above = S.red64[NCW];
    last_cnt = S.sc[SC_J];
    cbar();
  }
  Found f;
  f.w = prefix;
  f.above = above;
  f.n_w = last_cnt;
  const unsigned long long ew = X.wfx(prefix);
  long long j;
  if (ew == 0) {
    j = last_cnt;
  } else if (target < above) {
    j = 1;
  } else {
    const unsigned long long d = target - above;
    j = strict ? (long long)(d / ew) + 1 : (long long)((d + ew - 1) / ew);
  }
  if (j < 1) j = 1;
  if (j > last_cnt) j = last_cnt;
  f.j = (int)j;
  return f;
}

// index of the j-th (1-based) kept element with key == w, in ascending index order
template <typename TIn>
__device__ int exact_jth(const ExactRow<TIn>& X, const Cut& cut, uint32_t w, int j, Smem& S) {
  constexpr int PER = 8;
  for (int base = 0; base < X.V; base += NT * PER) {
    const int i0 = base + threadIdx.x * PER;
    int cntm = 0;
    for (int i = i0; i < min(i0 + PER, X.V); ++i) {
      const uint32_t key = X.key_at(i);
      if (key == w && cut.keep(key, i)) ++cntm;
    }
    int tot;
    const int ex = cta_excl_scan_i(cntm, &tot, S);
    if (j <= tot) {
      if (ex < j && j <= ex + cntm) {
        int r = j - ex;
        for (int i = i0; i < min(i0 + PER, X.V); ++i) {
          const uint32_t key = X.key_at(i);
          if (key == w && cut.keep(key, i) && --r == 0) {
            S.sc[SC_J] = i;
            break;
          }
        }
      }
      cbar();
      return S.sc[SC_J];
    }
    j -= tot;
  }
  return -1;
}

template <typename TIn>
__device__ void exact_row(const KParams& P, const RowCfg& c, int row, Smem& S,
                          unsigned char* scratch) {
  const int tid = threadIdx.x;
  const RowBits bm{(uint32_t*)S.cand, (uint32_t*)scratch};
  ExactRow<TIn> X{P, c, bm, (const TIn*)P.logits + (int64_t)row * P.ld, 0, 0, (int)P.V, 0.f};
  const int words = (X.V + 31) / 32;
  for (int w = tid; w < words; w += NT) bm.word(w) = 0u;
  cbar();
  if (c.pen) {
    const int64_t a = P.hrow[row], b = P.hrow[row + 1];
    X.hist_a = lower_bound_ids(P.hids, a, b, P.voff);
    X.hist_b = lower_bound_ids(P.hids, X.hist_a, b, P.voff + X.V);
    for (int64_t q = X.hist_a + tid; q < X.hist_b; q += NT) {
      if (__ldg(P.hcnt + q) > 0) {
        const int i = (int)(__ldg(P.hids + q) - P.voff);
        atomicOr(&bm.word(i >> 5), 1u << (i & 31));
      }
    }
  }
  cbar();
  // maximum (and, for greedy rows, the first index of it)
  unsigned long long best = ~0ull;
  for (int i = tid; i < X.V; i += NT) {
    const unsigned long long cc = comp(X.key_at(i), (int)(P.voff + i));
    best = cc < best ? cc : best;
  }
  best = cta_min_u64(best, S);
  X.mv = from_okey(comp_key(best));
  if (c.greedy) {
    if (tid == 0) write_state(P, row, 2, comp_id(best), 0.f, 0.f, 0u, 0);
    return;
  }
  if (!(X.mv > -INFINITY) || !(X.mv <= FLT_MAX)) {
    if (tid == 0) {
      write_state(P, row, 3, -1, 0.f, 0.f, 0u, 0);
      status_or(P, VINFER_ST_NONFINITE);
    }
    return;
  }
  // top-k threshold: radix select over the keys of the whole row (8-bit digits)
  uint32_t tk = 0;
  if (c.topk) {
    uint32_t* hist = S.bin_cnt;
    uint32_t prefix = 0;
    int need = c.k;
#pragma unroll 1
    for (int pass = 0; pass < 4; ++pass) {
      const int shift = 24 - 8 * pass;
      const uint32_t hmask = pass == 0 ? 0u : (0xFFFFFFFFu << (shift + 8));
      hist[tid] = 0;
      cbar();
      for (int base = 0; base < X.V; base += NT) {
        const int i = base + tid;
        bool ok = i < X.V;
        uint32_t k = 0;
        if (ok) {
          k = X.key_at(i);
          ok = (k & hmask) == prefix;
        }
        warp_bin_add(ok, (k >> shift) & 255u, 0ull, hist, nullptr);
      }
      cbar();
      const int d = 255 - tid;
      const int cnt = (int)hist[d];
      int tot;
      const int above = cta_excl_scan_i(cnt, &tot, S);
      if (above < need && above + cnt >= need) {
        S.sc[SC_B] = d;
        S.sc[SC_J] = need - above;
      }
      cbar();
      prefix |= (uint32_t)S.sc[SC_B] << shift;
      need = S.sc[SC_J];
      cbar();
    }
    tk = prefix;
  }
  const Cut base = {tk, 1, 0u, 0, 0u};
  // total mass of the kept-by-top-k set, fixed point
  unsigned long long part = 0;
  for (int i = tid; i < X.V; i += NT) {
    const uint32_t key = X.key_at(i);
    if (base.keep(key, i)) part += X.wfx(key);
  }
  const unsigned long long S_fx = cta_sum_u64(part, S);
  Cut fin = base;
  unsigned long long s_kept = S_fx;
  bool cut_set = false;
  if (c.p < 1.f) {
    const unsigned long long tgt = (unsigned long long)((double)c.p * (double)S_fx);
    const Found f = exact_search(X, base, tgt, false, S);
    if (f.n_w > 0) {
      const int id = exact_jth(X, base, f.w, f.j, S);
      fin.kind = 0;
      fin.ck = f.w;
      fin.cid = id;
      s_kept = f.above + (unsigned long long)f.j * X.wfx(f.w);
      cut_set = true;
    }
  }
  if (c.minp > 0.f) {
    // min-p keeps a prefix by value; it binds when the top-p cut lies below its threshold
    const bool binds = !cut_set || ((from_okey(fin.ck) - X.mv) * LOG2E < c.lm);
    if (binds) {
      unsigned long long pm = 0;
      uint32_t kmin = 0xFFFFFFFFu;
      for (int i = tid; i < X.V; i += NT) {
        const uint32_t key = X.key_at(i);
        if (!base.keep(key, i)) continue;
        if ((from_okey(key) - X.mv) * LOG2E < c.lm) continue;
        pm += X.wfx(key);
        kmin = min(kmin, key);
      }
      const unsigned long long pms = cta_sum_u64(pm, S);
      const uint32_t km = ~cta_max_u32(~kmin, S);
      fin = base;
      fin.mk = km;
      s_kept = pms;
    }
  }
  const unsigned long long tgt = (unsigned long long)((double)c.u * (double)s_kept);
  const Found fd = exact_search(X, fin, tgt, true, S);
  int tok = -1;
  if (fd.n_w > 0) tok = exact_jth(X, fin, fd.w, fd.j, S);
  if (tid == 0) {
    if (tok < 0) status_or(P, VINFER_ST_INTERNAL);
    const int gtok = tok < 0 ? -1 : (int)(P.voff + tok);
    const float sk = (float)((double)s_kept / FX_ONE);
    if (fin.kind == 0) write_state(P, row, 0, gtok, X.mv, sk, fin.ck, (int)(P.voff + fin.cid));
    else if (fin.mk != 0u) write_state(P, row, 0, gtok, X.mv, sk, fin.mk, 0x7FFFFFFF);
    else if (c.topk) write_state(P, row, 0, gtok, X.mv, sk, tk, 0x7FFFFFFF);
    else write_state(P, row, 1, gtok, X.mv, sk, 0u, 0);
  }
}

// ---------------------------------------------------------------------------------------------
// finishing a row: local shard record, final answer, or the exact search
// ---------------------------------------------------------------------------------------------
template <typename TIn>
__device__ void finish_row(const KParams& P, Smem& S, unsigned char* scratch, int row,
                           const unsigned char* src0, size_t stride, int nsrc, bool local,
                           int* unresolved) {
  const int tid = threadIdx.x;
  const RowCfg c = load_row(P, row);
  const MergeIn m = gather_sorted(src0, stride, nsrc, c, S, (unsigned long long*)scratch);
  const unsigned long long* e = (const unsigned long long*)scratch;
  if (local) {
    // this rank's shard record: entries at or above the K-th, all ties, <= shard_cap
    unsigned char* out = P.shard_out + (size_t)row * P.shard_stride;
    RecHdr* oh = (RecHdr*)out;
    unsigned long long* oe = (unsigned long long*)(out + sizeof(RecHdr));
    if ((m.flags & (REC_OVERFLOW | REC_BAD | REC_EXACT)) || m.n > MERGE_CAP) {
      if (tid == 0)
        write_flag_hdr(oh, (m.flags & REC_BAD) ? REC_BAD : REC_OVERFLOW, m.m_y, m.s);
      return;
    }
    int nr = m.n;
    uint32_t tkey = 0;
    if (m.n >= c.K) {
      tkey = comp_key(e[c.K - 1]);
      nr = count_ge(e, m.n, tkey);
    }
    const bool over = nr > P.shard_cap;
    const bool unret = (m.flags & REC_UNRETAINED) || nr < m.n;
    for (int j = tid; j < min(nr, P.shard_cap); j += NT) oe[j] = e[j];
    if (tid == 0) {
      oh->m_y = m.m_y;
      oh->s = m.s;
      oh->n = over ? 0 : nr;
      oh->t_key = unret ? max(tkey, m.d_key) : 0u;
      oh->flags = over ? REC_OVERFLOW : (unret ? REC_UNRETAINED : 0u);
    }
    return;
  }
  if (m.flags & REC_BAD) {
    if (tid == 0) {
      write_state(P, row, 3, -1, 0.f, 0.f, 0u, 0);
      status_or(P, VINFER_ST_BAD_PARAM);
      if (unresolved) unresolved[row] = 0;
    }
    return;
  }
  bool done = false;
  if (!(m.flags & (REC_OVERFLOW | REC_EXACT)) && m.n <= MERGE_CAP)
    done = finalize_sorted(P, c, row, m, e, S);
  if (unresolved) {  // sharded merge: the caller resolves the row from the full logits
    if (tid == 0) {
      unresolved[row] = done ? 0 : 1;
      if (!done) write_state(P, row, 3, -1, 0.f, 0.f, 0u, 0);
    }
    return;
  }
  cbar();
  if (!done) exact_row<TIn>(P, c, row, S, scratch);
}

// ---------------------------------------------------------------------------------------------
// work decomposition: CTA b owns segments [seg_begin(b), seg_begin(b + 1)) of the row-major list
// of B * nseg segments; a run is its maximal part inside one row
// ---------------------------------------------------------------------------------------------
__device__ __forceinline__ int seg_begin(const KParams& P, int b) {
  return (int)(((int64_t)b * P.total) / P.grid);
}
__device__ __forceinline__ int seg_owner(const KParams& P, int sg) {
  return (int)((((int64_t)sg + 1) * P.grid - 1) / P.total);
}

// ---------------------------------------------------------------------------------------------
// producer warp: stages segments for the consumers
// ---------------------------------------------------------------------------------------------
template <typename TIn>
__device__ void producer(const KParams& P, Smem& S) {
  using E = Elem<TIn>;
  constexpr int ES = 16 / E::A;
  const int lane = threadIdx.x & 31;
  const int s0 = seg_begin(P, blockIdx.x), s1 = seg_begin(P, blockIdx.x + 1);
  float prm = 0.f;
  bool pen = false;
  int64_t hp = 0, hend = 0;
  for (int i = 0; s0 + i < s1; ++i) {
    const int sg = s0 + i, row = sg / P.nseg, seg = sg - row * P.nseg;
    const int s = i % NSTAGE, use = i / NSTAGE;
    const Geo g = geometry<TIn>(P, row, seg);
    if (i == 0 || seg == 0) {  // a new run: the row's parameters and history position
      prm = lane < 8 ? load_param(P, row, lane) : 0.f;
      const float rep = __shfl_sync(FULLMASK, prm, 3);
      const float pres = __shfl_sync(FULLMASK, prm, 4);
      const float freq = __shfl_sync(FULLMASK, prm, 5);
      pen = P.hrow != nullptr && (rep != 1.f || pres != 0.f || freq != 0.f);
      if (pen) {
        const int64_t a = __ldg(P.hrow + row);
        hend = __ldg(P.hrow + row + 1);
        // the first entry at or after this segment's first global id (entries of lower
        // vocabulary shards precede it when the row is sharded)
        hp = (seg == 0 && P.voff == 0) ? a : warp_lower_bound(P.hids, a, hend, g.gbase, lane);
      }
    }
    // penalised tokens of this segment: the next entries of the row's ascending history
    int ns = 0;
    int rid[SIDE_PER_LANE], rcn[SIDE_PER_LANE];
    if (pen) {
      const int64_t lim = g.gbase + g.n;
#pragma unroll
      for (int q = 0; q < SIDE_PER_LANE; ++q) {
        const int64_t p = hp + lane + 32 * q;
        rid[q] = p < hend ? __ldg(P.hids + p) : 0x7FFFFFFF;
        rcn[q] = p < hend ? __ldg(P.hcnt + p) : 0;
      }
#pragma unroll
      for (int q = 0; q < SIDE_PER_LANE; ++q)
        ns += __popc(__ballot_sync(FULLMASK, (int64_t)rid[q] < lim));
      if (ns == SIDE_CAP) {  // the window is full: find the end of this segment's entries
        const int64_t e = warp_lower_bound(P.hids, hp + SIDE_CAP, hend, lim, lane);
        if (e > hp + SIDE_CAP) {
          hp = e;
          ns = -1;  // more penalised tokens than a stage holds: the row takes the exact search
        } else {
          hp += SIDE_CAP;
        }
      } else {
        hp += ns;
      }
    }
    uint32_t hv = 0, tv = 0;
    if (lane < g.head) hv = E::ldraw(g.rowp, g.lo + lane);
    if (lane < g.n - g.tail0) tv = E::ldraw(g.rowp, g.lo + g.tail0 + lane);
    // ---- wait until the consumers released this stage's previous segment
    if (use >= 1 && !mbar_wait_bounded(&S.empty[s], (use - 1) & 1)) {
      if (lane == 0) status_or(P, VINFER_ST_TIMEOUT);
      return;
    }
    Stage& st = S.st[s];
    if (lane < 8) st.prm[lane] = prm;
    if (lane == 0) st.ns = ns;
#pragma unroll
    for (int q = 0; q < SIDE_PER_LANE; ++q) {
      const int j = lane + 32 * q;
      if (j < ns) {
        st.side_id[j] = rid[q];
        st.side_cnt[j] = rcn[q];
      }
    }
    if (lane < g.off) E::neg_inf(st.data, lane);
    if (lane < g.pad_end) E::neg_inf(st.data, g.off + g.n + lane);
    if (lane < g.head) E::straw(st.data, g.off + lane, hv);
    if (lane < g.n - g.tail0) E::straw(st.data, g.off + g.tail0 + lane, tv);
    __syncwarp();
    if (lane == 0) {
      const uint32_t bytes = (uint32_t)g.inter * ES;
      mbar_arrive_expect_tx(&S.full[s], bytes);
      for (uint32_t b = 0; b < bytes; b += 16384u) {
        tma_load_1d(st.data + (size_t)(g.off + g.head) * ES + b,
                    (const unsigned char*)((const TIn*)g.rowp + g.lo + g.head) + b,
                    min(16384u, bytes - b), &S.full[s]);
      }
    }
    __syncwarp();
  }
}

// ---------------------------------------------------------------------------------------------
// consumers
// ---------------------------------------------------------------------------------------------
// smallest y with vf(y) >= vt: about y = vt * T; the boundary lies within a few keys of it in
// the normal range, found by one round of 32 probes (a full binary search otherwise)
__device__ float ylo_for(float vt, const RowCfg& c) {
  if (c.greedy || vt == -INFINITY) return vt;
  const int lane = threadIdx.x & 31;
  const uint32_t k0 = okey(vt * c.T);
  const bool inside = k0 > okey(-INFINITY) + 16u && k0 < okey(INFINITY) - 16u;
  const uint32_t kp = inside ? k0 - 16u + (uint32_t)lane : k0;  // probes k0 - 16 .. k0 + 15
  const bool ge = vf(from_okey(kp), c) >= vt;
  const unsigned b = __ballot_sync(FULLMASK, ge);
  if (inside && b != 0u && b != FULLMASK &&
      (b >> (__ffs(b) - 1)) == (FULLMASK >> (__ffs(b) - 1)))
    return from_okey(k0 - 16u + (uint32_t)(__ffs(b) - 1));  // the flip lies inside the window
  // outside the window (extreme temperatures, subnormals): binary search over ordered keys
  uint32_t lo = okey(-INFINITY), hi = okey(INFINITY);
  if (vf(from_okey(lo), c) >= vt) return -INFINITY;
  while (hi - lo > 1) {
    const uint32_t mid = lo + (hi - lo) / 2;
    if (vf(from_okey(mid), c) >= vt) hi = mid; else lo = mid;
  }
  return from_okey(hi);
}

// append a candidate to the run's buffer (overflow is flagged, never written past the end)
__device__ __forceinline__ void add_cand(Smem& S, unsigned long long e) {
  const int pos = atomicAdd(&S.sc[SC_NC], 1);
  if (pos < RUN_CAP) S.cand[pos] = e;
}

// Sorts the run's candidates and keeps the K largest with every tie of the K-th: the kept
// entries land sorted in out[0, n_ret). Returns n_ret; *tkey receives the K-th key (0 when all
// n candidates are kept because n < K). The candidates stay untouched.
__device__ int select_sorted(Smem& S, int n, int K, unsigned long long* out, uint32_t* tkey) {
  const int tid = threadIdx.x;
  if (n <= NT) {  // rank by counting: one candidate per thread
    unsigned long long x = 0ull;
    int rank = 0;
    if (tid < n) {
      x = S.cand[tid];
      for (int j = 0; j < n; ++j) rank += S.cand[j] < x;
      if (rank == K - 1) S.sc[SC_TKEY] = (int)comp_key(x);
    }
    cbar();
    const uint32_t t = n >= K ? (uint32_t)S.sc[SC_TKEY] : 0u;
    if (tid == 0) S.sc[SC_NRET] = 0;
    cbar();
    if (tid < n && comp_key(x) >= t) {
      out[rank] = x;
      atomicMax(&S.sc[SC_NRET], rank + 1);
    }
    cbar();
    *tkey = t;
    return S.sc[SC_NRET];
  }
  // larger sets (rare): bitonic sort of a padded copy, then cut at the K-th
  int np = 1;
  while (np < n) np <<= 1;
  for (int j = tid; j < np; j += NT) out[j] = j < n ? S.cand[j] : ~0ull;
  cbar();
  for (int k = 2; k <= np; k <<= 1) {
    for (int j = k >> 1; j > 0; j >>= 1) {
      for (int i = tid; i < np; i += NT) {
        const int ixj = i ^ j;
        if (ixj > i) {
          const unsigned long long a = out[i], b = out[ixj];
          if ((a > b) == ((i & k) == 0)) {
            out[i] = b;
            out[ixj] = a;
          }
        }
      }
      cbar();
    }
  }
  const uint32_t t = n >= K ? comp_key(out[K - 1]) : 0u;
  *tkey = t;
  return n >= K ? count_ge(out, n, t) : n;
}

// the elements of one staged vector at or above ylo become candidates
template <typename TIn>
__device__ __noinline__ void expand_vector(Smem& S, const RowCfg& c, const Geo& g, uint4 q, int j,
                                           float ylo, bool checkbits) {
  using E = Elem<TIn>;
#pragma unroll 1
  for (int e = 0; e < E::A; ++e) {
    const int slot = j * E::A + e;
    const int li = slot - g.off;
    if (li < 0 || li >= g.n) continue;
    if (checkbits && ((S.bitmap[slot >> 5] >> (slot & 31)) & 1u)) continue;
    const float y = E::at(q, e);
    if (y >= ylo) add_cand(S, comp(okey(vf(y, c)), (int)(g.gbase + li)));
  }
}

struct RunState {        // per consumer thread, carried across the segments of a run
  float m_t, s_t;        // online softmax max and sum (top-k off)
  unsigned long long gbest;  // greedy: smallest composite key (max value, first index)
};

// One segment of the current run: penalties, then either the running greedy minimum, or the
// candidates at or above the run's threshold (established on the run's first segment).
template <typename TIn>
__device__ void run_segment(const KParams& P, const RowCfg& c, const Geo& g, Stage& st, Smem& S,
                            RunState& R) {
  using E = Elem<TIn>;
  constexpr int A = E::A;
  const int tid = threadIdx.x, lane = tid & 31, w = tid >> 5;
  void* sv = st.data;
  const int ns = st.ns;
  if (ns < 0) {
    if (tid == 0) S.sc[SC_RFL] |= RUN_OVER;
    cbar();
    return;
  }
  // ---- penalised tokens: exact float32 values on the side, -inf in the staged copy
  if (ns > 0) {
    const int nwords = (g.nvec * A + 31) / 32;
    for (int wd = tid; wd < nwords; wd += NT) S.bitmap[wd] = 0u;
    cbar();
    for (int j = tid; j < ns; j += NT) {
      const int cnt = st.side_cnt[j];
      const int64_t li = (int64_t)st.side_id[j] - g.gbase;
      const int slot = g.off + (int)li;
      const bool inside = li >= 0 && li < g.n;  // false only for a history out of order
      if (!inside) status_or(P, VINFER_ST_INTERNAL);
      if (cnt > 0 && inside) {
        S.side_y[j] = penalize(E::sm(sv, slot), cnt, c);
        atomicOr(&S.bitmap[slot >> 5], 1u << (slot & 31));
        E::neg_inf(sv, slot);
      } else {
        S.side_y[j] = __int_as_float(0x7fc00000);  // NaN: not penalised, value stays in place
      }
    }
    cbar();
  }
  const uint4* sv4 = (const uint4*)sv;
  if (c.greedy) {  // running first argmax
    float best = R.gbest == ~0ull ? -INFINITY : from_okey(comp_key(R.gbest));
    for (int j = tid; j < g.nvec; j += NT) {
      const uint4 q = sv4[j];
      const float vm = E::vmax(q);
      if (vm > best) {
        int e = 0;
        while (e < A - 1 && E::at(q, e) != vm) ++e;
        const unsigned long long cc = comp(okey(vm), (int)(g.gbase + j * A + e - g.off));
        R.gbest = cc < R.gbest ? cc : R.gbest;
        best = vm;
      }
    }
    for (int j = tid; j < ns; j += NT) {
      const float y = S.side_y[j];
      if (isnan(y)) continue;
      const unsigned long long cc = comp(okey(y), st.side_id[j]);
      R.gbest = cc < R.gbest ? cc : R.gbest;
    }
    cbar();
    return;
  }
  const float ylo0 = S.sf[SF_YLO];
  const bool known = !isnan(ylo0);  // the run's collection threshold exists
  const bool checkbits = ns > 0;    // penalised slots hold -inf; only a -inf bound reaches them
  float ylo = ylo0;
  if (known) {
    // ---- stream: each vector's maximum against the threshold; the rare vector that reaches
    //      it is expanded in place by the thread that read it
    for (int j = tid; j < g.nvec; j += NT) {
      const uint4 q = sv4[j];
      const float vm = E::vmax(q);
      if (c.need_sum) {
        if (vm > R.m_t) {
          R.s_t *= ex2((R.m_t - vm) * c.c2);
          R.m_t = vm;
        }
#pragma unroll
        for (int e = 0; e < A; ++e) R.s_t += ex2((E::at(q, e) - R.m_t) * c.c2);
      }
      if (vm >= ylo) expand_vector<TIn>(S, c, g, q, j, ylo, checkbits && ylo == -INFINITY);
    }
    for (int j = tid; j < ns; j += NT) {
      const float y = S.side_y[j];
      if (isnan(y)) continue;
      if (c.need_sum) {
        if (y > R.m_t) {
          R.s_t *= ex2((R.m_t - y) * c.c2);
          R.m_t = y;
        }
        R.s_t += ex2((y - R.m_t) * c.c2);
      }
      if (y >= ylo) add_cand(S, comp(okey(vf(y, c)), st.side_id[j]));
    }
  } else {
    // ---- first segment of the run: per-thread maxima, then a bound on the K-th largest
    float tmax = -INFINITY;
    for (int j = tid; j < g.nvec; j += NT) {
      const uint4 q = sv4[j];
      const float vm = E::vmax(q);
      tmax = fmaxf(tmax, vm);
      if (c.need_sum) {
        if (vm > R.m_t) {
          R.s_t *= ex2((R.m_t - vm) * c.c2);
          R.m_t = vm;
        }
#pragma unroll
        for (int e = 0; e < A; ++e) R.s_t += ex2((E::at(q, e) - R.m_t) * c.c2);
      }
    }
    for (int j = tid; j < ns; j += NT) {
      const float y = S.side_y[j];
      if (isnan(y)) continue;
      tmax = fmaxf(tmax, y);
      if (c.need_sum) {
        if (y > R.m_t) {
          R.s_t *= ex2((R.m_t - y) * c.c2);
          R.m_t = y;
        }
        R.s_t += ex2((y - R.m_t) * c.c2);
      }
    }
    // each warp extracts its kw = ceil(K / 8) largest lane maxima (distinct elements); the
    // K-th largest of those 8 * kw values bounds the segment's K-th largest value from below
    const int kw = min((c.K + NCW - 1) / NCW, 32);
    {
      float mine = tmax;
      for (int r = 0; r < kw; ++r) {
        float m = mine;
#pragma unroll
        for (int o = 16; o > 0; o >>= 1) m = fmaxf(m, __shfl_xor_sync(FULLMASK, m, o));
        const unsigned b = __ballot_sync(FULLMASK, mine == m && m > -INFINITY);
        if (lane == 0) S.ext[w * 32 + r] = b ? m : -INFINITY;
        if (b && lane == __ffs(b) - 1) mine = -INFINITY;
      }
    }
    if (tid == 0) S.sf[SF_TH] = -INFINITY;  // fewer than K finite values: no bound
    cbar();
    if (tid < NCW * kw) {
      // rank of this value in the union of the eight descending lists (ties by list index)
      const int wl = tid / kw, r = tid - wl * kw;
      const float x = S.ext[wl * 32 + r];
      int rank = r;
      for (int o = 0; o < NCW; ++o) {
        if (o == wl) continue;
        const float* L = S.ext + o * 32;
        int a = 0, b = kw;
        while (a < b) {
          const int mid = (a + b) >> 1;
          if (o < wl ? (L[mid] >= x) : (L[mid] > x)) a = mid + 1; else b = mid;
        }
        rank += a;
      }
      if (rank == c.K - 1 && x > -INFINITY) S.sf[SF_TH] = x;
    }
    cbar();
    if (w == 0) {
      const float th = S.sf[SF_TH];
      const float y = th == -INFINITY ? -INFINITY : ylo_for(vf(th, c), c);
      if (lane == 0) S.sf[SF_YLO] = y;
    }
    cbar();
    ylo = S.sf[SF_YLO];
    for (int j = tid; j < g.nvec; j += NT) {
      const uint4 q = sv4[j];
      if (E::vmax(q) >= ylo) expand_vector<TIn>(S, c, g, q, j, ylo, checkbits && ylo == -INFINITY);
    }
    for (int j = tid; j < ns; j += NT) {
      const float y = S.side_y[j];
      if (y >= ylo) add_cand(S, comp(okey(vf(y, c)), st.side_id[j]));
    }
  }
  cbar();
  const int nc = S.sc[SC_NC];
  if (nc > RUN_CAP) {
    if (tid == 0) S.sc[SC_RFL] |= RUN_OVER;
    cbar();
    return;
  }
  // ---- tighten: whenever the buffer holds more than max(2K, 64) candidates (and after the
  //      run's first segment), keep only the K largest (with ties) and raise the threshold to
  //      the K-th value, so later segments contribute fewer candidates
  if ((!known && nc > c.K) || nc > max(2 * c.K, 64)) {
    unsigned long long* tmp = (unsigned long long*)st.data;  // the segment is done with
    uint32_t t;
    const int nr = select_sorted(S, nc, c.K, tmp, &t);
    for (int j = tid; j < nr; j += NT) S.cand[j] = tmp[j];
    if (tid == 0) S.sc[SC_NC] = nr;
    if (w == 0) {
      const float y = ylo_for(from_okey(t), c);
      if (lane == 0) S.sf[SF_YLO] = y;
    }
    cbar();
  }
}

// Completes the run: its sorted candidates become the row's answer (single-run rows), a shard
// record (local mode), or a run record for the CTA that completes the row last to merge.
template <typename TIn>
__device__ void run_end(const KParams& P, const RowCfg& c, int row, int first_seg, int last_seg,
                        Smem& S, RunState& R, unsigned char* scratch) {
  const int tid = threadIdx.x;
  const int nruns = seg_owner(P, row * P.nseg + P.nseg - 1) - seg_owner(P, row * P.nseg) + 1;
  const int run_idx = blockIdx.x - seg_owner(P, row * P.nseg);
  const int64_t lo = (int64_t)first_seg * P.seg_len;
  const int64_t hi = min(P.V, (int64_t)(last_seg + 1) * P.seg_len);
  const int n_run = (int)(hi - lo);
  unsigned long long* sorted = (unsigned long long*)scratch;
  // the run's own record, in shared memory first
  uint32_t flags = 0, tkey = 0;
  int nret = 0;
  float m_y = -INFINITY, s_run = 0.f;
  if (c.bad) {
    flags = REC_BAD;
  } else if (c.exact || (S.sc[SC_RFL] & RUN_OVER)) {
    flags = c.exact ? REC_EXACT : REC_OVERFLOW;
  } else if (c.greedy) {
    const unsigned long long b = cta_min_u64(R.gbest, S);
    if (b != ~0ull) {
      sorted[0] = b;
      nret = 1;
      m_y = from_okey(comp_key(b));
      tkey = comp_key(b);
    }
    if (n_run > 1) flags = REC_UNRETAINED;
  } else {
    const int nc = S.sc[SC_NC];
    nret = select_sorted(S, nc, c.K, sorted, &tkey);
    if (nret > CAND_CAP) flags = REC_OVERFLOW;
    else if (nret < n_run) flags = REC_UNRETAINED;
    else tkey = 0u;
    if (c.need_sum) {  // rescale every partial sum to the run maximum, fixed order
      const uint32_t mk = cta_max_u32(okey(R.m_t == -FLT_MAX ? -INFINITY : R.m_t), S);
      m_y = from_okey(mk);
      const float part = (R.m_t == -FLT_MAX) ? 0.f : R.s_t * ex2((R.m_t - m_y) * c.c2);
      float tot;
      cta_excl_scan_f(part, &tot, S);
      s_run = tot;
    }
  }
  cbar();
  if (nruns == 1 && P.mode == 0) {  // the whole row is here: answer it directly
    if (flags & REC_BAD) {
      if (tid == 0) {
        write_state(P, row, 3, -1, 0.f, 0.f, 0u, 0);
        status_or(P, VINFER_ST_BAD_PARAM);
      }
      return;
    }
    bool done = false;
    if (!(flags & (REC_OVERFLOW | REC_EXACT))) {
      MergeIn m;
      m.m_y = m_y;
      m.s = s_run;
      m.d_key = tkey;
      m.flags = flags;
      m.n = nret;
      done = finalize_sorted(P, c, row, m, sorted, S);
    }
    cbar();
    if (!done) exact_row<TIn>(P, c, row, S, scratch);
    return;
  }
  // write the record: this run's slot of the row, or this rank's shard record (single run)
  const bool shard = nruns == 1;  // local mode with the whole row here
  unsigned char* rec = shard ? P.shard_out + (size_t)row * P.shard_stride
                             : P.recs + ((size_t)row * P.nseg + run_idx) * REC_STRIDE;
  const int cap = shard ? P.shard_cap : CAND_CAP;
  if (nret > cap && !(flags & (REC_BAD | REC_EXACT))) flags = REC_OVERFLOW;
  RecHdr* h = (RecHdr*)rec;
  unsigned long long* ent = (unsigned long long*)(rec + sizeof(RecHdr));
  const bool listed = !(flags & (REC_BAD | REC_EXACT | REC_OVERFLOW));
  if (listed)
    for (int j = tid; j < nret; j += NT) ent[j] = sorted[j];
  if (tid == 0) {
    h->m_y = m_y;
    h->s = s_run;
    h->n = listed ? nret : 0;
    h->t_key = listed ? tkey : 0u;
    h->flags = flags;
  }
  if (shard) return;
  // the CTA that completes the row merges it
  __threadfence();
  cbar();
  if (tid == 0) {
    const int old = atom_add_acq_rel(&P.counters[row], 1);
    const int last = old == nruns - 1;
    if (last) P.counters[row] = 0;  // ready for the next call
    S.sc[SC_LAST] = last;
  }
  cbar();
  if (!S.sc[SC_LAST]) return;
  finish_row<TIn>(P, S, scratch, row, P.recs + (size_t)row * P.nseg * REC_STRIDE, REC_STRIDE,
                  nruns, P.mode == 1, nullptr);
}

template <typename TIn>
__device__ void consumer(const KParams& P, Smem& S) {
  const int tid = threadIdx.x;
  const int s0 = seg_begin(P, blockIdx.x), s1 = seg_begin(P, blockIdx.x + 1);
  RowCfg c{};
  RunState R{};
  int first_seg = 0;
  for (int i = 0; s0 + i < s1; ++i) {
    const int sg = s0 + i, row = sg / P.nseg, seg = sg - row * P.nseg;
    const int s = i % NSTAGE, use = i / NSTAGE;
    Stage& st = S.st[s];
    const bool ok = mbar_wait_bounded(&S.full[s], use & 1);
    if (cbar_or(!ok)) {
      mbar_wait_bounded(&S.full[s], use & 1);  // a copy may still be in flight
      if (tid == 0) status_or(P, VINFER_ST_TIMEOUT);
      return;
    }
    if (i == 0 || seg == 0) {  // a new run
      c = cfg_from(P, st.prm);
      R.m_t = -FLT_MAX;
      R.s_t = 0.f;
      R.gbest = ~0ull;
      first_seg = seg;
      if (tid == 0) {
        S.sc[SC_NC] = 0;
        S.sc[SC_RFL] = 0;
        S.sf[SF_YLO] = __int_as_float(0x7fc00000);  // NaN: no threshold yet
      }
      cbar();
    }
    if (!(c.bad || c.exact) && !(S.sc[SC_RFL] & RUN_OVER)) {
      const Geo g = geometry<TIn>(P, row, seg);
      run_segment<TIn>(P, c, g, st, S, R);  // ends with a consumer barrier
    }
    if (sg + 1 == s1 || seg == P.nseg - 1) {
      run_end<TIn>(P, c, row, first_seg, seg, S, R, st.data);
      cbar();
    }
    if (tid == 0) mbar_arrive(&S.empty[s]);
  }
}

// ---------------------------------------------------------------------------------------------
// kernels
// ---------------------------------------------------------------------------------------------
template <typename TIn>
__global__ void __launch_bounds__(NTHR, 2) k_sample(const KParams P) {
  extern __shared__ __align__(128) unsigned char smraw[];
  Smem& S = *reinterpret_cast<Smem*>(smraw);
  if (threadIdx.x == 0) {
    for (int s = 0; s < NSTAGE; ++s) {
      mbar_init(&S.full[s], 1);
      mbar_init(&S.empty[s], 1);
    }
    mbar_fence_init();
  }
  __syncthreads();
  if (threadIdx.x >= NT) {
    producer<TIn>(P, S);
    return;
  }
  consumer<TIn>(P, S);
}

// merge of gathered shard records: one CTA of consumer threads per row
template <typename TIn>
__global__ void __launch_bounds__(NT, 1) k_merge(const KParams P, const unsigned char* recs,
                                              int world, int* unresolved) {
  extern __shared__ __align__(128) unsigned char smraw[];
  Smem& S = *reinterpret_cast<Smem*>(smraw);
  const int row = blockIdx.x;
  finish_row<TIn>(P, S, S.st[0].data, row, recs + (size_t)row * P.shard_stride,
                  (size_t)P.B * P.shard_stride, world, false, unresolved);
}

// final probabilities [B, V] from the row states (parity checks only)
template <typename TIn>
__global__ void __launch_bounds__(256) k_probs(const KParams P) {
  const int row = blockIdx.y;
  const RowCfg c = load_row(P, row);
  const RowState st = P.rows[row];
  const TIn* rowp = (const TIn*)P.logits + (int64_t)row * P.ld;
  float* out = P.out_probs + (int64_t)row * P.V;
  int64_t ha = 0, hb = 0;
  if (c.pen) {
    ha = P.hrow[row];
    hb = P.hrow[row + 1];
  }
  const float inv = st.s_kept > 0.f ? 1.0f / st.s_kept : 0.f;
  for (int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; i < P.V;
       i += (int64_t)gridDim.x * blockDim.x) {
    const int64_t gid = P.voff + i;
    float q = 0.f;
    if (st.kind == 2) {
      q = (gid == st.token) ? 1.f : 0.f;
    } else if (st.kind != 3) {
      float y = Elem<TIn>::ld(rowp, i);
      if (c.pen) {
        const int64_t p = lower_bound_ids(P.hids, ha, hb, gid);
        if (p < hb && __ldg(P.hids + p) == gid && __ldg(P.hcnt + p) > 0)
          y = penalize(y, __ldg(P.hcnt + p), c);
      }
      const float v = vf(y, c);
      const uint32_t key = okey(v);
      const bool keep =
          st.kind == 1 || key > st.cut_key || (key == st.cut_key && gid <= st.cut_id);
      if (keep) q = ex2((v - st.m_v) * LOG2E) * inv;
    }
    out[i] = q;
  }
}

// ---------------------------------------------------------------------------------------------
// host side
// ---------------------------------------------------------------------------------------------
struct Shape {
  int nseg, seg_len, grid;
};

// Segments per row and CTAs for a batch. With fewer rows than CTAs, each row is split into
// c = ctas / B runs of whole segments (nseg a multiple of c), so every CTA streams one run and
// only split rows need a merge; with more rows than CTAs, the CTAs share the row-major list of
// segments in equal contiguous ranges.
Shape plan(int64_t B, int64_t V, int dtype, int ctas) {
  const int es = dtype == VINFER_DTYPE_BF16 ? 2 : 4;
  const int A = 16 / es;
  const int64_t min_seg = (V * es + SEG_BYTES - 1) / SEG_BYTES;
  int64_t c = 1;
  if (B < ctas) c = std::min<int64_t>(ctas / B, MAX_NSEG);
  c = std::max<int64_t>(1, std::min<int64_t>(c, V / 2048));  // segments of >= 2048 tokens
  int64_t nseg = std::max<int64_t>(min_seg, c);
  nseg = (nseg + c - 1) / c * c;
  nseg = std::min<int64_t>(nseg, MAX_NSEG);
  int64_t len = (V + nseg - 1) / nseg;
  len = (len + A - 1) / A * A;
  nseg = (V + len - 1) / len;
  Shape s;
  s.nseg = (int)nseg;
  s.seg_len = (int)len;
  const int64_t total = B * nseg;
  s.grid = (int)std::min<int64_t>(total, B < ctas ? B * c : ctas);
  return s;
}

constexpr size_t ALIGN = 256;
size_t align_up(size_t x) { return (x + ALIGN - 1) / ALIGN * ALIGN; }

struct WsLayout {
  size_t counters, rows, recs, total;
};
// Records: one slot per (row, run). Rows are split into at most nseg runs; nseg is at most
// MAX_NSEG when rows may be split for parallelism (B below the resident-CTA bound), otherwise
// the count the segment size alone needs.
WsLayout ws_layout(int64_t B, int64_t V, int dtype) {
  const int64_t nseg = B < CTA_CAP ? MAX_NSEG : plan(B, V, dtype, CTA_CAP).nseg;
  WsLayout L;
  L.counters = 0;
  L.rows = align_up((size_t)B * sizeof(int));
  L.recs = L.rows + align_up((size_t)B * sizeof(RowState));
  L.total = L.recs + (size_t)B * nseg * REC_STRIDE;
  return L;
}

int check_args(const VinferSampleArgs* a) {
  if (!a || !a->logits || !a->out_ids) return VINFER_E_ARG;
  if (a->dtype != VINFER_DTYPE_F32 && a->dtype != VINFER_DTYPE_BF16) return VINFER_E_ARG;
  if (a->batch < 1 || a->vocab < 1 || a->ld < a->vocab) return VINFER_E_ARG;
  if (a->batch > VINFER_MAX_BATCH) return VINFER_E_LIMIT;
  if (a->vocab > VINFER_MAX_VOCAB || a->vocab_total > VINFER_MAX_VOCAB) return VINFER_E_LIMIT;
  if (a->vocab_offset < 0 || a->vocab_total < a->vocab_offset + a->vocab) return VINFER_E_ARG;
  const size_t es = a->dtype == VINFER_DTYPE_BF16 ? 2 : 4;
  if (((uintptr_t)a->logits) % es) return VINFER_E_ARG;
  if (a->hist_row_ptr && (!a->hist_ids || !a->hist_counts)) return VINFER_E_ARG;
  return VINFER_OK;
}

KParams make_params(const VinferSampleArgs* a, const Shape& s, void* ws) {
  KParams P = {};
  P.logits = a->logits;
  P.ld = a->ld;
  P.V = a->vocab;
  P.voff = a->vocab_offset;
  P.vtotal = a->vocab_total;
  P.B = (int)a->batch;
  P.nseg = s.nseg;
  P.seg_len = s.seg_len;
  P.total = (int)(a->batch * s.nseg);
  P.grid = s.grid;
  P.flags = a->flags;
  P.temperature = a->temperature;
  P.top_k = a->top_k;
  P.top_p = a->top_p;
  P.min_p = a->min_p;
  P.rep = a->repetition_penalty;
  P.pres = a->presence_penalty;
  P.freq = a->frequency_penalty;
  P.hrow = a->hist_row_ptr;
  P.hids = a->hist_ids;
  P.hcnt = a->hist_counts;
  P.uni = a->uniforms;
  P.out_ids = a->out_ids;
  P.out_probs = a->out_probs;
  P.status = a->status;
  const WsLayout L = ws_layout(a->batch, a->vocab, a->dtype);
  unsigned char* base = (unsigned char*)ws;
  P.counters = (int*)(base + L.counters);
  P.rows = (RowState*)(base + L.rows);
  P.recs = base + L.recs;
  return P;
}

// per device and kernel: opt in to the dynamic shared memory once, and remember how many
// CTAs of it fit on the device at once
struct KernInfo {
  bool ready;
  int ctas;
};
int kernel_info(const void* kern, int slot, int threads, int* ctas) {
  static KernInfo info[64][4] = {};
  int dev = 0;
  if (cudaGetDevice(&dev) != cudaSuccess || dev < 0 || dev >= 64) return VINFER_E_CUDA;
  KernInfo& k = info[dev][slot];
  if (!k.ready) {
    if (cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize,
                             (int)sizeof(Smem)) != cudaSuccess)
      return VINFER_E_CUDA;
    int sms = 0, per_sm = 0;
    if (cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev) != cudaSuccess)
      return VINFER_E_CUDA;
    if (cudaOccupancyMaxActiveBlocksPerMultiprocessor(&per_sm, kern, threads, sizeof(Smem)) !=
        cudaSuccess)
      return VINFER_E_CUDA;
    k.ctas = std::max(1, sms * per_sm);
    k.ready = true;
  }
  *ctas = k.ctas;
  return VINFER_OK;
}

// resident CTAs of k_sample on the current device (at most CTA_CAP)
int sample_ctas(int dtype, int* ctas) {
  const void* kern = dtype == VINFER_DTYPE_BF16 ? (const void*)k_sample<__nv_bfloat16>
                                                : (const void*)k_sample<float>;
  if (kernel_info(kern, dtype == VINFER_DTYPE_BF16 ? 0 : 1, NTHR, ctas) != VINFER_OK)
    return VINFER_E_CUDA;
  *ctas = std::min(*ctas, CTA_CAP);
  return VINFER_OK;
}

int launch_sample(const KParams& P, int dtype, cudaStream_t st) {
  const dim3 grid(P.grid);
  if (dtype == VINFER_DTYPE_BF16) k_sample<__nv_bfloat16><<<grid, NTHR, sizeof(Smem), st>>>(P);
  else k_sample<float><<<grid, NTHR, sizeof(Smem), st>>>(P);
  return cudaGetLastError() == cudaSuccess ? VINFER_OK : VINFER_E_CUDA;
}

int launch_probs(const KParams& P, int dtype, cudaStream_t st) {
  if (!P.out_probs) return VINFER_OK;
  const int bx = (int)std::min<int64_t>(64, (P.V + 256 * 8 - 1) / (256 * 8));
  const dim3 grid(std::max(bx, 1), P.B);
  if (dtype == VINFER_DTYPE_BF16) k_probs<__nv_bfloat16><<<grid, 256, 0, st>>>(P);
  else k_probs<float><<<grid, 256, 0, st>>>(P);
  return cudaGetLastError() == cudaSuccess ? VINFER_OK : VINFER_E_CUDA;
}

}  // namespace

// ---------------------------------------------------------------------------------------------
// C ABI
// ---------------------------------------------------------------------------------------------
extern "C" {

int vinfer_sampler_abi_version(void) { return VINFER_SAMPLER_ABI_VERSION; }

size_t vinfer_sampler_workspace_bytes(int64_t batch, int64_t vocab, int32_t dtype) {
  if (batch < 1 || vocab < 1 || vocab > VINFER_MAX_VOCAB || batch > VINFER_MAX_BATCH) return 0;
  if (dtype != VINFER_DTYPE_F32 && dtype != VINFER_DTYPE_BF16) return 0;
  return ws_layout(batch, vocab, dtype).total;
}

int vinfer_sampler_workspace_init(void* workspace, size_t bytes, void* stream) {
  if (!workspace || bytes == 0) return VINFER_E_ARG;
  return cudaMemsetAsync(workspace, 0, bytes, (cudaStream_t)stream) == cudaSuccess
             ? VINFER_OK
             : VINFER_E_CUDA;
}

int vinfer_sample(const VinferSampleArgs* a, void* workspace, size_t workspace_bytes,
                  void* stream) {
  int rc = check_args(a);
  if (rc != VINFER_OK) return rc;
  if (a->vocab_offset != 0 || a->vocab_total != a->vocab) return VINFER_E_ARG;
  if (!workspace) return VINFER_E_ARG;
  if (workspace_bytes < ws_layout(a->batch, a->vocab, a->dtype).total) return VINFER_E_LIMIT;
  int ctas = 0;
  if (sample_ctas(a->dtype, &ctas) != VINFER_OK) return VINFER_E_CUDA;
  const Shape s = plan(a->batch, a->vocab, a->dtype, ctas);
  KParams P = make_params(a, s, workspace);
  P.mode = 0;
  cudaStream_t st = (cudaStream_t)stream;
  rc = launch_sample(P, a->dtype, st);
  if (rc != VINFER_OK) return rc;
  return launch_probs(P, a->dtype, st);
}

size_t vinfer_sample_record_bytes(int32_t record_cap) {
  if (record_cap < 1 || record_cap > CAND_CAP) return 0;
  return sizeof(RecHdr) + 8 * (size_t)record_cap;
}

int vinfer_sample_local(const VinferSampleArgs* a, int32_t record_cap, void* records,
                        void* workspace, size_t workspace_bytes, void* stream) {
  int rc = check_args(a);
  if (rc != VINFER_OK) return rc;
  if (!records || !workspace || record_cap < 1 || record_cap > CAND_CAP) return VINFER_E_ARG;
  if (workspace_bytes < ws_layout(a->batch, a->vocab, a->dtype).total) return VINFER_E_LIMIT;
  int ctas = 0;
  if (sample_ctas(a->dtype, &ctas) != VINFER_OK) return VINFER_E_CUDA;
  const Shape s = plan(a->batch, a->vocab, a->dtype, ctas);
  KParams P = make_params(a, s, workspace);
  P.mode = 1;
  P.shard_out = (unsigned char*)records;
  P.shard_cap = record_cap;
  P.shard_stride = vinfer_sample_record_bytes(record_cap);
  return launch_sample(P, a->dtype, (cudaStream_t)stream);
}

int vinfer_sample_merge(const VinferSampleArgs* a, int32_t record_cap, const void* records,
                        int32_t world_size, int32_t* unresolved, void* workspace,
                        size_t workspace_bytes, void* stream) {
  int rc = check_args(a);
  if (rc != VINFER_OK) return rc;
  if (!records || !workspace || world_size < 1 || world_size > MAX_NSEG || record_cap < 1 ||
      record_cap > CAND_CAP)
    return VINFER_E_ARG;
  if (world_size * record_cap > MERGE_CAP) return VINFER_E_LIMIT;
  if (workspace_bytes < ws_layout(a->batch, a->vocab, a->dtype).total) return VINFER_E_LIMIT;
  const Shape s = plan(a->batch, a->vocab, a->dtype, 1);
  KParams P = make_params(a, s, workspace);
  P.mode = 2;
  P.shard_cap = record_cap;
  P.shard_stride = vinfer_sample_record_bytes(record_cap);
  cudaStream_t st = (cudaStream_t)stream;
  const void* kern = a->dtype == VINFER_DTYPE_BF16 ? (const void*)k_merge<__nv_bfloat16>
                                                   : (const void*)k_merge<float>;
  int ctas = 0;
  if (kernel_info(kern, a->dtype == VINFER_DTYPE_BF16 ? 2 : 3, NT, &ctas) != VINFER_OK)
    return VINFER_E_CUDA;
  if (a->dtype == VINFER_DTYPE_BF16)
    k_merge<__nv_bfloat16><<<(unsigned)a->batch, NT, sizeof(Smem), st>>>(
        P, (const unsigned char*)records, world_size, unresolved);
  else
    k_merge<float><<<(unsigned)a->batch, NT, sizeof(Smem), st>>>(
        P, (const unsigned char*)records, world_size, unresolved);
  if (cudaGetLastError() != cudaSuccess) return VINFER_E_CUDA;
  return launch_probs(P, a->dtype, st);
}

}  // extern "C"

// The allocation-free entry point, vinfer_sample_static, runs on this fixed scratch array
// instead of a caller-allocated workspace. Every device that loads the library holds it until
// the process exits. Host code must not hand the symbol itself to a kernel: on the host it
// names a stand-in, not device memory. The device address comes from cudaGetSymbolAddress.
static __device__ __align__(256) unsigned char g_sample_scratch[VINFER_STATIC_SCRATCH_BYTES];

namespace {
std::mutex g_scratch_mu;
void* g_scratch_addr[64] = {};

// Device address of g_sample_scratch on the current device, looked up on the first call there
// (with that device current, as cudaGetSymbolAddress requires).
int static_scratch(void** out) {
  int dev = 0;
  if (cudaGetDevice(&dev) != cudaSuccess || dev < 0 || dev >= 64) return VINFER_E_CUDA;
  std::lock_guard<std::mutex> lock(g_scratch_mu);
  if (!g_scratch_addr[dev]) {
    void* p = nullptr;
    if (cudaGetSymbolAddress(&p, g_sample_scratch) != cudaSuccess || !p) return VINFER_E_CUDA;
    g_scratch_addr[dev] = p;
  }
  *out = g_scratch_addr[dev];
  return VINFER_OK;
}
}  // namespace

extern "C" {

// vinfer_sample without a caller workspace, for callers that cannot allocate device memory.
// Allocates nothing: the scratch is the static array above; only kernels and one
// cudaMemsetAsync are issued. Shapes whose workspace exceeds the array are refused with
// VINFER_E_LIMIT. All calls on a device share the array, so calls that overlap on the GPU race.
int vinfer_sample_static(const VinferSampleArgs* a, void* stream) {
  int rc = check_args(a);
  if (rc != VINFER_OK) return rc;
  if (a->vocab_offset != 0 || a->vocab_total != a->vocab) return VINFER_E_ARG;
  const WsLayout L = ws_layout(a->batch, a->vocab, a->dtype);
  if (L.total > sizeof(g_sample_scratch)) return VINFER_E_LIMIT;
  void* ws = nullptr;
  if (static_scratch(&ws) != VINFER_OK) return VINFER_E_CUDA;
  cudaStream_t st = (cudaStream_t)stream;
  // The per-row arrival counters must start at zero. The array keeps whatever the previous
  // call left, possibly for another shape whose records overlap these counters: clear them.
  if (cudaMemsetAsync((unsigned char*)ws + L.counters, 0, (size_t)a->batch * sizeof(int), st) !=
      cudaSuccess)
    return VINFER_E_CUDA;
  int ctas = 0;
  if (sample_ctas(a->dtype, &ctas) != VINFER_OK) return VINFER_E_CUDA;
  const Shape s = plan(a->batch, a->vocab, a->dtype, ctas);
  KParams P = make_params(a, s, ws);
  P.mode = 0;
  rc = launch_sample(P, a->dtype, st);
  if (rc != VINFER_OK) return rc;
  return launch_probs(P, a->dtype, st);
}

}  // extern "C"

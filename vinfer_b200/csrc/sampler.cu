// sampler.cu — fused token sampler for B200 (sm_100a).
//
// The path restated here is vinfer's reference sampler (src/vinfer/runtime/sampler.py:50-77):
// temperature, top-k (ties at the k-th value kept, :53-55), softmax (:56), top-p on the mass
// strictly before each token (:57-64), renormalisation, and one draw per row, extended with
// repetition / presence / frequency penalties, min-p and an inverse-CDF draw from a caller
// uniform. Tokens are ordered canonically: descending processed logit, ties by ascending id.
//
// Layout and passes (one launch of k_sample per batch):
//   * The grid is (segments, rows). A CTA owns one contiguous segment of one row (<= 32 KiB of
//     logits), copies it HBM -> shared memory with one TMA bulk copy, and reads HBM nowhere
//     else on the fast path.
//   * Penalised tokens of the segment (the row's CSR histogram entries in range) are taken out
//     of the resident copy (set to -inf) and kept as a side list of exact float32 values.
//   * One pass over shared memory computes, per group of 16 bytes x 2 vectors, the group
//     maximum, and (top-k off) an online softmax max/sum. The K-th largest group maximum is a
//     lower bound of the K-th largest value, so only groups at or above it are rescanned to
//     collect candidates; an exact radix select on them gives the segment's top-K with all
//     ties. The segment record (candidates, max, sum, completeness threshold) goes to the
//     workspace.
//   * The last CTA of a row to finish (threadfence + atomic counter) merges the records:
//     bitonic sort into canonical order, top-k, top-p and min-p cuts by prefix sums, and the
//     draw. A row whose cut or draw lies below what the records hold completely, or whose
//     candidates overflowed, is finished by an exact multi-pass search over the row (radix
//     histograms of mass in 2^-44 fixed point, ties resolved in id order) in the same CTA.
//
// All reductions run in a fixed order, so results are deterministic run to run.

#include <cuda_runtime.h>
#include <cuda_bf16.h>
#include <stdint.h>
#include <float.h>
#include <math.h>

#include <algorithm>

#include "vinfer_sampler.h"

namespace {

// ---------------------------------------------------------------------------------------------
// configuration
// ---------------------------------------------------------------------------------------------
constexpr int NT = 256;                 // threads per CTA
constexpr int NWARP = NT / 32;
constexpr int SEG_BYTES = 32768;        // largest segment held in shared memory
constexpr int SBUF_BYTES = SEG_BYTES + 64;
constexpr int CAND_CAP = 1024;          // candidates collected per segment
constexpr int SIDE_CAP = 2048;          // penalised tokens per segment
constexpr int KMAX = 256;               // largest top-k served by the candidate path
constexpr int KC = 128;                 // candidates kept per segment when top-k is off
constexpr int MAX_NSEG = 32;
constexpr int GROUP_VECS = 2;           // 16-byte vectors per group
constexpr int MAX_VEC = SBUF_BYTES / 16;
constexpr int MAX_R = (MAX_VEC + NT - 1) / NT;
constexpr int MAX_GSLOT = ((MAX_R + GROUP_VECS - 1) / GROUP_VECS) * NT;
constexpr int SIDE_GROUP = 8;
constexpr int MAX_SGROUP = SIDE_CAP / SIDE_GROUP;
constexpr int MERGE_CAP = SBUF_BYTES / 8 / 2 * 2 >= 4096 ? 4096 : 0;
constexpr int BM_WORDS = SEG_BYTES / 2 / 32 + 8;
constexpr int FB_BINS = 2048;           // radix bins of the exact search (11 + 11 + 10 bits)
constexpr float LOG2E = 1.4426950408889634f;
constexpr double FX_ONE = 17592186044416.0;  // 2^44: fixed-point unit of probability mass
constexpr long long WAIT_CYCLES = 4000000000LL;  // ~2 s at 2 GHz: bound on any wait

static_assert(MERGE_CAP == 4096, "merge buffer must hold 4096 entries");
static_assert((size_t)VINFER_MAX_VOCAB / 8 <= (size_t)SBUF_BYTES, "row bitmap must fit");

// record flags
constexpr uint32_t REC_UNRETAINED = 1u;  // elements below t_key exist that are not listed
constexpr uint32_t REC_OVERFLOW = 2u;    // candidates did not fit: the row needs the exact search
constexpr uint32_t REC_BAD = 4u;         // invalid parameters
constexpr uint32_t REC_EXACT = 8u;       // the row is resolved by the exact search

struct RecHdr {
  float m_y;        // largest penalised logit of the source (pre-temperature)
  float s;          // sum of exp2((y - m_y) * log2(e) / T) over the source (top-k off only)
  uint32_t t_key;   // every element with key >= t_key is listed
  int32_t n;        // listed entries
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
  int B, nseg, seg_len, mode;  // mode 0: finalize, 1: local (write shard records)
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

// shared memory of k_sample; the merge and the exact search reuse the same bytes
struct __align__(16) Smem {
  unsigned char sbuf[SBUF_BYTES];             // segment / merge entries / row bitmap
  uint32_t gkey[MAX_GSLOT + MAX_SGROUP];      // group maxima (keys)
  uint32_t ckey[CAND_CAP];                    // candidate keys    } exact search: counts
  int32_t cid[CAND_CAP];                      // candidate ids     }
  int32_t side_li[SIDE_CAP];                  // penalised: local index } exact search: masses
  float side_y[SIDE_CAP];                     // penalised: value       }
  uint32_t bitmap[BM_WORDS];                  // penalised positions of the segment
  uint32_t hist[256];
  unsigned long long red64[NWARP + 1];
  float redf[2 * NWARP + 2];
  int32_t redi[NWARP + 2];
  int32_t sc[16];
  float sf[8];
  unsigned long long mbar;
};

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

// ---- TMA bulk copy (global -> shared) with an mbarrier, waits bounded -----------------------
__device__ __forceinline__ void mbar_init(unsigned long long* bar, uint32_t count) {
  asm volatile("mbarrier.init.shared::cta.b64 [%0], %1;" ::"r"(smem_u32(bar)), "r"(count)
               : "memory");
  asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
}
__device__ __forceinline__ void mbar_expect_tx(unsigned long long* bar, uint32_t bytes) {
  asm volatile("mbarrier.arrive.expect_tx.shared::cta.b64 _, [%0], %1;" ::"r"(smem_u32(bar)),
               "r"(bytes)
               : "memory");
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
__device__ bool mbar_wait_bounded(unsigned long long* bar, uint32_t parity) {
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
  __device__ static float sm(const void* s, int i) { return ((const float*)s)[i]; }
  __device__ static void neg_inf(void* s, int i) { ((uint32_t*)s)[i] = 0xFF800000u; }
  __device__ static void copy(void* s, int i, const void* p, int64_t j) {
    ((float*)s)[i] = __ldg((const float*)p + j);
  }
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
  __device__ static float sm(const void* s, int i) {
    return __uint_as_float((uint32_t)((const unsigned short*)s)[i] << 16);
  }
  __device__ static void neg_inf(void* s, int i) { ((unsigned short*)s)[i] = 0xFF80u; }
  __device__ static void copy(void* s, int i, const void* p, int64_t j) {
    ((unsigned short*)s)[i] = __ldg((const unsigned short*)p + j);
  }
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

// ---------------------------------------------------------------------------------------------
// per-row configuration
// ---------------------------------------------------------------------------------------------
struct RowCfg {
  float T, c2, p, minp, lm, rep, pres, freq, u;
  int k, K;
  bool greedy, topk, need_sum, pen, bad, exact;
};

__device__ RowCfg load_row(const KParams& P, int row) {
  RowCfg c;
  c.T = P.temperature ? P.temperature[row] : 1.f;
  c.k = P.top_k ? P.top_k[row] : 0;
  c.p = P.top_p ? P.top_p[row] : 1.f;
  c.minp = P.min_p ? P.min_p[row] : 0.f;
  c.rep = P.rep ? P.rep[row] : 1.f;
  c.pres = P.pres ? P.pres[row] : 0.f;
  c.freq = P.freq ? P.freq[row] : 0.f;
  c.u = P.uni ? P.uni[row] : 0.f;
  c.greedy = (c.T == 0.f);
  bool bad = !(c.T >= 0.f && c.T <= FLT_MAX) || !(c.p > 0.f && c.p <= 1.f) || c.k < 0 ||
             !(c.minp >= 0.f && c.minp <= 1.f) || !(c.rep > 0.f && c.rep <= FLT_MAX) ||
             !(fabsf(c.pres) <= FLT_MAX) || !(fabsf(c.freq) <= FLT_MAX);
  if (!c.greedy) bad = bad || P.uni == nullptr || !(c.u >= 0.f && c.u < 1.f);
  c.bad = bad;
  c.topk = !c.greedy && c.k > 0 && (int64_t)c.k < P.vtotal;
  c.K = c.greedy ? 1 : (c.topk ? c.k : KC);
  c.need_sum = !c.greedy && !c.topk;
  c.exact = (P.flags & VINFER_FLAG_EXACT_ALL) != 0 || (c.topk && c.k > KMAX);
  c.c2 = c.greedy ? 0.f : __fdiv_rn(LOG2E, c.T);
  c.lm = c.minp > 0.f ? log2f(c.minp) : -INFINITY;
  c.pen = P.hrow != nullptr && (c.rep != 1.f || c.pres != 0.f || c.freq != 0.f);
  return c;
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
// smallest y with vf(y) >= vt, given vf(yhi) >= vt (binary search over ordered keys)
__device__ float preimage_lo(float vt, float yhi, const RowCfg& c) {
  if (c.greedy || vt == -INFINITY) return vt;
  uint32_t lo = okey(-INFINITY), hi = okey(yhi);
  if (vf(from_okey(lo), c) >= vt) return -INFINITY;
  while (hi - lo > 1) {
    const uint32_t mid = lo + (hi - lo) / 2;
    if (vf(from_okey(mid), c) >= vt) hi = mid; else lo = mid;
  }
  return from_okey(hi);
}

// first index >= target in the ascending ids[a, b)
__device__ int64_t lower_bound_ids(const int* ids, int64_t a, int64_t b, int64_t target) {
  while (a < b) {
    const int64_t mid = a + (b - a) / 2;
    if ((int64_t)__ldg(ids + mid) < target) a = mid + 1; else b = mid;
  }
  return a;
}

// ---------------------------------------------------------------------------------------------
// block-wide building blocks (all threads of the CTA call them)
// ---------------------------------------------------------------------------------------------
// exclusive scan of one float per thread, in thread order; returns the total too
__device__ float block_excl_scan_f(float x, float* total, Smem& S) {
  const int lane = threadIdx.x & 31, w = threadIdx.x >> 5;
  float inc = x;
#pragma unroll
  for (int o = 1; o < 32; o <<= 1) {
    const float t = __shfl_up_sync(0xffffffffu, inc, o);
    if (lane >= o) inc += t;
  }
  __syncthreads();
  if (lane == 31) S.redf[w] = inc;
  __syncthreads();
  if (threadIdx.x == 0) {
    float run = 0.f;
    for (int i = 0; i < NWARP; ++i) {
      const float t = S.redf[i];
      S.redf[i] = run;
      run += t;
    }
    S.redf[NWARP] = run;
  }
  __syncthreads();
  const float r = S.redf[w] + inc - x;
  *total = S.redf[NWARP];
  return r;
}
__device__ unsigned long long block_excl_scan_u64(unsigned long long x, unsigned long long* total,
                                                  Smem& S) {
  const int lane = threadIdx.x & 31, w = threadIdx.x >> 5;
  unsigned long long inc = x;
#pragma unroll
  for (int o = 1; o < 32; o <<= 1) {
    const unsigned long long t = __shfl_up_sync(0xffffffffu, inc, o);
    if (lane >= o) inc += t;
  }
  __syncthreads();
  if (lane == 31) S.red64[w] = inc;
  __syncthreads();
  if (threadIdx.x == 0) {
    unsigned long long run = 0;
    for (int i = 0; i < NWARP; ++i) {
      const unsigned long long t = S.red64[i];
      S.red64[i] = run;
      run += t;
    }
    S.red64[NWARP] = run;
  }
  __syncthreads();
  const unsigned long long r = S.red64[w] + inc - x;
  *total = S.red64[NWARP];
  return r;
}
__device__ int block_excl_scan_i(int x, int* total, Smem& S) {
  const int lane = threadIdx.x & 31, w = threadIdx.x >> 5;
  int inc = x;
#pragma unroll
  for (int o = 1; o < 32; o <<= 1) {
    const int t = __shfl_up_sync(0xffffffffu, inc, o);
    if (lane >= o) inc += t;
  }
  __syncthreads();
  if (lane == 31) S.redi[w] = inc;
  __syncthreads();
  if (threadIdx.x == 0) {
    int run = 0;
    for (int i = 0; i < NWARP; ++i) {
      const int t = S.redi[i];
      S.redi[i] = run;
      run += t;
    }
    S.redi[NWARP] = run;
  }
  __syncthreads();
  const int r = S.redi[w] + inc - x;
  *total = S.redi[NWARP];
  return r;
}
__device__ unsigned long long block_min_u64(unsigned long long x, Smem& S) {
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) {
    const unsigned long long t = __shfl_xor_sync(0xffffffffu, x, o);
    x = t < x ? t : x;
  }
  __syncthreads();
  if ((threadIdx.x & 31) == 0) S.red64[threadIdx.x >> 5] = x;
  __syncthreads();
  if (threadIdx.x == 0) {
    unsigned long long m = S.red64[0];
    for (int i = 1; i < NWARP; ++i) m = S.red64[i] < m ? S.red64[i] : m;
    S.red64[NWARP] = m;
  }
  __syncthreads();
  return S.red64[NWARP];
}
__device__ uint32_t block_max_u32(uint32_t x, Smem& S) {
  unsigned long long y = ~(unsigned long long)x;  // max via min of complements
  return (uint32_t)~block_min_u64(y, S);
}
__device__ unsigned long long block_sum_u64(unsigned long long x, Smem& S) {
  unsigned long long tot;
  block_excl_scan_u64(x, &tot, S);
  return tot;
}

// K-th largest of keys[0, n) (1 <= K <= n): exact radix select, 8-bit digits from the top.
// *rank_in_ties receives how many elements equal to the result are needed to reach K.
__device__ uint32_t block_kth_largest(const uint32_t* keys, int n, int K, Smem& S,
                                      int* rank_in_ties = nullptr) {
  uint32_t prefix = 0;
  int need = K;
#pragma unroll 1
  for (int pass = 0; pass < 4; ++pass) {
    const int shift = 24 - 8 * pass;
    const uint32_t hmask = pass == 0 ? 0u : (0xFFFFFFFFu << (shift + 8));
    S.hist[threadIdx.x] = 0;  // NT == 256 bins
    __syncthreads();
    for (int i = threadIdx.x; i < n; i += NT) {
      const uint32_t k = keys[i];
      if ((k & hmask) == prefix) atomicAdd(&S.hist[(k >> shift) & 255u], 1u);
    }
    __syncthreads();
    // thread t owns digit 255 - t: exclusive scan of counts from the top digit down
    const int d = 255 - (int)threadIdx.x;
    const int cnt = (int)S.hist[d];
    int tot;
    const int above = block_excl_scan_i(cnt, &tot, S);
    if (above < need && above + cnt >= need) {
      S.sc[14] = d;
      S.sc[15] = need - above;
    }
    __syncthreads();
    prefix |= (uint32_t)S.sc[14] << shift;
    need = S.sc[15];
    __syncthreads();
  }
  if (rank_in_ties) *rank_in_ties = need;
  return prefix;
}

// ascending bitonic sort of e[0, n), n a power of two
__device__ void block_bitonic_sort(unsigned long long* e, int n) {
  for (int k = 2; k <= n; k <<= 1) {
    for (int j = k >> 1; j > 0; j >>= 1) {
      for (int i = threadIdx.x; i < n; i += NT) {
        const int ixj = i ^ j;
        if (ixj > i) {
          const unsigned long long a = e[i], b = e[ixj];
          const bool up = (i & k) == 0;
          if ((a > b) == up) {
            e[i] = b;
            e[ixj] = a;
          }
        }
      }
      __syncthreads();
    }
  }
}

// ---------------------------------------------------------------------------------------------
// the segment pass: one CTA, one segment of one row -> one record
// ---------------------------------------------------------------------------------------------
template <typename TIn>
__device__ void segment_pass(const KParams& P, const RowCfg& c, int row, int seg, Smem& S,
                             unsigned char* rec) {
  using E = Elem<TIn>;
  constexpr int A = E::A;
  constexpr int ES = 16 / A;
  const int tid = threadIdx.x;
  const int64_t lo = (int64_t)seg * P.seg_len;
  const int64_t hi = min(P.V, lo + (int64_t)P.seg_len);
  const int n = (int)(hi - lo);
  const TIn* rowp = (const TIn*)P.logits + (int64_t)row * P.ld;
  const int64_t gbase = P.voff + lo;  // global id of local index 0

  // ---- 1. stage the segment in shared memory: 16-byte-aligned interior by TMA, edges by hand
  const uintptr_t gaddr = (uintptr_t)(rowp + lo);
  int head = (int)(((16u - (uint32_t)(gaddr & 15u)) & 15u) / ES);
  if (head > n) head = n;
  const int inter = (int)((((int64_t)(n - head) * ES) / 16) * 16 / ES);
  const int tail0 = head + inter;
  const int off = (A - head % A) % A;  // local index i lives at slot off + i
  const int nvec = (off + n + A - 1) / A;
  void* sv = S.sbuf;
  if (tid == 0) {
    mbar_init(&S.mbar, 1);
  }
  __syncthreads();
  if (tid == 0 && inter > 0) {
    const uint32_t bytes = (uint32_t)inter * ES;
    mbar_expect_tx(&S.mbar, bytes);
    for (uint32_t b = 0; b < bytes; b += 16384u) {
      const uint32_t len = min(16384u, bytes - b);
      tma_load_1d(S.sbuf + (size_t)(off + head) * ES + b,
                  (const unsigned char*)(rowp + lo + head) + b, len, &S.mbar);
    }
  }
  if (tid < off) E::neg_inf(sv, tid);
  const int pad_end = nvec * A - (off + n);
  if (tid < pad_end) E::neg_inf(sv, off + n + tid);
  if (tid < head) E::copy(sv, off + tid, rowp, lo + tid);
  if (tid < n - tail0) E::copy(sv, off + tail0 + tid, rowp, lo + tail0 + tid);
  const int nwords = (nvec * A + 31) / 32;
  for (int w = tid; w < nwords; w += NT) S.bitmap[w] = 0u;

  // ---- 2. this segment's history entries (ids ascending within the row)
  if (tid == 0) {
    int64_t sa = 0, sb = 0;
    if (c.pen) {
      const int64_t a = P.hrow[row], b = P.hrow[row + 1];
      sa = lower_bound_ids(P.hids, a, b, gbase);
      sb = lower_bound_ids(P.hids, sa, b, gbase + n);
    }
    S.sc[0] = (int)(sb - sa);
    S.sc[1] = (int)sa;
    S.sc[2] = 0;  // candidate counter
    S.sc[3] = 0;  // retained counter
  }
  // wait for the bulk copy (every thread observes the barrier phase itself)
  bool ok = true;
  if (inter > 0) ok = mbar_wait_bounded(&S.mbar, 0);
  if (__syncthreads_or(!ok)) {
    // the copy may still be in flight: wait once more, bounded, before touching anything
    if (inter > 0) mbar_wait_bounded(&S.mbar, 0);
    if (tid == 0) status_or(P, VINFER_ST_TIMEOUT);
    RecHdr* h = (RecHdr*)rec;
    if (tid == 0) { h->n = 0; h->flags = REC_OVERFLOW; h->t_key = 0; h->m_y = -INFINITY; h->s = 0.f; }
    return;
  }
  const int ns_all = S.sc[0];
  const int sbase = S.sc[1];
  const bool side_over = ns_all > SIDE_CAP;
  const int ns = side_over ? 0 : ns_all;
  for (int j = tid; j < ns; j += NT) {
    const int li = (int)((int64_t)__ldg(P.hids + sbase + j) - gbase);
    const int cnt = __ldg(P.hcnt + sbase + j);
    if (cnt > 0) {
      const int slot = off + li;
      S.side_li[j] = li;
      S.side_y[j] = penalize(E::sm(sv, slot), cnt, c);
      atomicOr(&S.bitmap[slot >> 5], 1u << (slot & 31));
      E::neg_inf(sv, slot);
    } else {
      S.side_li[j] = -1;
      S.side_y[j] = -INFINITY;
    }
  }
  __syncthreads();

  RecHdr* hdr = (RecHdr*)rec;
  unsigned long long* ent = (unsigned long long*)(rec + sizeof(RecHdr));
  if (side_over) {  // more penalised tokens than the side list holds: exact search
    if (tid == 0) { hdr->n = 0; hdr->flags = REC_OVERFLOW; hdr->t_key = 0; hdr->m_y = -INFINITY; hdr->s = 0.f; }
    return;
  }

  // ---- 3. one pass over shared memory: group maxima, online softmax sum, greedy argmax
  const uint4* sv4 = (const uint4*)S.sbuf;
  const int R = (nvec + NT - 1) / NT;
  const int ngs = (R + GROUP_VECS - 1) / GROUP_VECS;
  float m_t = -FLT_MAX, s_t = 0.f;
  float best = -INFINITY;
  int best_i = 0x7FFFFFFF;
  float segmax = -INFINITY;
  for (int g = 0; g < ngs; ++g) {
    float gmx = -INFINITY;
#pragma unroll
    for (int rr = 0; rr < GROUP_VECS; ++rr) {
      const int j = tid + (g * GROUP_VECS + rr) * NT;
      if (j < nvec) {
        const uint4 q = sv4[j];
        const float vm = E::vmax(q);
        gmx = fmaxf(gmx, vm);
        if (c.need_sum) {
          if (vm > m_t) {
            s_t *= ex2((m_t - vm) * c.c2);
            m_t = vm;
          }
#pragma unroll
          for (int e = 0; e < A; ++e) s_t += ex2((E::at(q, e) - m_t) * c.c2);
        }
        if (c.greedy && vm > best) {
          int e = 0;
          while (e < A - 1 && E::at(q, e) != vm) ++e;
          best = vm;
          best_i = j * A + e - off;
        }
      }
    }
    S.gkey[g * NT + tid] = okey(gmx);
    segmax = fmaxf(segmax, gmx);
  }
  // penalised tokens: singleton values in the side list, grouped by eight
  const int nsg = (ns + SIDE_GROUP - 1) / SIDE_GROUP;
  for (int sg = tid; sg < nsg; sg += NT) {
    float gmx = -INFINITY;
    for (int j = sg * SIDE_GROUP; j < min(ns, (sg + 1) * SIDE_GROUP); ++j) {
      const float y = S.side_y[j];
      gmx = fmaxf(gmx, y);
      if (c.need_sum && S.side_li[j] >= 0) {
        if (y > m_t) {
          s_t *= ex2((m_t - y) * c.c2);
          m_t = y;
        }
        s_t += ex2((y - m_t) * c.c2);
      }
      if (c.greedy && S.side_li[j] >= 0 &&
          (y > best || (y == best && S.side_li[j] < best_i))) {
        best = y;
        best_i = S.side_li[j];
      }
    }
    S.gkey[ngs * NT + sg] = okey(gmx);
    segmax = fmaxf(segmax, gmx);
  }
  const uint32_t segmax_key = block_max_u32(okey(segmax), S);
  const float m_seg = from_okey(segmax_key);

  float s_seg = 0.f;
  if (c.need_sum) {  // rescale every partial to the segment maximum, fixed order
    const float part = (m_t == -FLT_MAX) ? 0.f : s_t * ex2((m_t - m_seg) * c.c2);
    float tot;
    block_excl_scan_f(part, &tot, S);
    s_seg = tot;
  }

  if (c.greedy) {  // one entry: the first index of the maximum
    const uint32_t k = okey(best);
    const unsigned long long mine =
        (best_i == 0x7FFFFFFF) ? ~0ull : comp(k, (int)(gbase + best_i));
    const unsigned long long w = block_min_u64(mine, S);
    if (tid == 0) {
      hdr->m_y = m_seg;
      hdr->s = 0.f;
      hdr->t_key = 0;
      hdr->flags = n > 1 ? REC_UNRETAINED : 0u;
      hdr->n = (w == ~0ull) ? 0 : 1;
      if (w != ~0ull) {
        ent[0] = w;
        hdr->t_key = comp_key(w);
      }
    }
    return;
  }

  // ---- 4. threshold: the K-th largest group maximum bounds the K-th largest value from below
  const int nkeys = ngs * NT + nsg;
  uint32_t gk = 0;
  if (c.K <= nkeys) gk = block_kth_largest(S.gkey, nkeys, c.K, S);
  if (tid == 0) {
    float ylo = -INFINITY;
    if (gk > okey(-INFINITY)) {
      const float g = from_okey(gk);
      ylo = preimage_lo(vf(g, c), g, c);
    }
    S.sf[0] = ylo;
  }
  __syncthreads();
  const float ylo = S.sf[0];
  const uint32_t ylo_key = okey(ylo);

  // ---- 5. rescan qualifying groups: every element with vf(y) >= vf(g) becomes a candidate
  for (int g = 0; g < ngs; ++g) {
    if (S.gkey[g * NT + tid] < ylo_key) continue;
    for (int rr = 0; rr < GROUP_VECS; ++rr) {
      const int j = tid + (g * GROUP_VECS + rr) * NT;
      if (j >= nvec) break;
      const uint4 q = sv4[j];
#pragma unroll 1
      for (int e = 0; e < A; ++e) {
        const int slot = j * A + e;
        const int li = slot - off;
        if (li < 0 || li >= n) continue;
        if (S.bitmap[slot >> 5] & (1u << (slot & 31))) continue;
        const float y = E::at(q, e);
        if (!(y >= ylo)) continue;
        const int pos = atomicAdd(&S.sc[2], 1);
        if (pos < CAND_CAP) {
          S.ckey[pos] = okey(vf(y, c));
          S.cid[pos] = (int)(gbase + li);
        }
      }
    }
  }
  for (int sg = tid; sg < nsg; sg += NT) {
    if (S.gkey[ngs * NT + sg] < ylo_key) continue;
    for (int j = sg * SIDE_GROUP; j < min(ns, (sg + 1) * SIDE_GROUP); ++j) {
      if (S.side_li[j] < 0 || !(S.side_y[j] >= ylo)) continue;
      const int pos = atomicAdd(&S.sc[2], 1);
      if (pos < CAND_CAP) {
        S.ckey[pos] = okey(vf(S.side_y[j], c));
        S.cid[pos] = (int)(gbase + S.side_li[j]);
      }
    }
  }
  __syncthreads();
  const int nc_all = S.sc[2];
  if (nc_all > CAND_CAP) {
    if (tid == 0) { hdr->n = 0; hdr->flags = REC_OVERFLOW; hdr->t_key = 0; hdr->m_y = m_seg; hdr->s = s_seg; }
    return;
  }
  const int nc = nc_all;

  // ---- 6. exact K-th largest among candidates; keep everything at or above it (all ties)
  uint32_t tk = 0;
  if (nc >= c.K) tk = block_kth_largest(S.ckey, nc, c.K, S);
  for (int i = tid; i < nc; i += NT) {
    if (S.ckey[i] >= tk) {
      const int pos = atomicAdd(&S.sc[3], 1);
      ent[pos] = comp(S.ckey[i], S.cid[i]);
    }
  }
  __syncthreads();
  if (tid == 0) {
    const int nr = S.sc[3];
    hdr->m_y = m_seg;
    hdr->s = s_seg;
    hdr->n = nr;
    hdr->t_key = tk;
    hdr->flags = (nr < n) ? REC_UNRETAINED : 0u;
  }
}

// ---------------------------------------------------------------------------------------------
// merge: records -> canonical order -> cuts and draw
// ---------------------------------------------------------------------------------------------
struct MergeIn {
  float m_y, s;
  uint32_t d_key;  // every element with key >= d_key is among the entries
  uint32_t flags;
  int n;
};

// Gather the records of one row (nsrc sources at src0 + i * src_stride) into S.sbuf, sorted.
__device__ MergeIn gather_records(const unsigned char* src0, size_t src_stride, int nsrc,
                                  const RowCfg& c, Smem& S) {
  unsigned long long* e = (unsigned long long*)S.sbuf;
  int* offs = (int*)S.gkey;  // [nsrc + 1]
  if (threadIdx.x == 0) {
    float m_y = -INFINITY;
    for (int i = 0; i < nsrc; ++i) {
      const RecHdr* h = (const RecHdr*)(src0 + (size_t)i * src_stride);
      m_y = fmaxf(m_y, __ldcg(&h->m_y));
    }
    float s = 0.f;
    uint32_t d = 0, fl = 0;
    int tot = 0;
    for (int i = 0; i < nsrc; ++i) {
      const RecHdr* h = (const RecHdr*)(src0 + (size_t)i * src_stride);
      const uint32_t f = __ldcg(&h->flags);
      const int n = __ldcg(&h->n);
      const float hm = __ldcg(&h->m_y);
      if (c.need_sum && hm > -INFINITY) s += __ldcg(&h->s) * ex2((hm - m_y) * c.c2);
      if (f & REC_UNRETAINED) d = max(d, __ldcg(&h->t_key));
      fl |= f;
      offs[i] = tot;
      tot += n;
    }
    offs[nsrc] = tot;
    S.sf[1] = m_y;
    S.sf[2] = s;
    S.sc[4] = (int)d;
    S.sc[5] = (int)fl;
    S.sc[6] = tot;
  }
  __syncthreads();
  MergeIn m;
  m.m_y = S.sf[1];
  m.s = S.sf[2];
  m.d_key = (uint32_t)S.sc[4];
  m.flags = (uint32_t)S.sc[5];
  m.n = S.sc[6];
  if ((m.flags & (REC_OVERFLOW | REC_BAD | REC_EXACT)) || m.n > MERGE_CAP) return m;
  for (int i = 0; i < nsrc; ++i) {
    const unsigned char* r = src0 + (size_t)i * src_stride;
    const unsigned long long* re = (const unsigned long long*)(r + sizeof(RecHdr));
    const int n = offs[i + 1] - offs[i];
    for (int j = threadIdx.x; j < n; j += NT) e[offs[i] + j] = __ldcg(re + j);
  }
  int np = 1;
  while (np < m.n) np <<= 1;
  for (int j = m.n + threadIdx.x; j < np; j += NT) e[j] = ~0ull;
  __syncthreads();
  block_bitonic_sort(e, np);
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

// Finalize one row from sorted entries. Returns false when the row must take the exact search.
__device__ bool finalize_sorted(const KParams& P, const RowCfg& c, int row, const MergeIn& m,
                                Smem& S) {
  const unsigned long long* e = (const unsigned long long*)S.sbuf;
  const int tid = threadIdx.x;
  if (m.n == 0) {
    if (tid == 0) {
      P.out_ids[row] = -1;
      status_or(P, VINFER_ST_NONFINITE);
      RowState st = {};
      st.kind = 3;
      st.token = -1;
      P.rows[row] = st;
    }
    return true;
  }
  if (c.greedy) {
    if (tid == 0) {
      const int tok = comp_id(e[0]);
      P.out_ids[row] = tok;
      RowState st = {};
      st.kind = 2;
      st.token = tok;
      P.rows[row] = st;
    }
    return true;
  }
  const float mv = from_okey(comp_key(e[0]));
  if (!(mv > -INFINITY) || !(mv <= FLT_MAX)) {
    if (tid == 0) {
      P.out_ids[row] = -1;
      status_or(P, VINFER_ST_NONFINITE);
      RowState st = {};
      st.kind = 3;
      st.token = -1;
      P.rows[row] = st;
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
  const float pre = block_excl_scan_f(loc, &total, S);
  const float Ssum = c.topk ? total : m.s;
  const bool listed_all = c.topk || !more;  // every kept-by-top-k token is among the entries

  // first index in [0, lim) whose inclusive prefix C_j satisfies C_j >= t (ge) or C_j > t
  auto first_cross = [&](float t, bool ge, int lim) -> int {
    int hit = 0x7FFFFFFF;
    float run = pre;
    for (int j = j0; j < min(j1, lim); ++j) {
      run += ex2((from_okey(comp_key(e[j])) - mv) * LOG2E);
      if (ge ? (run >= t) : (run > t)) { hit = j; break; }
    }
    return (int)block_min_u64((unsigned long long)(unsigned)hit, S);
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
      if ((from_okey(comp_key(e[j])) - mv) * LOG2E < c.lm) { hit = j; break; }
    hit = (int)block_min_u64((unsigned long long)(unsigned)hit, S);
    if (hit != 0x7FFFFFFF) L = min(L, max(hit, 1));
    else if (!listed_all) cut_beyond = true;
  }
  const bool L_known = L <= avail;
  if (!L_known && cut_beyond) return false;  // the cut needs elements the records do not hold
  // kept-set mass
  float s_kept;
  if (L_known) {
    if (tid == 0) S.sf[3] = 0.f;
    __syncthreads();
    const int last = L - 1;
    if (last >= j0 && last < j1) {
      float run = pre;
      for (int j = j0; j <= last; ++j) run += ex2((from_okey(comp_key(e[j])) - mv) * LOG2E);
      S.sf[3] = run;
    }
    __syncthreads();
    s_kept = S.sf[3];
  } else {
    s_kept = Ssum;  // no cut at all: the kept set is every token
  }
  const int lim = L_known ? min(L, avail) : avail;
  int j = first_cross(c.u * s_kept, false, lim);
  if (j == 0x7FFFFFFF) {
    if (L_known && L <= avail) j = L - 1;
    else return false;
  }
  if (tid == 0) {
    const int tok = comp_id(e[j]);
    P.out_ids[row] = tok;
    RowState st = {};
    st.m_v = mv;
    st.s_kept = s_kept;
    st.token = tok;
    if (L_known) {
      st.kind = 0;
      st.cut_key = comp_key(e[L - 1]);
      st.cut_id = comp_id(e[L - 1]);
    } else {
      st.kind = 1;
    }
    P.rows[row] = st;
  }
  return true;
}

// ---------------------------------------------------------------------------------------------
// exact multi-pass search over one row (global memory), for rows the records cannot resolve
// ---------------------------------------------------------------------------------------------
template <typename TIn>
struct ExactRow {
  const KParams& P;
  const RowCfg& c;
  Smem& S;
  const TIn* rowp;
  int64_t hist_a, hist_b;
  int V;
  float mv;
  uint32_t tk;  // kept by top-k: key >= tk

  __device__ bool pen_bit(int i) const {
    const uint32_t* bm = (const uint32_t*)S.sbuf;
    return (bm[i >> 5] >> (i & 31)) & 1u;
  }
  __device__ float y_at(int i) const {
    float x = Elem<TIn>::ld(rowp, i);
    if (c.pen && pen_bit(i)) {
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

// kept-set predicate of the exact search
struct Cut {
  uint32_t tk;       // top-k: key >= tk
  int kind;          // 0: (key > ck) or (key == ck and i <= cid); 1: all
  uint32_t ck;
  int cid;
  uint32_t mk;       // min-p: key >= mk
  __device__ bool keep(uint32_t key, int i) const {
    if (key < tk || key < mk) return false;
    if (kind == 1) return true;
    return key > ck || (key == ck && i <= cid);
  }
};

struct Found {
  uint32_t w;                 // key of the tie group reached
  unsigned long long above;   // fixed-point mass strictly above w (kept elements)
  int j;                      // 1-based rank inside the tie group, ascending id
  int n_w;
};

template <typename TIn>
__device__ Found exact_search(ExactRow<TIn>& X, const Cut& cut, unsigned long long target,
                              bool strict) {
  Smem& S = X.S;
  static_assert(FB_BINS * 4 <= sizeof(Smem::ckey) + sizeof(Smem::cid), "count bins fit");
  static_assert(FB_BINS * 8 <= sizeof(Smem::side_li) + sizeof(Smem::side_y), "mass bins fit");
  uint32_t* cnt = (uint32_t*)S.ckey;                // FB_BINS counts (ckey + cid region)
  unsigned long long* mass = (unsigned long long*)S.side_li;  // FB_BINS masses
  uint32_t prefix = 0;
  unsigned long long above = 0;
  int last_cnt = 0;
  const int shifts[3] = {21, 10, 0};
  const int bitsv[3] = {11, 11, 10};
#pragma unroll 1
  for (int lv = 0; lv < 3; ++lv) {
    const int sh = shifts[lv], nb = 1 << bitsv[lv];
    for (int b = threadIdx.x; b < nb; b += NT) { cnt[b] = 0; mass[b] = 0ull; }
    __syncthreads();
    for (int i = threadIdx.x; i < X.V; i += NT) {
      const uint32_t key = X.key_at(i);
      if (!cut.keep(key, i)) continue;
      if (lv > 0 && (key >> (sh + bitsv[lv])) != prefix) continue;
      const uint32_t b = (key >> sh) & (uint32_t)(nb - 1);
      atomicAdd(&cnt[b], 1u);
      atomicAdd(&mass[b], X.wfx(key));
    }
    __syncthreads();
    // bins in descending order; thread t owns nb / NT consecutive ones
    const int per = nb / NT;
    const int b_hi = nb - 1 - threadIdx.x * per;
    unsigned long long mine = 0;
    for (int q = 0; q < per; ++q) mine += mass[b_hi - q];
    unsigned long long tot;
    const unsigned long long ex = block_excl_scan_u64(mine, &tot, S);
    unsigned long long hit = ~0ull;
    {
      unsigned long long run = above + ex;
      for (int q = 0; q < per; ++q) {
        const int b = b_hi - q;
        if (cnt[b] == 0) continue;
        const unsigned long long nxt = run + mass[b];
        if (strict ? (nxt > target) : (nxt >= target)) {
          hit = ((unsigned long long)(threadIdx.x * per + q) << 32) | (unsigned)b;
          break;
        }
        run = nxt;
      }
    }
    hit = block_min_u64(hit, S);
    if (hit == ~0ull) {
      // target at or beyond the total (rounding): take the lowest non-empty bin
      unsigned long long lowb = ~0ull;
      for (int q = 0; q < per; ++q) {
        const int b = b_hi - q;
        if (cnt[b]) lowb = ((unsigned long long)(NT * per - (threadIdx.x * per + q)) << 32) | (unsigned)b;
      }
      hit = block_min_u64(lowb, S);
      if (hit == ~0ull) {  // nothing kept at all
        Found f = {0, 0, 0, 0};
        return f;
      }
    }
    const int b = (int)(uint32_t)hit;
    // mass strictly above bin b at this level
    unsigned long long part = 0;
    for (int q = 0; q < per; ++q)
      if (b_hi - q > b) part += mass[b_hi - q];
    const unsigned long long ab = block_sum_u64(part, S);
    above += ab;
    prefix = (prefix << bitsv[lv]) | (uint32_t)b;
    last_cnt = (int)cnt[b];
    __syncthreads();
  }
  Found f;
  f.w = prefix;
  f.above = above;
  f.n_w = last_cnt;
  const unsigned long long ew = X.wfx(prefix);
  long long j;
  if (ew == 0) {
    j = last_cnt;
  } else if (target <= above) {
    j = strict ? 1 : 1;
    if (strict && target >= above) j = (long long)((target - above) / ew) + 1;
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
__device__ int exact_jth(ExactRow<TIn>& X, const Cut& cut, uint32_t w, int j) {
  Smem& S = X.S;
  constexpr int PER = 8;
  for (int base = 0; base < X.V; base += NT * PER) {
    const int i0 = base + threadIdx.x * PER;
    int cntm = 0;
    for (int i = i0; i < min(i0 + PER, X.V); ++i) {
      const uint32_t key = X.key_at(i);
      if (key == w && cut.keep(key, i)) ++cntm;
    }
    int tot;
    const int ex = block_excl_scan_i(cntm, &tot, S);
    if (j <= tot) {
      if (ex < j && j <= ex + cntm) {
        int r = j - ex;
        for (int i = i0; i < min(i0 + PER, X.V); ++i) {
          const uint32_t key = X.key_at(i);
          if (key == w && cut.keep(key, i) && --r == 0) { S.sc[7] = i; break; }
        }
      }
      __syncthreads();
      return S.sc[7];
    }
    j -= tot;
    __syncthreads();
  }
  return -1;
}

template <typename TIn>
__device__ void exact_row(const KParams& P, const RowCfg& c, int row, Smem& S) {
  const int tid = threadIdx.x;
  ExactRow<TIn> X{P, c, S, (const TIn*)P.logits + (int64_t)row * P.ld, 0, 0, (int)P.V,
                  0.f, 0u};
  // penalised-position bitmap of the whole row
  uint32_t* bm = (uint32_t*)S.sbuf;
  const int words = (X.V + 31) / 32;
  for (int w = tid; w < words; w += NT) bm[w] = 0u;
  __syncthreads();
  if (c.pen) {
    const int64_t a = P.hrow[row], b = P.hrow[row + 1];
    const int64_t sa = lower_bound_ids(P.hids, a, b, P.voff);
    const int64_t sb = lower_bound_ids(P.hids, sa, b, P.voff + X.V);
    X.hist_a = sa;
    X.hist_b = sb;
    for (int64_t q = sa + tid; q < sb; q += NT) {
      if (__ldg(P.hcnt + q) > 0) {
        const int i = (int)(__ldg(P.hids + q) - P.voff);
        atomicOr(&bm[i >> 5], 1u << (i & 31));
      }
    }
  }
  __syncthreads();
  // maximum (and, for greedy rows, the first index of it)
  unsigned long long best = ~0ull;
  for (int i = tid; i < X.V; i += NT) {
    const unsigned long long cc = comp(X.key_at(i), (int)(P.voff + i));
    best = cc < best ? cc : best;
  }
  best = block_min_u64(best, S);
  const uint32_t mkey = comp_key(best);
  X.mv = from_okey(mkey);
  if (c.greedy) {
    if (tid == 0) {
      P.out_ids[row] = comp_id(best);
      RowState st = {};
      st.kind = 2;
      st.token = comp_id(best);
      P.rows[row] = st;
    }
    return;
  }
  if (!(X.mv > -INFINITY) || !(X.mv <= FLT_MAX)) {
    if (tid == 0) {
      P.out_ids[row] = -1;
      status_or(P, VINFER_ST_NONFINITE);
      RowState st = {};
      st.kind = 3;
      st.token = -1;
      P.rows[row] = st;
    }
    return;
  }
  // top-k threshold: radix select over the keys of the whole row (8-bit digits)
  uint32_t tk = 0;
  if (c.topk) {
    uint32_t prefix = 0;
    int need = c.k;
#pragma unroll 1
    for (int pass = 0; pass < 4; ++pass) {
      const int shift = 24 - 8 * pass;
      const uint32_t hmask = pass == 0 ? 0u : (0xFFFFFFFFu << (shift + 8));
      S.hist[tid] = 0;
      __syncthreads();
      for (int i = tid; i < X.V; i += NT) {
        const uint32_t k = X.key_at(i);
        if ((k & hmask) == prefix) atomicAdd(&S.hist[(k >> shift) & 255u], 1u);
      }
      __syncthreads();
      const int d = 255 - tid;
      const int cnt = (int)S.hist[d];
      int tot;
      const int above = block_excl_scan_i(cnt, &tot, S);
      if (above < need && above + cnt >= need) {
        S.sc[14] = d;
        S.sc[15] = need - above;
      }
      __syncthreads();
      prefix |= (uint32_t)S.sc[14] << shift;
      need = S.sc[15];
      __syncthreads();
    }
    tk = prefix;
  }
  Cut base = {tk, 1, 0u, 0, 0u};
  // total mass of the kept-by-top-k set, fixed point
  unsigned long long part = 0;
  for (int i = tid; i < X.V; i += NT) {
    const uint32_t key = X.key_at(i);
    if (base.keep(key, i)) part += X.wfx(key);
  }
  const unsigned long long S_fx = block_sum_u64(part, S);
  Cut fin = base;
  unsigned long long s_kept = S_fx;
  bool cut_set = false;
  if (c.p < 1.f) {
    const unsigned long long tgt = (unsigned long long)((double)c.p * (double)S_fx);
    const Found f = exact_search(X, base, tgt, false);
    if (f.n_w > 0) {
      const int id = exact_jth(X, base, f.w, f.j);
      fin.kind = 0;
      fin.ck = f.w;
      fin.cid = id;
      s_kept = f.above + (unsigned long long)f.j * X.wfx(f.w);
      cut_set = true;
    }
  }
  if (c.minp > 0.f) {
    // smallest key passing min-p: keys are monotone in v, test by value
    const bool binds = !cut_set || ((from_okey(fin.ck) - X.mv) * LOG2E < c.lm);
    if (binds) {
      Cut mc = base;
      unsigned long long pm = 0;
      uint32_t kmin = 0xFFFFFFFFu;
      for (int i = tid; i < X.V; i += NT) {
        const uint32_t key = X.key_at(i);
        if (!base.keep(key, i)) continue;
        if ((from_okey(key) - X.mv) * LOG2E < c.lm) continue;
        pm += X.wfx(key);
        kmin = min(kmin, key);
      }
      const unsigned long long pms = block_sum_u64(pm, S);
      const uint32_t km = (uint32_t)(~block_max_u32(~kmin, S));
      mc.mk = km;
      fin = mc;
      s_kept = pms;
      cut_set = true;
    }
  }
  const unsigned long long tgt = (unsigned long long)((double)c.u * (double)s_kept);
  const Found fd = exact_search(X, fin, tgt, true);
  int tok = -1;
  if (fd.n_w > 0) tok = exact_jth(X, fin, fd.w, fd.j);
  if (tid == 0) {
    if (tok < 0) status_or(P, VINFER_ST_INTERNAL);
    P.out_ids[row] = tok < 0 ? -1 : (int)(P.voff + tok);
    RowState st = {};
    st.m_v = X.mv;
    st.s_kept = (float)((double)s_kept / FX_ONE);
    st.token = P.out_ids[row];
    if (fin.kind == 0) {
      st.kind = 0;
      st.cut_key = fin.ck;
      st.cut_id = (int)(P.voff + fin.cid);
    } else if (fin.mk != 0u) {
      st.kind = 0;
      st.cut_key = fin.mk;
      st.cut_id = 0x7FFFFFFF;
    } else if (c.topk) {
      st.kind = 0;
      st.cut_key = tk;
      st.cut_id = 0x7FFFFFFF;
    } else {
      st.kind = 1;
    }
    P.rows[row] = st;
  }
}

// ---------------------------------------------------------------------------------------------
// kernels
// ---------------------------------------------------------------------------------------------
template <typename TIn>
__global__ void __launch_bounds__(NT, 3) k_sample(const KParams P) {
  extern __shared__ __align__(128) unsigned char smraw[];
  Smem& S = *reinterpret_cast<Smem*>(smraw);
  const int seg = blockIdx.x, row = blockIdx.y, tid = threadIdx.x;
  const RowCfg c = load_row(P, row);
  unsigned char* rec = P.recs + ((size_t)row * P.nseg + seg) * REC_STRIDE;
  const bool local = P.mode == 1;
  if (c.bad || c.exact) {
    if (tid == 0) {
      RecHdr* h = (RecHdr*)rec;
      h->n = 0;
      h->flags = c.bad ? REC_BAD : REC_EXACT;
      h->t_key = 0;
      h->m_y = -INFINITY;
      h->s = 0.f;
    }
  } else {
    segment_pass<TIn>(P, c, row, seg, S, rec);
  }
  // completion count: the last CTA of the row merges
  __threadfence();
  __syncthreads();
  if (tid == 0) {
    const int old = atomicAdd(&P.counters[row], 1);
    const int last = (old == P.nseg - 1);
    if (last) {
      __threadfence();
      P.counters[row] = 0;  // ready for the next call
    }
    S.sc[8] = last;
  }
  __syncthreads();
  if (!S.sc[8]) return;
  __threadfence();

  const MergeIn m = gather_records(P.recs + (size_t)row * P.nseg * REC_STRIDE, REC_STRIDE,
                                   P.nseg, c, S);
  if (local) {
    // write this rank's shard record: entries at or above the K-th, all ties, <= shard_cap
    unsigned char* out = P.shard_out + (size_t)row * P.shard_stride;
    RecHdr* oh = (RecHdr*)out;
    unsigned long long* oe = (unsigned long long*)(out + sizeof(RecHdr));
    const unsigned long long* e = (const unsigned long long*)S.sbuf;
    if ((m.flags & (REC_OVERFLOW | REC_BAD | REC_EXACT)) || m.n > MERGE_CAP) {
      if (tid == 0) {
        oh->n = 0;
        oh->flags = (m.flags & REC_BAD) ? REC_BAD : REC_OVERFLOW;
        oh->t_key = 0;
        oh->m_y = m.m_y;
        oh->s = m.s;
      }
      return;
    }
    int nr = m.n;
    uint32_t tkey = 0;
    if (m.n >= c.K) {
      tkey = comp_key(e[c.K - 1]);
      nr = count_ge(e, m.n, tkey);
    }
    const bool over = nr > P.shard_cap;
    for (int j = tid; j < min(nr, P.shard_cap); j += NT) oe[j] = e[j];
    if (tid == 0) {
      oh->m_y = m.m_y;
      oh->s = m.s;
      oh->n = over ? 0 : nr;
      oh->t_key = (m.flags & REC_UNRETAINED) || nr < m.n ? max(tkey, m.d_key) : 0u;
      oh->flags = over ? REC_OVERFLOW
                       : (((m.flags & REC_UNRETAINED) || nr < m.n) ? REC_UNRETAINED : 0u);
    }
    return;
  }
  if (m.flags & REC_BAD) {
    if (tid == 0) {
      P.out_ids[row] = -1;
      status_or(P, VINFER_ST_BAD_PARAM);
      RowState st = {};
      st.kind = 3;
      st.token = -1;
      P.rows[row] = st;
    }
    return;
  }
  bool done = false;
  if (!(m.flags & (REC_OVERFLOW | REC_EXACT)) && m.n <= MERGE_CAP) {
    done = finalize_sorted(P, c, row, m, S);
  }
  __syncthreads();
  if (!done) exact_row<TIn>(P, c, row, S);
}

// merge of gathered shard records: one CTA per row
__global__ void __launch_bounds__(NT) k_merge(const KParams P, const unsigned char* recs,
                                              int world, int* unresolved) {
  extern __shared__ __align__(128) unsigned char smraw[];
  Smem& S = *reinterpret_cast<Smem*>(smraw);
  const int row = blockIdx.x;
  const RowCfg c = load_row(P, row);
  const MergeIn m =
      gather_records(recs + (size_t)row * P.shard_stride, (size_t)P.B * P.shard_stride, world,
                     c, S);
  bool done = false;
  if (m.flags & REC_BAD) {
    if (threadIdx.x == 0) {
      P.out_ids[row] = -1;
      status_or(P, VINFER_ST_BAD_PARAM);
      RowState st = {};
      st.kind = 3;
      st.token = -1;
      P.rows[row] = st;
    }
    done = true;
  } else if (!(m.flags & (REC_OVERFLOW | REC_EXACT)) && m.n <= MERGE_CAP) {
    done = finalize_sorted(P, c, row, m, S);
  }
  if (threadIdx.x == 0) {
    if (unresolved) unresolved[row] = done ? 0 : 1;
    if (!done) {
      P.out_ids[row] = -1;
      RowState st = {};
      st.kind = 3;
      st.token = -1;
      P.rows[row] = st;
    }
  }
}

// final probabilities [B, V] from the row states (parity checks only)
template <typename TIn>
__global__ void __launch_bounds__(NT) k_probs(const KParams P) {
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
  for (int64_t i = (int64_t)blockIdx.x * NT + threadIdx.x; i < P.V; i += (int64_t)gridDim.x * NT) {
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
      bool keep = st.kind == 1 || key > st.cut_key || (key == st.cut_key && gid <= st.cut_id);
      if (keep) q = ex2((v - st.m_v) * LOG2E) * inv;
    }
    out[i] = q;
  }
}

// ---------------------------------------------------------------------------------------------
// host side
// ---------------------------------------------------------------------------------------------
struct Shape {
  int nseg, seg_len;
};

Shape choose_shape(int64_t B, int64_t V, int dtype) {
  const int es = dtype == VINFER_DTYPE_BF16 ? 2 : 4;
  const int A = 16 / es;
  const int64_t min_seg = (V * es + SEG_BYTES - 1) / SEG_BYTES;
  const int64_t target_ctas = 2048;
  int64_t want = (target_ctas + B - 1) / B;
  want = std::min<int64_t>(want, (V + 2047) / 2048);
  int64_t nseg = std::max<int64_t>(min_seg, std::max<int64_t>(want, 1));
  nseg = std::min<int64_t>(nseg, MAX_NSEG);
  int64_t len = (V + nseg - 1) / nseg;
  len = (len + A - 1) / A * A;
  nseg = (V + len - 1) / len;
  Shape s;
  s.nseg = (int)nseg;
  s.seg_len = (int)len;
  return s;
}

constexpr size_t ALIGN = 256;
size_t align_up(size_t x) { return (x + ALIGN - 1) / ALIGN * ALIGN; }

struct WsLayout {
  size_t counters, rows, recs, total;
};
WsLayout ws_layout(int64_t B, int64_t V, int dtype) {
  const Shape s = choose_shape(B, V, dtype);
  WsLayout L;
  L.counters = 0;
  L.rows = align_up((size_t)B * sizeof(int));
  L.recs = L.rows + align_up((size_t)B * sizeof(RowState));
  L.total = L.recs + (size_t)B * s.nseg * REC_STRIDE;
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

// opt in to the dynamic shared memory of a kernel, once per device and kernel
int set_smem(const void* kern, int slot) {
  static bool done[64][4] = {};
  int dev = 0;
  if (cudaGetDevice(&dev) != cudaSuccess || dev < 0 || dev >= 64) return VINFER_E_CUDA;
  if (done[dev][slot]) return VINFER_OK;
  if (cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize,
                           (int)sizeof(Smem)) != cudaSuccess)
    return VINFER_E_CUDA;
  done[dev][slot] = true;
  return VINFER_OK;
}

int launch_sample(const KParams& P, int dtype, cudaStream_t st) {
  const dim3 grid(P.nseg, P.B);
  if (dtype == VINFER_DTYPE_BF16) {
    if (set_smem((const void*)k_sample<__nv_bfloat16>, 0) != VINFER_OK) return VINFER_E_CUDA;
    k_sample<__nv_bfloat16><<<grid, NT, sizeof(Smem), st>>>(P);
  } else {
    if (set_smem((const void*)k_sample<float>, 1) != VINFER_OK) return VINFER_E_CUDA;
    k_sample<float><<<grid, NT, sizeof(Smem), st>>>(P);
  }
  return cudaGetLastError() == cudaSuccess ? VINFER_OK : VINFER_E_CUDA;
}

int launch_probs(const KParams& P, int dtype, cudaStream_t st) {
  if (!P.out_probs) return VINFER_OK;
  const int bx = (int)std::min<int64_t>(64, (P.V + NT * 8 - 1) / (NT * 8));
  const dim3 grid(std::max(bx, 1), P.B);
  if (dtype == VINFER_DTYPE_BF16) k_probs<__nv_bfloat16><<<grid, NT, 0, st>>>(P);
  else k_probs<float><<<grid, NT, 0, st>>>(P);
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
  const Shape s = choose_shape(a->batch, a->vocab, a->dtype);
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
  const Shape s = choose_shape(a->batch, a->vocab, a->dtype);
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
  const Shape s = choose_shape(a->batch, a->vocab, a->dtype);
  KParams P = make_params(a, s, workspace);
  P.mode = 2;
  P.shard_cap = record_cap;
  P.shard_stride = vinfer_sample_record_bytes(record_cap);
  cudaStream_t st = (cudaStream_t)stream;
  if (set_smem((const void*)k_merge, 2) != VINFER_OK) return VINFER_E_CUDA;
  k_merge<<<(unsigned)a->batch, NT, sizeof(Smem), st>>>(P, (const unsigned char*)records,
                                                        world_size, unresolved);
  if (cudaGetLastError() != cudaSuccess) return VINFER_E_CUDA;
  return launch_probs(P, a->dtype, st);
}

}  // extern "C"

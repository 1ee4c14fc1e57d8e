// sampler.cu — fused token sampler for B200 (sm_100a).
//
// The path restated here is vinfer's reference sampler (src/vinfer/runtime/sampler.py:50-77):
// temperature, top-k (ties at the k-th value kept, :53-55), softmax (:56), top-p on the mass
// strictly before each token (:57-64), renormalisation, and one draw per row, extended with
// repetition / presence / frequency penalties, min-p and an inverse-CDF draw from a caller
// uniform. Tokens are ordered canonically: descending processed logit, ties by ascending id.
//
// Execution (two launches per batch; sharded mode adds an all-gather and k_merge):
//   * k_stream streams every row once. A row is cut into runs of whole segments (64 KiB: one
//     round of 16-byte loads of the CTA, held in registers); with fewer rows than resident CTAs
//     each run is one CTA's. Per vector only its maximum is compared with the CTA's threshold
//     (a shared word raised as the run goes: the K-th largest of K distinct history-free
//     vector maxima, from the first segment, then from blocks of noted "delegate" vectors).
//     At the end of the run the delegates at or above the final threshold are read again and
//     expanded into exact candidates; top-k rows add their penalised tokens with exact values.
//     The run's record is counted on a per-row counter (release).
//   * k_finish is launched as a programmatic dependent of k_stream: one CTA per row starts as
//     SMs free up, waits (bounded) for its row's runs, selects the K largest candidates, checks
//     that the K-th reaches every run's threshold, applies top-p / min-p by prefix sums and
//     draws. Rows the candidates cannot decide take an exact search over the row (key-interval
//     refinement with count and fixed-point mass histograms, 2^-44 units, ties in id order).
//
// All reductions run in a fixed order, so results are deterministic run to run.

#include <cuda_runtime.h>
#include <cuda_bf16.h>
#include <stdint.h>
#include <float.h>
#include <math.h>

#include <algorithm>
#include <cstddef>
#include <mutex>

#include <nvtx3/nvToolsExt.h>

#include "vinfer_sampler.h"

namespace {

// ---------------------------------------------------------------------------------------------
// configuration
// ---------------------------------------------------------------------------------------------
constexpr int NCW = 8;                  // warps per CTA
constexpr int NT = NCW * 32;            // threads per CTA
constexpr int U = 16;                   // 16-byte vectors a thread loads per segment
constexpr int SEG_BYTES = NT * U * 16;  // 64 KiB: one round of loads of the CTA
constexpr int CAND_BUF = 2048;          // candidates held for the run being processed
constexpr int SCRATCH = 4096;           // 8-byte words of the scratch region (32 KiB)
constexpr int CAND_CAP = 1024;          // entries of one record
constexpr int KMAX = 192;               // largest top-k served by the candidate path
constexpr int KC = 32;                  // candidates kept per run when top-k is off (< TB)
constexpr int MAX_NSEG = 64;
constexpr int CTA_CAP = 1024;          // resident CTAs assumed when sizing workspaces
constexpr int MERGE_CAP = 2048;         // merged entries (input in cand, sorted in scratch)
constexpr int DV_CAP = 1024;            // delegates whose 16 bytes are kept in shared memory
constexpr float LOG2E = 1.4426950408889634f;
constexpr double FX_ONE = 17592186044416.0;      // 2^44: fixed-point unit of probability mass
constexpr unsigned FULLMASK = 0xffffffffu;

static_assert(NT == 256, "block helpers assume 256 threads");
static_assert(KMAX <= NCW * 32, "warp extraction covers at most 8 x 32 values");
static_assert(KC <= 64, "block tightening ranks 64 delegates");
static_assert(MERGE_CAP <= CAND_BUF && MERGE_CAP <= SCRATCH, "merge input and output fit");
static_assert(SCRATCH * 64 >= VINFER_MAX_VOCAB, "a row's penalised-id bitmap fits scratch");
static_assert((int64_t)VINFER_MAX_VOCAB * 4 <= (int64_t)MAX_NSEG * SEG_BYTES,
              "the largest float32 row fits MAX_NSEG segments");
static_assert((CAND_BUF * 2 + SCRATCH * 2) * 32 >= VINFER_MAX_VOCAB,
              "the exact search's row bitmap fits the candidate and scratch regions");

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
  int B, nseg, seg_len, mode;  // mode 0: finalize, 1: local (write shard records), 2: merge,
                               // 3: top log-probabilities of rows a mode-0 call just sampled
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
  int topn;          // mode 3: entries of each row's top list
  int* top_ids;      // mode 3: [B, topn] token ids (-1: none)
  float* top_lp;     // mode 3: [B, topn] log-probabilities
  int* slot_ids;     // decode: the slotted histories (the same arrays as hids / hcnt), updated
  int* slot_cnt;     //   in place by k_finish with each row's sampled id; null otherwise
  int* hlen;         // decode: tokens held by each slot
  int hcap;          // decode: entries of a slot
};

struct RowCfg {
  float T, c2, p, minp, lm, rep, pres, freq, u;
  int k, K;
  bool greedy, topk, need_sum, pen, bad, exact;
};

struct __align__(16) Smem {
  unsigned long long cand[CAND_BUF];   // run candidates (composite keys), sorted in place;
                                       // merge input; exact search: row bitmap words
  unsigned long long scratch[SCRATCH]; // the run's history entries while streaming; merge
                                       // output; exact search: more row bitmap words
  float ext[NT];                       // lane maxima extracted per warp
  unsigned long long bin_mass[256];    // exact search: radix bins
  uint32_t bin_cnt[256];
  RecHdr mh[MAX_NSEG];
  int moff[MAX_NSEG + 1];
  unsigned long long red64[NCW + 1];
  float redf[NCW + 1];
  int redi[NCW + 1];
  int sc[16];
  float sf[8];
  int64_t hpos;                        // first history entry of the run
  int wcnt[NCW];                       // candidates per warp slice at the end of a run
  uint32_t ylo_key;                    // the run's threshold: ordered key of a raw logit
  unsigned long long dkth;             // the run's K-th largest unflagged delegate
  int rhi[MAX_NSEG];                   // k_finish: end (global id) of each run of the row
  uint4 dv[DV_CAP];                    // the first delegates' 16 bytes (or edge element)
  float prm[8];                        // the run's row parameters (load_param order)
  RowCfg cfg;                          // ... and the configuration made from them
};

// k_stream's shared memory: the common part, then the run's staged history (ids ascending, and
// their counts) and the run's candidates, which a CTA that streams a whole row finishes from
constexpr int HCAP = 2048;
struct __align__(16) SSmem {
  Smem s;
  int hid[HCAP];
  int hcnt[HCAP];
  unsigned long long rc[CAND_CAP];
};

// A row's arrival counter (workspace): runs of a row split over several CTAs add 1 each as their
// records complete; the CTA completing the row (or the only one) then stores one of these marks.
constexpr int CNT_READY = 0x20000000;  // the records are complete: k_finish finishes the row
constexpr int CNT_DONE = 0x40000000;   // the streaming kernel finished the row
static_assert(MAX_NSEG < CNT_READY, "run counts stay below the marks");

// scalar slots in Smem::sc / Smem::sf
enum { SC_NC = 0, SC_NRET, SC_TKEY, SC_LAST, SC_B, SC_J, SC_X0, SC_X1, SC_NQ, SC_RFL, SC_NH,
       SC_FB, SC_LOCK, SC_NBEST };
enum { SF_TH = 0, SF_SK = 2, SF_M };

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

__device__ __forceinline__ void status_or(const KParams& P, uint32_t bits) {
  if (P.status) atomicOr(reinterpret_cast<unsigned int*>(P.status), bits);
}
// CTA barrier (named barrier 1 over all threads)
__device__ __forceinline__ void cbar() { asm volatile("bar.sync 1, %0;" ::"n"(NT) : "memory"); }
__device__ __forceinline__ int ld_acquire(const int* p) {
  int v;
  asm volatile("ld.acquire.gpu.global.s32 %0, [%1];" : "=r"(v) : "l"(p) : "memory");
  return v;
}
__device__ __forceinline__ int atom_add_acq_rel(int* p, int v) {
  int old;
  asm volatile("atom.acq_rel.gpu.global.add.s32 %0, [%1], %2;" : "=r"(old) : "l"(p), "r"(v)
               : "memory");
  return old;
}
__device__ __forceinline__ void st_release(int* p, int v) {
  asm volatile("st.release.gpu.global.s32 [%0], %1;" ::"l"(p), "r"(v) : "memory");
}
// 4-byte asynchronous copy global -> shared memory (no registers held while in flight)
__device__ __forceinline__ void cp_async4(void* sdst, const void* gsrc) {
  asm volatile("cp.async.ca.shared.global [%0], [%1], 4;" ::"r"(
                   (uint32_t)__cvta_generic_to_shared(sdst)),
               "l"(gsrc)
               : "memory");
}
__device__ __forceinline__ void cp_async_wait_all() {
  asm volatile("cp.async.wait_all;" ::: "memory");
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
  __device__ static float vmin(const uint4& q) {
    return fminf(fminf(__uint_as_float(q.x), __uint_as_float(q.y)),
                 fminf(__uint_as_float(q.z), __uint_as_float(q.w)));
  }
  // is any element a NaN with the sign bit clear? (bit patterns 0x7F800001 .. 0x7FFFFFFF)
  __device__ static bool pos_nan(const uint4& q) {
    return (q.x - 0x7F800001u) < 0x007FFFFFu || (q.y - 0x7F800001u) < 0x007FFFFFu ||
           (q.z - 0x7F800001u) < 0x007FFFFFu || (q.w - 0x7F800001u) < 0x007FFFFFu;
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
  __device__ static float vmin(const uint4& q) {
    const __nv_bfloat162 a = *reinterpret_cast<const __nv_bfloat162*>(&q.x);
    const __nv_bfloat162 b = *reinterpret_cast<const __nv_bfloat162*>(&q.y);
    const __nv_bfloat162 c = *reinterpret_cast<const __nv_bfloat162*>(&q.z);
    const __nv_bfloat162 d = *reinterpret_cast<const __nv_bfloat162*>(&q.w);
    const __nv_bfloat162 m = __hmin2(__hmin2(a, b), __hmin2(c, d));
    return fminf(__low2float(m), __high2float(m));
  }
  // is any element a NaN with the sign bit clear? (halves 0x7F81 .. 0x7FFF)
  __device__ static bool pos_nan(const uint4& q) {
    const uint32_t lo = 0x7F807F80u, hi = 0x80008000u;
    const uint32_t r = (__vcmpgtu2(q.x, lo) & __vcmpltu2(q.x, hi)) |
                       (__vcmpgtu2(q.y, lo) & __vcmpltu2(q.y, hi)) |
                       (__vcmpgtu2(q.z, lo) & __vcmpltu2(q.z, hi)) |
                       (__vcmpgtu2(q.w, lo) & __vcmpltu2(q.w, hi));
    return r != 0u;
  }
  __device__ static float at(const uint4& q, int e) {
    const uint32_t w = (e >> 1) == 0 ? q.x : (e >> 1) == 1 ? q.y : (e >> 1) == 2 ? q.z : q.w;
    return __uint_as_float((e & 1) ? (w & 0xFFFF0000u) : (w << 16));
  }
};

// ---------------------------------------------------------------------------------------------
// per-row configuration
// ---------------------------------------------------------------------------------------------

__device__ RowCfg make_cfg(const KParams& P, float T, int k, float p, float minp, float rep,
                           float pres, float freq, float u) {
  if (P.mode == 3) {  // the n largest processed values: top-k n, no cut, no draw
    k = P.topn;
    p = 1.f;
    minp = 0.f;
    u = 0.f;
  }
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
__device__ __noinline__ bool finalize_sorted(const KParams& P, const RowCfg& c, int row, const MergeIn& m,
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
  float Ssum = c.topk ? total : m.s;
  // the sums are relative to the largest raw logit; rescale when that one was penalised
  if (!c.topk && vf(m.m_y, c) != mv) Ssum *= ex2(m.m_y * c.c2 - mv * LOG2E);
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

// finalize_sorted for short lists (m.n <= 64), by one warp with no CTA barrier: each lane holds
// entries 2 * lane and 2 * lane + 1; prefix sums are a warp scan. Same decisions as
// finalize_sorted; called by the 32 lanes of one warp, every lane returns the same value.
__device__ bool finalize_warp(const KParams& P, const RowCfg& c, int row, const MergeIn& m,
                              const unsigned long long* e) {
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
  int nk, avail;
  if (c.topk) {
    nk = (n >= c.K) ? count_ge(e, n, comp_key(e[c.K - 1])) : n;
    avail = nk;
  } else {
    avail = more ? count_ge(e, n, m.d_key) : n;
    nk = 0x7FFFFFFF;
  }
  const int j0 = 2 * lane, j1 = j0 + 1;
  const float v0 = j0 < n ? from_okey(comp_key(e[j0])) : -INFINITY;
  const float v1 = j1 < n ? from_okey(comp_key(e[j1])) : -INFINITY;
  const float w0 = j0 < avail ? ex2((v0 - mv) * LOG2E) : 0.f;
  const float w1 = j1 < avail ? ex2((v1 - mv) * LOG2E) : 0.f;
  float inc = w0 + w1;
#pragma unroll
  for (int o = 1; o < 32; o <<= 1) {
    const float t = __shfl_up_sync(FULLMASK, inc, o);
    if (lane >= o) inc += t;
  }
  const float C0 = inc - w1, C1 = inc;  // inclusive prefixes at j0 and j1
  const float total = __shfl_sync(FULLMASK, inc, 31);
  float Ssum = c.topk ? total : m.s;
  if (!c.topk && vf(m.m_y, c) != mv) Ssum *= ex2(m.m_y * c.c2 - mv * LOG2E);
  const bool listed_all = c.topk || !more;
  // first index whose pair flag is set (lane order, then j0 before j1); -1 when none
  auto first = [&](bool f0, bool f1) -> int {
    const unsigned b = __ballot_sync(FULLMASK, f0 || f1);
    if (!b) return -1;
    const int l = __ffs(b) - 1;
    return 2 * l + (__shfl_sync(FULLMASK, f0, l) ? 0 : 1);
  };
  int L = 0x7FFFFFFF;
  if (c.topk) L = nk;
  else if (!more) L = n;
  bool cut_beyond = false;
  if (c.p < 1.f) {  // top-p: keep tokens whose mass strictly before them is < top_p
    const float t = c.p * Ssum;
    const int h = first(j0 < avail && C0 >= t, j1 < avail && C1 >= t);
    if (h >= 0) L = min(L, h + 1);
    else if (!listed_all) cut_beyond = true;
  }
  if (c.minp > 0.f) {  // min-p: keep tokens with exp(v - max) >= min_p
    const int h = first(j0 < avail && (v0 - mv) * LOG2E < c.lm,
                        j1 < avail && (v1 - mv) * LOG2E < c.lm);
    if (h >= 0) L = min(L, max(h, 1));
    else if (!listed_all) cut_beyond = true;
  }
  const bool L_known = L <= avail;
  if (!L_known && cut_beyond) return false;
  float s_kept = Ssum;
  if (L_known) {
    const int last = L - 1;
    const float cl = (last & 1) ? C1 : C0;
    s_kept = __shfl_sync(FULLMASK, cl, last >> 1);
  }
  const int lim = L_known ? L : avail;
  const float t = c.u * s_kept;
  int j = first(j0 < lim && C0 > t, j1 < lim && C1 > t);
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

// ---------------------------------------------------------------------------------------------
// exact multi-pass search over one row (global memory), for rows the records cannot resolve
// ---------------------------------------------------------------------------------------------
// penalised-position bitmap of a whole row: the candidate region's words, then scratch's
struct RowBits {
  uint32_t* w0;
  uint32_t* w1;
  static constexpr int N0 = CAND_BUF * 2;
  __device__ uint32_t& word(int w) const { return w < N0 ? w0[w] : w1[w - N0]; }
  __device__ bool bit(int i) const { return (word(i >> 5) >> (i & 31)) & 1u; }
};
// history entries staged for the exact search (second half of scratch): local index, key
constexpr int XSTAGE = SCRATCH / 2;
// a bin of the exact search holding at most this many elements is collected and sorted
// (Smem::mh viewed as 8-byte entries)
constexpr int XCOLLECT = (int)(sizeof(RecHdr) * MAX_NSEG / 8);

template <typename TIn>
struct ExactRow {
  const KParams& P;
  const RowCfg& c;
  RowBits bm;  // penalised positions of the row
  const TIn* rowp;
  int64_t hist_a, hist_b;
  int V;
  float mv;
  const int* sid;        // staged history entries, ascending local index ...
  const uint32_t* skey;  // ... and the processed key of each penalised one
  int ns;                // staged entries; -1 when they did not fit (searched in global memory)

  // processed key of penalised position i
  __device__ uint32_t pen_key(int i) const {
    if (ns >= 0) {
      int lo = 0, hi = ns;
      while (lo < hi) {
        const int mid = (lo + hi) >> 1;
        if (sid[mid] < i) lo = mid + 1; else hi = mid;
      }
      return skey[lo];
    }
    const int64_t p = lower_bound_ids(P.hids, hist_a, hist_b, P.voff + i);
    return okey(vf(penalize(Elem<TIn>::ld(rowp, i), __ldg(P.hcnt + p), c), c));
  }
  __device__ uint32_t key_at(int i) const {
    if (c.pen && bm.bit(i)) return pen_key(i);
    return okey(vf(Elem<TIn>::ld(rowp, i), c));
  }
  __device__ unsigned long long wfx(uint32_t key) const {
    const float e = ex2((from_okey(key) - mv) * LOG2E);
    const unsigned long long w = (unsigned long long)__float2ull_rn(e * (float)FX_ONE);
    return w <= (1ull << 44) ? w : (1ull << 44);  // e <= 1 (a NaN converts to anything)
  }
};

// are any of the positions [i0, i0 + n) set in the bitmap? (n <= 32, i0 + n <= V)
__device__ __forceinline__ bool bits_any(const RowBits& bm, int V, int i0, int n) {
  const int w = i0 >> 5;
  unsigned long long win = bm.word(w);
  if (((i0 & 31) + n) > 32 && (w + 1) * 32 < V) win |= (unsigned long long)bm.word(w + 1) << 32;
  return ((win >> (i0 & 31)) & ((1ull << n) - 1ull)) != 0ull;
}
// the first element of a vector, and the vector shifted down by one element
template <typename TIn>
__device__ __forceinline__ void shift_elem(uint4& q) {
  constexpr int SB = 128 / Elem<TIn>::A;  // bits per element
  if constexpr (SB == 32) {
    q.x = q.y;
    q.y = q.z;
    q.z = q.w;
  } else {
    q.x = __funnelshift_r(q.x, q.y, SB);
    q.y = __funnelshift_r(q.y, q.z, SB);
    q.z = __funnelshift_r(q.z, q.w, SB);
    q.w >>= SB;
  }
}

// Walks a row of V logits: vec(q, i0, valid) once per 16-byte vector slot of every thread
// (whole warps call it together; i0 = position of the vector's first element), then
// edge(valid, y, i) once per lane of warp 0 for the ragged head and tail (fewer than 32
// positions, any alignment). Four vectors per thread are in flight; they are visited one per
// iteration, rotated through registers, which keeps the loop body at one vector's worth of code.
template <typename TIn, typename FV, typename FE>
__device__ __forceinline__ void row_walk(const TIn* rowp, int V, FV&& vec, FE&& edge) {
  using E = Elem<TIn>;
  constexpr int A = E::A;
  constexpr int UE = 4;
  const int tid = threadIdx.x;
  const uintptr_t addr = (uintptr_t)rowp;
  int head = (int)(((16u - (uint32_t)(addr & 15u)) & 15u) / sizeof(TIn));
  if (head > V) head = V;
  const int nv = (V - head) / A;
  const int tail0 = head + nv * A;
  const uint4* vb = reinterpret_cast<const uint4*>(rowp + head);
  for (int j0 = 0; j0 < nv; j0 += NT * UE) {
    uint4 q0, q1, q2, q3;
    {
      const int j = j0 + tid;
      q0 = j < nv ? __ldg(vb + j) : make_uint4(0u, 0u, 0u, 0u);
      q1 = j + NT < nv ? __ldg(vb + j + NT) : make_uint4(0u, 0u, 0u, 0u);
      q2 = j + 2 * NT < nv ? __ldg(vb + j + 2 * NT) : make_uint4(0u, 0u, 0u, 0u);
      q3 = j + 3 * NT < nv ? __ldg(vb + j + 3 * NT) : make_uint4(0u, 0u, 0u, 0u);
    }
#pragma unroll 1
    for (int u = 0; u < UE; ++u) {
      const int j = j0 + u * NT + tid;
      vec(q0, head + j * A, j < nv);
      q0 = q1;
      q1 = q2;
      q2 = q3;
    }
  }
  if (tid < 32) {
    const int nht = head + (V - tail0);
    const bool valid = tid < nht;
    const int i = tid < head ? tid : tail0 + (tid - head);
    edge(valid, valid ? E::ld(rowp, i) : 0.f, i);
  }
}

// Visits every position of the row once: f(ok, key, i), called by whole warps (f may use warp
// collectives). A position is visited with its key and ok = true when it is penalised or when
// its raw logit y satisfies !(y < ylo) && !(y >= ynext); otherwise with ok = false and no key
// (the caller chose the interval so that such positions cannot hold a key it looks for, which
// skips the division).
template <typename TIn, typename F>
__device__ __forceinline__ void row_pass(const ExactRow<TIn>& X, float ylo, float ynext, F&& f) {
  using E = Elem<TIn>;
  constexpr int A = E::A;
  // everything the loop reads, in registers (X may live in memory)
  const int V = X.V;
  const bool pen = X.c.pen;
  const RowBits bm = X.bm;
  RowCfg cl{};  // what vf() needs
  cl.T = X.c.T;
  cl.greedy = X.c.greedy;
  auto visit = [&](bool valid, bool maybe_pen, float y, int i) {
    bool ok = false;
    uint32_t key = 0;
    if (valid) {
      if (maybe_pen && bm.bit(i)) {
        key = X.pen_key(i);
        ok = true;
      } else if (!(y < ylo) && !(y >= ynext)) {
        key = okey(vf(y, cl));
        ok = true;
      }
    }
    f(ok, key, i);
  };
  row_walk<TIn>(
      X.rowp, V,
      [&](uint4 q, int i0, bool vv) {
        const bool mp = vv && pen && bits_any(bm, V, i0, A);
#pragma unroll 1
        for (int e = 0; e < A; ++e) {
          visit(vv, mp, E::at(q, 0), i0 + e);
          shift_elem<TIn>(q);
        }
      },
      [&](bool valid, float y, int i) { visit(valid, pen, y, i); });
}

// Calls f(key, i), lane by lane (f uses no warp collectives), for the positions that are
// penalised or whose raw logit y satisfies !(y < ylo) && !(y >= ynext). Vectors whose
// minimum and maximum rule out both are skipped whole, so a narrow interval costs little more
// than reading the row.
template <typename TIn, typename F>
__device__ __forceinline__ void row_pass_sparse(const ExactRow<TIn>& X, float ylo, float ynext, F&& f) {
  using E = Elem<TIn>;
  constexpr int A = E::A;
  const int V = X.V;
  const bool pen = X.c.pen;
  const RowBits bm = X.bm;
  RowCfg cl{};
  cl.T = X.c.T;
  cl.greedy = X.c.greedy;
  const bool open_hi = !(ynext == ynext);  // NaN: no upper bound
  // penalised positions come from the staged list after the walk (no lookup per element)
  const bool staged = pen && X.ns >= 0;
  auto elem = [&](bool maybe_pen, float y, int i) {
    if (maybe_pen && bm.bit(i)) {
      if (!staged) f(X.pen_key(i), i);
    } else if (!(y < ylo) && !(y >= ynext)) {
      f(okey(vf(y, cl)), i);
    }
  };
  row_walk<TIn>(
      X.rowp, V,
      [&](uint4 q, int i0, bool vv) {
        if (!vv) return;
        const bool mp = pen && bits_any(bm, V, i0, A);
        if ((!mp || staged) && (E::vmax(q) < ylo || !(open_hi || E::vmin(q) < ynext))) return;
#pragma unroll 1
        for (int e = 0; e < A; ++e) {
          elem(mp, E::at(q, 0), i0 + e);
          shift_elem<TIn>(q);
        }
      },
      [&](bool valid, float y, int i) {
        if (valid) elem(pen, y, i);
      });
  if (staged)
    for (int s = threadIdx.x; s < X.ns; s += NT) {
      const int i = X.sid[s];
      if (bm.bit(i)) f(X.skey[s], i);
    }
}

// Radix bins of the exact search: element counts and fixed-point masses. 64-bit shared-memory
// adds contend badly on the few hot bins of a float radix, so a mass (at most 2^44, 45 bits) is
// added as four 12-bit parts to four 32-bit bins; a bin receives at most VINFER_MAX_VOCAB
// = 2^18 elements, so no part sum overflows. All adds are lane by lane.
static_assert(VINFER_MAX_VOCAB <= (1 << 18), "12-bit mass parts of a bin cannot overflow");
static_assert(sizeof(RecHdr) * MAX_NSEG >= 2 * 256 * sizeof(uint32_t), "parts 2 and 3 fit Smem::mh");
struct BinHist {
  uint32_t* cnt;  // [256]
  uint32_t* p01;  // mass parts 0 and 1: [2][256] (Smem::bin_mass)
  uint32_t* p23;  // mass parts 2 and 3: [2][256] (Smem::mh)
  __device__ explicit BinHist(Smem& S)
      : cnt(S.bin_cnt), p01(reinterpret_cast<uint32_t*>(S.bin_mass)),
        p23(reinterpret_cast<uint32_t*>(S.mh)) {}
  __device__ void clear() const {  // by every thread of the CTA (NT == 256)
    const int t = threadIdx.x;
    cnt[t] = 0u;
    p01[t] = 0u;
    p01[256 + t] = 0u;
    p23[t] = 0u;
    p23[256 + t] = 0u;
  }
  __device__ void add(uint32_t b, bool with_mass, unsigned long long w) const {
    atomicAdd(&cnt[b], 1u);
    if (!with_mass) return;
    const uint32_t q0 = (uint32_t)w & 0xFFFu, q1 = (uint32_t)(w >> 12) & 0xFFFu;
    const uint32_t q2 = (uint32_t)(w >> 24) & 0xFFFu, q3 = (uint32_t)(w >> 36) & 0xFFFu;
    if (q0) atomicAdd(&p01[b], q0);
    if (q1) atomicAdd(&p01[256 + b], q1);
    if (q2) atomicAdd(&p23[b], q2);
    if (q3) atomicAdd(&p23[256 + b], q3);
  }
  __device__ unsigned long long mass(int b) const {
    return (unsigned long long)p01[b] + ((unsigned long long)p01[256 + b] << 12) +
           ((unsigned long long)p23[b] << 24) + ((unsigned long long)p23[256 + b] << 36);
  }
};

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

// One thread's bin of the first radix level (thread t holds bin 255 - t): returned by a search
// (out) and, adjusted to a narrower cut, given to the next one (in) in place of its first pass.
struct Level0 {
  bool in;
  int cut_bin;           // (in) the bin the narrower cut passes through: its count is unknown
  unsigned long long m;  // weight of the bin
  uint32_t c;            // elements in it
  unsigned long long mo;
  uint32_t co;
};

struct Found {
  uint32_t w;                // key of the tie group reached
  unsigned long long above;  // weight strictly above w (kept elements)
  int j;                     // 1-based rank inside the tie group, ascending id
  int n_w;
  int id;                    // local index of the element, -1 when left to exact_jth
};

__device__ float ylo_for(float vt, const RowCfg& c);
// Raw-logit interval [ylo, ynext) of the positions whose processed key lies in [klo, khi]
// (vf is monotone): ylo is the smallest y with vf(y) >= from_okey(klo), ynext the smallest y
// with vf(y) above from_okey(khi). Keys outside the finite range leave the bound open (NaN
// upper bound: nothing compares >= it). Warp-wide (ylo_for).
__device__ void raw_range(const RowCfg& c, uint32_t klo, uint32_t khi, float* ylo, float* ynext) {
  const uint32_t kninf = okey(-INFINITY), kpinf = okey(INFINITY);
  if (klo <= kninf) *ylo = -INFINITY;
  else if (klo > kpinf) *ylo = INFINITY;
  else *ylo = ylo_for(from_okey(klo), c);
  if (khi >= kpinf) *ynext = __int_as_float(0x7fc00000);
  else if (khi < kninf) *ynext = -INFINITY;
  else *ynext = ylo_for(from_okey(khi + 1u == 0x7FFFFFFFu ? 0x80000000u : khi + 1u), c);
}

// Mass-scale bins, the first step of a mass search: bin of a key by d = (mv - v) log2(e) in
// quarter units; bin 255 holds d >= 63.75 (and NaN), keys above the finite range count as bin 0.
// Non-increasing in the key, so ascending bins are keys in descending order, and each bin holds
// a narrow slice of the probability mass whatever the spread of the row.
__device__ __forceinline__ int dbin(uint32_t key, float mv) {
  if (key > 0xFF800000u) return 0;  // above +inf: a NaN with the sign bit clear
  const float d = (mv - from_okey(key)) * LOG2E;
  if (!(d < 63.75f)) return 255;
  return d > 0.f ? (int)(d * 4.f) : 0;
}
// smallest key whose mass-scale bin is <= b (the bins are monotone in the key)
__device__ uint32_t dbin_lowkey(int b, float mv) {
  uint32_t lo = 0u, hi = 0xFFFFFFFFu;
  while (lo < hi) {
    const uint32_t mid = lo + (hi - lo) / 2u;
    if (dbin(mid, mv) <= b) hi = mid; else lo = mid + 1u;
  }
  return lo;
}

// Canonical position where the cumulative kept weight first reaches (>=) or passes (>)
// `target`: weight = fixed-point mass (mass_w) or 1. The search narrows a key interval known
// to hold that position: for a mass search the first step bins by mass scale (dbin), then
// 8-bit radix digits over the highest bits in which the interval's ends differ; once the
// interval holds at most XCOLLECT kept elements they are collected and sorted, which resolves
// the element itself. With frac >= 0 the target is frac x the total weight (the first step's
// histogram gives the total, also returned). l0 carries the first step's bins out, or in
// (adjusted to a narrower cut) in place of its pass.
template <typename TIn>
__device__ Found exact_search(const ExactRow<TIn>& X, const Cut& cut_in,
                              unsigned long long target, double frac, bool strict, bool mass_w,
                              Smem& S, unsigned long long* total_out, Level0* l0) {
  const Cut cut = cut_in;  // in registers: the passes test it per element
  const float mv = X.mv;
  const BinHist hist(S);
  unsigned long long* buf = reinterpret_cast<unsigned long long*>(S.mh);
  const int tid = threadIdx.x;
  auto weight = [&](uint32_t key) -> unsigned long long {
    if (!mass_w) return 1ull;
    const float e = ex2((from_okey(key) - mv) * LOG2E);
    const unsigned long long w = (unsigned long long)__float2ull_rn(e * (float)FX_ONE);
    return w <= (1ull << 44) ? w : (1ull << 44);  // e <= 1 (a NaN converts to anything)
  };
  // no kept key lies below this (the prefilter's floor)
  uint32_t klo = max(max(cut.tk, cut.mk), cut.kind == 0 ? cut.ck : 0u);
  uint32_t khi = 0xFFFFFFFFu;
  unsigned long long above = 0;  // kept weight above khi
  int n_in = 0x7FFFFFFF;         // kept elements in [klo, khi] (not known before the first step)
#pragma unroll 1
  for (int step = 0; step < 8; ++step) {
    if (n_in <= XCOLLECT) {
      // ---- collect the interval, sort it (canonical order) and walk its cumulative weight
      float ylo, ynext;
      raw_range(X.c, klo, khi, &ylo, &ynext);
      if (tid == 0) S.sc[SC_NQ] = 0;
      cbar();
      row_pass_sparse(X, ylo, ynext, [&](uint32_t key, int i) {
        if (key >= klo && key <= khi && cut.keep(key, i)) {
          const int pos = atomicAdd(&S.sc[SC_NQ], 1);
          if (pos < XCOLLECT) buf[pos] = comp(key, i);
        }
      });
      cbar();
      const int n = min(S.sc[SC_NQ], XCOLLECT);
      if (n == 0) {
        Found f = {0u, 0ull, 0, 0, -1};
        return f;
      }
      unsigned long long x = tid < n ? buf[tid] : ~0ull;
      int rank = 0;
      if (tid < n)
        for (int t = 0; t < n; ++t) rank += buf[t] < x;
      cbar();
      if (tid < n) buf[rank] = x;
      cbar();
      x = tid < n ? buf[tid] : ~0ull;
      const uint32_t kx = comp_key(x);
      const unsigned long long wx = tid < n ? weight(kx) : 0ull;
      unsigned long long tot2;
      const unsigned long long exw = cta_excl_scan_u64(wx, &tot2, S);
      const unsigned long long bef = above + exw, aft = bef + wx;
      const bool cr = tid < n && (strict ? (aft > target) : (aft >= target));
      unsigned long long first = cta_min_u64(cr ? (unsigned long long)tid : ~0ull, S);
      if (first == ~0ull) first = (unsigned long long)(n - 1);  // rounding: the last element
      const uint32_t w = comp_key(buf[(int)first]);
      // the tie group of w: its first index, size and the weight above it
      const unsigned long long g0 =
          cta_min_u64(tid < n && kx == w ? (unsigned long long)tid : ~0ull, S);
      int ng;
      cta_excl_scan_i(tid < n && kx == w ? 1 : 0, &ng, S);
      if (tid == (int)g0) S.red64[NCW] = bef;
      cbar();
      Found f;
      f.w = w;
      f.above = S.red64[NCW];
      f.n_w = ng;
      const unsigned long long ew = weight(w);
      long long j;
      if (ew == 0) {
        j = ng;
      } else if (target < f.above) {
        j = 1;
      } else {
        const unsigned long long d = target - f.above;
        j = strict ? (long long)(d / ew) + 1 : (long long)((d + ew - 1) / ew);
      }
      if (j < 1) j = 1;
      if (j > ng) j = ng;
      f.j = (int)j;
      f.id = comp_id(buf[(int)g0 + f.j - 1]);
      cbar();
      return f;
    }
    if (klo == khi) break;  // one key: a tie group too large to collect
    // ---- one step: bins over [klo, khi]; thread t holds the bin at position t in descending
    // key order
    const bool dstep = step == 0;
    int sh = 0;
    uint32_t base = 0u;
    if (!dstep) {
      const int hb = 31 - __clz(klo ^ khi);
      sh = hb >= 7 ? hb - 7 : 0;
      base = klo >> sh;
    }
    unsigned long long mb;
    uint32_t cb;
    const bool given = step == 0 && l0 && l0->in;
    if (given) {
      mb = l0->m;
      cb = l0->c;
    } else {
      float ylo, ynext;
      raw_range(X.c, klo, khi, &ylo, &ynext);
      hist.clear();
      cbar();
      row_pass_sparse(X, ylo, ynext, [&](uint32_t key, int i) {
        if (key < klo || key > khi || !cut.keep(key, i)) return;
        const int bi = dstep ? dbin(key, mv) : 255 - (int)((key >> sh) - base);
        hist.add((uint32_t)bi, mass_w, mass_w ? weight(key) : 0ull);
      });
      cbar();
      cb = hist.cnt[tid];
      mb = mass_w ? hist.mass(tid) : (unsigned long long)cb;
    }
    if (step == 0 && l0) {
      l0->mo = mb;
      l0->co = cb;
    }
    unsigned long long tot;
    const unsigned long long ex = cta_excl_scan_u64(mb, &tot, S);
    if (step == 0) {
      if (total_out) *total_out = tot;
      if (frac >= 0.0) target = (unsigned long long)(frac * (double)tot);
    }
    const unsigned long long before = above + ex, after = before + mb;
    const bool cross_after = strict ? (after > target) : (after >= target);
    const bool cross_before = strict ? (before > target) : (before >= target);
    unsigned long long pick = ~0ull;
    if (cb > 0 && cross_after && !cross_before) pick = (unsigned long long)tid;
    pick = cta_min_u64(pick, S);
    if (pick == ~0ull) {  // target at or beyond the total (rounding): the last non-empty bin
      pick = cta_min_u64(cb > 0 ? (unsigned long long)(NT - 1 - tid) : ~0ull, S);
      if (pick == ~0ull) {
        Found f = {0u, 0ull, 0, 0, -1};
        return f;
      }
      pick = (unsigned long long)(NT - 1 - (int)pick);
    }
    if ((int)pick == tid) {
      S.red64[NCW] = before;
      S.sc[SC_J] = (given && tid == l0->cut_bin) ? 0x7FFFFFFF : (int)cb;
    }
    cbar();
    const int t = (int)pick;
    uint32_t kl, kh;
    if (dstep) {
      kl = dbin_lowkey(t, mv);
      kh = t == 0 ? 0xFFFFFFFFu : dbin_lowkey(t - 1, mv) - 1u;
    } else {
      kl = (base + (uint32_t)(255 - t)) << sh;
      kh = kl | ((1u << sh) - 1u);
    }
    klo = max(klo, kl);
    khi = min(khi, kh);
    above = S.red64[NCW];
    n_in = S.sc[SC_J];
    cbar();
  }
  // a single key holding more than XCOLLECT kept elements: its j-th by index, found later
  Found f;
  f.w = klo;
  f.above = above;
  f.n_w = n_in;
  f.id = -1;
  const unsigned long long ew = weight(klo);
  long long j;
  if (ew == 0) {
    j = n_in;
  } else if (target < above) {
    j = 1;
  } else {
    const unsigned long long d = target - above;
    j = strict ? (long long)(d / ew) + 1 : (long long)((d + ew - 1) / ew);
  }
  if (j < 1) j = 1;
  if (j > n_in) j = n_in;
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
__device__ int found_index(const ExactRow<TIn>& X, const Cut& cut, const Found& f, Smem& S) {
  if (f.n_w <= 0) return -1;
  return f.id >= 0 ? f.id : exact_jth(X, cut, f.w, f.j, S);
}

template <typename TIn>
__device__ __noinline__ void exact_row(const KParams& P, const RowCfg& c, int row, Smem& S,
                                       unsigned char* scratch) {
  const int tid = threadIdx.x;
  const RowBits bm{(uint32_t*)S.cand, (uint32_t*)scratch};
  int* sid = reinterpret_cast<int*>(reinterpret_cast<unsigned long long*>(scratch) + XSTAGE);
  uint32_t* skey = reinterpret_cast<uint32_t*>(sid + XSTAGE);
  ExactRow<TIn> X{P, c, bm, (const TIn*)P.logits + (int64_t)row * P.ld, 0, 0, (int)P.V, 0.f,
                  sid, skey, -1};
  const int words = (X.V + 31) / 32;
  for (int w = tid; w < words; w += NT) bm.word(w) = 0u;
  cbar();
  if (c.pen) {
    const int64_t a = P.hrow[row], b = P.hrow[row + 1];
    X.hist_a = lower_bound_ids(P.hids, a, b, P.voff);
    X.hist_b = lower_bound_ids(P.hids, X.hist_a, b, P.voff + X.V);
    const int64_t nh = X.hist_b - X.hist_a;
    X.ns = nh <= XSTAGE ? (int)nh : -1;
    for (int64_t q = X.hist_a + tid; q < X.hist_b; q += NT) {
      const int i = (int)(__ldg(P.hids + q) - P.voff);
      const int cn = __ldg(P.hcnt + q);
      if (cn > 0) atomicOr(&bm.word(i >> 5), 1u << (i & 31));
      if (X.ns >= 0) {
        sid[q - X.hist_a] = i;
        skey[q - X.hist_a] =
            cn > 0 ? okey(vf(penalize(Elem<TIn>::ld(X.rowp, i), cn, c), c)) : 0u;
      }
    }
  }
  cbar();
  const float NO_BOUND = __int_as_float(0x7fc00000);  // an open upper bound of row_pass
  if (c.greedy) {  // the first index of the maximum (keys are the penalised logits themselves)
    unsigned long long best = ~0ull;
    row_pass(X, -INFINITY, NO_BOUND, [&](bool ok, uint32_t key, int i) {
      if (!ok) return;
      const unsigned long long cc = comp(key, (int)(P.voff + i));
      best = cc < best ? cc : best;
    });
    best = cta_min_u64(best, S);
    if (tid == 0) write_state(P, row, 2, comp_id(best), 0.f, 0.f, 0u, 0);
    return;
  }
  // the largest processed value: vf is monotone, so the largest raw logit of the positions
  // without penalty gives theirs with one division; penalised positions bring their keys. A
  // NaN with the sign bit clear is the largest key of all (the row is then refused below).
  {
    using E = Elem<TIn>;
    uint32_t kb = 0u;
    float ymax = -INFINITY;
    bool pnan = false;
    const bool staged = c.pen && X.ns >= 0;
    auto one = [&](bool maybe_pen, float y, int i) {
      if (maybe_pen && bm.bit(i)) {
        if (!staged) kb = max(kb, X.pen_key(i));
      } else {
        ymax = fmaxf(ymax, y);
        pnan = pnan || (__float_as_uint(y) - 0x7F800001u) < 0x007FFFFFu;
      }
    };
    row_walk<TIn>(
        X.rowp, X.V,
        [&](uint4 q, int i0, bool vv) {
          if (!vv) return;
          if (c.pen && bits_any(bm, X.V, i0, E::A)) {
#pragma unroll 1
            for (int e = 0; e < E::A; ++e) {
              one(true, E::at(q, 0), i0 + e);
              shift_elem<TIn>(q);
            }
          } else {
            ymax = fmaxf(ymax, E::vmax(q));
            pnan = pnan || E::pos_nan(q);
          }
        },
        [&](bool valid, float y, int i) {
          if (valid) one(c.pen, y, i);
        });
    if (staged)
      for (int s = tid; s < X.ns; s += NT)
        if (bm.bit(sid[s])) kb = max(kb, skey[s]);
    kb = pnan ? 0xFFC00000u : max(kb, okey(vf(ymax, c)));
    S.ext[tid] = ymax;  // this thread's largest raw logit without penalty (the top-k floor)
    X.mv = from_okey(cta_max_u32(kb, S));
  }
  if (!(X.mv > -INFINITY) || !(X.mv <= FLT_MAX)) {
    if (tid == 0) {
      write_state(P, row, 3, -1, 0.f, 0.f, 0u, 0);
      status_or(P, VINFER_ST_NONFINITE);
    }
    return;
  }
  // top-k threshold: the key of the k-th element in canonical order (ties of it kept). The
  // k-th largest of the threads' largest raw logits (distinct positions) bounds it from below
  // for k <= 256, so only the positions above that bound are searched.
  uint32_t tk = 0;
  if (c.topk) {
    uint32_t kfl = 0u;
    if (c.k <= NT) {
      const float mine = S.ext[tid];
      int rank = 0;
      for (int t = 0; t < NT; ++t) {
        const float o = S.ext[t];
        rank += (o > mine) || (o == mine && t < tid);
      }
      const unsigned long long cand = rank == c.k - 1 && mine > -INFINITY
                                          ? (unsigned long long)okey(vf(mine, c))
                                          : 0ull;
      kfl = (uint32_t)~cta_min_u64(~cand, S);
    }
    const Cut all = {kfl, 1, 0u, 0, 0u};
    const Found fk =
        exact_search(X, all, (unsigned long long)c.k, -1.0, false, false, S, nullptr, nullptr);
    tk = fk.n_w > 0 ? fk.w : 0u;
  }
  const Cut base = {tk, 1, 0u, 0, 0u};
  Cut fin = base;
  unsigned long long S_fx = 0, s_kept = 0;
  bool cut_set = false;
  Level0 l0 = {false, -1, 0ull, 0u, 0ull, 0u};
  bool have_l0 = false;  // l0.mo/co: this thread's first-level bin of the top-k kept set
  if (c.p < 1.f) {
    // the total kept mass comes with the first level of the search
    const Found f = exact_search(X, base, 0ull, (double)c.p, false, true, S, &S_fx, &l0);
    have_l0 = true;
    s_kept = S_fx;
    if (f.n_w > 0) {
      const int id = found_index(X, base, f, S);
      fin.kind = 0;
      fin.ck = f.w;
      fin.cid = id;
      s_kept = f.above + (unsigned long long)f.j * X.wfx(f.w);
      cut_set = true;
    }
  } else {
    unsigned long long part = 0;
    float ylo_k, yn_k;
    raw_range(c, tk, 0xFFFFFFFFu, &ylo_k, &yn_k);
    row_pass_sparse(X, ylo_k, yn_k, [&](uint32_t key, int i) {
      if (base.keep(key, i)) part += X.wfx(key);
    });
    S_fx = cta_sum_u64(part, S);
    s_kept = S_fx;
  }
  if (c.minp > 0.f) {
    // min-p keeps a prefix by value; it binds when the top-p cut lies below its threshold
    const bool binds = !cut_set || ((from_okey(fin.ck) - X.mv) * LOG2E < c.lm);
    if (binds) {
      unsigned long long pm = 0;
      uint32_t kmin = 0xFFFFFFFFu;
      float ylo_k, yn_k;
      raw_range(c, tk, 0xFFFFFFFFu, &ylo_k, &yn_k);
      row_pass_sparse(X, ylo_k, yn_k, [&](uint32_t key, int i) {
        if (!base.keep(key, i)) return;
        if ((from_okey(key) - X.mv) * LOG2E < c.lm) return;
        pm += X.wfx(key);
        kmin = min(kmin, key);
      });
      const unsigned long long pms = cta_sum_u64(pm, S);
      const uint32_t km = ~cta_max_u32(~kmin, S);
      fin = base;
      fin.mk = km;
      s_kept = pms;
    }
  }
  const unsigned long long tgt = (unsigned long long)((double)c.u * (double)s_kept);
  if (have_l0) {
    // the draw's first step from the top-p search's mass-scale bins (thread t holds bin t):
    // bins above the cut's bin are kept whole, the cut's bin keeps s_kept less the bins above
    // it, lower bins nothing
    const bool cut_k = fin.kind == 0 || fin.mk != 0u;
    const int cbin = cut_k ? dbin(fin.kind == 0 ? fin.ck : fin.mk, X.mv) : -1;
    const unsigned long long m_above = cta_sum_u64(cut_k && tid < cbin ? l0.mo : 0ull, S);
    l0.in = true;
    l0.cut_bin = cbin;
    l0.m = l0.mo;
    l0.c = l0.co;
    if (cut_k && tid == cbin) {
      l0.m = s_kept - m_above;
      l0.c = 1u;
    } else if (cut_k && tid > cbin) {
      l0.m = 0ull;
      l0.c = 0u;
    }
  }
  const Found fd = exact_search(X, fin, tgt, -1.0, true, true, S, nullptr, have_l0 ? &l0 : nullptr);
  const int tok = found_index(X, fin, fd, S);
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
__device__ __noinline__ void finish_row(const KParams& P, Smem& S, unsigned char* scratch, int row,
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
// streaming: each CTA streams its segments with plain 16-byte loads held in registers
// ---------------------------------------------------------------------------------------------
// smallest y with vf(y) >= vt: about y = vt * T; the boundary lies within a few keys of it in
// the normal range, found by one round of 32 probes (a full binary search otherwise). Warp-wide.
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

// Sorts buf[0, n) in place (n <= CAND_BUF) and keeps the K largest with every tie of the K-th
// at the front. Returns the kept count; *tkey receives the K-th key (0 when n < K).
__device__ int select_inplace(unsigned long long* buf, int n, int K, uint32_t* tkey, Smem& S) {
  const int tid = threadIdx.x;
  if (n <= NT) {  // rank by counting: one candidate per thread
    unsigned long long x = 0ull;
    int rank = 0;
    if (tid < n) {
      x = buf[tid];
#pragma unroll 8
      for (int j = 0; j < n; ++j) rank += buf[j] < x;
      if (rank == K - 1) S.sc[SC_TKEY] = (int)comp_key(x);
    }
    if (tid == 0) S.sc[SC_NRET] = 0;
    cbar();
    const uint32_t t = n >= K ? (uint32_t)S.sc[SC_TKEY] : 0u;
    if (tid < n && comp_key(x) >= t) {
      buf[rank] = x;
      atomicMax(&S.sc[SC_NRET], rank + 1);
    }
    cbar();
    *tkey = t;
    const int r = S.sc[SC_NRET];
    cbar();
    return r;
  }
  // larger sets (rare): bitonic sort, padded to a power of two with the largest key
  int np = 1;
  while (np < n) np <<= 1;
  for (int j = n + tid; j < np; j += NT) buf[j] = ~0ull;
  cbar();
  for (int k = 2; k <= np; k <<= 1) {
    for (int j = k >> 1; j > 0; j >>= 1) {
      for (int i = tid; i < np; i += NT) {
        const int ixj = i ^ j;
        if (ixj > i) {
          const unsigned long long a = buf[i], b = buf[ixj];
          if ((a > b) == ((i & k) == 0)) {
            buf[i] = b;
            buf[ixj] = a;
          }
        }
      }
      cbar();
    }
  }
  const uint32_t t = n >= K ? comp_key(buf[K - 1]) : 0u;
  *tkey = t;
  return n >= K ? count_ge(buf, n, t) : n;
}

// The streaming kernel's view of a row's history: a bitmap, in shared memory, of the ids of this
// shard (bit i = global id voff + i) that have a positive count, i.e. the penalised tokens.
struct RunHist {
  const uint32_t* bits;
  int64_t voff;
};
__device__ __forceinline__ RunHist hist_view(const KParams& P, Smem& S) {
  return RunHist{reinterpret_cast<const uint32_t*>(S.scratch), P.voff};
}
// is `id` a penalised token?
__device__ __forceinline__ int hist_count(const RunHist& h, int id) {
  const int i = (int)(id - h.voff);
  return (h.bits[i >> 5] >> (i & 31)) & 1u;
}

// ---- delegates --------------------------------------------------------------------------------
// While streaming, a vector (or an edge element) whose maximum reaches the threshold is only
// noted: its maximum raw logit and the id of its first element. At the end of the run the K-th
// largest delegate bounds the run's K-th largest value closely, and only the vectors at or above
// that bound are read again and expanded. Entry: (~okey(max) << 32) | DL_ONE flag | first
// id, so ascending entries are descending maxima.
constexpr uint32_t DL_ONE = 0x40000000u;  // an edge element, not a 16-byte vector
constexpr uint32_t DL_ID = 0x3FFFFFFFu;
static_assert(2 * (int64_t)VINFER_MAX_VOCAB <= (int64_t)DL_ID, "global ids fit a delegate");

__device__ __forceinline__ unsigned long long dele(float vmax, uint32_t bits) {
  return ((unsigned long long)(~okey(vmax)) << 32) | bits;
}
__device__ __forceinline__ float dele_max(unsigned long long d) {
  return from_okey(~(uint32_t)(d >> 32));
}

// is any of the ids [id0, id0 + n) a penalised token? (n <= 32)
__device__ __forceinline__ bool hist_any(const RunHist& h, int id0, int n) {
  const int i = (int)(id0 - h.voff);
  const int w = i >> 5, b = i & 31;
  const uint64_t two = (uint64_t)h.bits[w] | ((b + n > 32) ? (uint64_t)h.bits[w + 1] << 32 : 0ull);
  const uint64_t mask = ((n >= 64) ? ~0ull : ((1ull << n) - 1ull)) << b;
  return (two & mask) != 0ull;
}

// Note one delegate in the run's list (any lane), with its data (the 16-byte vector, or the edge
// element in .x) for the first DV_CAP, so the run's end expands them without reading them again.
// Returns its slot; slots past the list are counted, not written (the run then takes the exact
// search).
__device__ __forceinline__ int dele_push(Smem& S, unsigned long long d, const uint4& q) {
  const int pos = atomicAdd(&S.sc[SC_NC], 1);
  if (pos < CAND_BUF) S.cand[pos] = d;
  if (pos < DV_CAP) S.dv[pos] = q;
  return pos;
}

constexpr int TB = 64;  // the list is tightened once per block of TB delegates
static_assert(KC < TB, "rows without top-k tighten on the KC-th delegate of a block");

// A list entry once its writer has stored it (the list starts filled with ~0); gives up after a
// bounded number of polls and reports the entry as absent, which only weakens the bound.
__device__ __forceinline__ unsigned long long list_entry(const Smem& S, int i) {
  const volatile unsigned long long* v = S.cand;
  unsigned long long x = v[i];
  for (int it = 0; x == ~0ull && it < 4096; ++it) x = v[i];
  return x;
}

// The warp that completed block [b0, b0 + TB) of the list raises the CTA's threshold to the
// K-th largest unflagged delegate of that block (K distinct vectors without history ids reach
// it). Warp-wide; K <= TB.
__device__ __forceinline__ void block_tighten(const KParams& P, int b0, int K, float T, bool greedy,
                                           bool pen, int vec_len, Smem& S) {
  const int lane = threadIdx.x & 31;
  unsigned long long v0 = list_entry(S, b0 + lane), v1 = list_entry(S, b0 + 32 + lane);
  if (pen) {  // delegates holding a history id are not counted
    const RunHist h = hist_view(P, S);
    if (v0 != ~0ull && hist_any(h, (int)((uint32_t)v0 & DL_ID), ((uint32_t)v0 & DL_ONE) ? 1 : vec_len))
      v0 = ~0ull;
    if (v1 != ~0ull && hist_any(h, (int)((uint32_t)v1 & DL_ID), ((uint32_t)v1 & DL_ONE) ? 1 : vec_len))
      v1 = ~0ull;
  }
  // the K-th largest ordered key of the block's counted delegates (absent ones have key 0): a
  // radix select, most significant bit first, one pair of ballots per bit
  const int nv = __popc(__ballot_sync(FULLMASK, v0 != ~0ull)) +
                 __popc(__ballot_sync(FULLMASK, v1 != ~0ull));
  if (nv < K) return;
  const uint32_t ka = ~(uint32_t)(v0 >> 32), kb = ~(uint32_t)(v1 >> 32);
  uint32_t prefix = 0u;
  int need = K;
#pragma unroll 4
  for (int bit = 31; bit >= 0; --bit) {
    const uint32_t hi = ~((1u << bit) - 1u), cand = prefix | (1u << bit);
    const int n = __popc(__ballot_sync(FULLMASK, (ka & hi) == cand)) +
                  __popc(__ballot_sync(FULLMASK, (kb & hi) == cand));
    if (n >= need) prefix = cand;
    else need -= n;
  }
  RowCfg c{};
  c.T = T;
  c.greedy = greedy;
  const float y = ylo_for(vf(from_okey(prefix), c), c);
  if (lane == 0) atomicMax(&S.ylo_key, okey(y));
}

// one segment's loads for this thread: U coalesced vectors and at most one edge scalar
template <typename TIn>
struct SegLoad {
  uint4 q[U];
  float sy;       // edge scalar (ragged head or tail), -inf when none
  int64_t sid;    // its global id, -1 when none
  int64_t gid0;   // global id of the first element of the segment's first vector
  const uint4* vb;  // the segment's first vector in global memory
  int nvec;       // vectors in the segment
};

// One 16-byte streaming load: read once, so it allocates no L1 line and is the first to go from
// L2 (the kernels' code, parameters, histories and records stay cached while logits stream by).
__device__ __forceinline__ uint4 ld_stream(const uint4* p, uint64_t pol) {
  uint4 r;
  asm("ld.global.nc.L1::no_allocate.L2::cache_hint.v4.u32 {%0, %1, %2, %3}, [%4], %5;"
      : "=r"(r.x), "=r"(r.y), "=r"(r.z), "=r"(r.w)
      : "l"(p), "l"(pol));
  return r;
}
__device__ __forceinline__ uint64_t evict_first_policy() {
  uint64_t pol;
  asm("createpolicy.fractional.L2::evict_first.b64 %0, 1.0;" : "=l"(pol));
  return pol;
}

template <typename TIn>
__device__ __forceinline__ void load_segment(const KParams& P, const TIn* rowp, int seg,
                                             SegLoad<TIn>& L) {
  using E = Elem<TIn>;
  constexpr int A = E::A;
  constexpr int ES = 16 / A;
  const int tid = threadIdx.x;
  const int64_t lo = (int64_t)seg * P.seg_len;
  const int n = (int)(min(P.V, lo + (int64_t)P.seg_len) - lo);
  const uintptr_t gaddr = (uintptr_t)(rowp + lo);
  int head = (int)(((16u - (uint32_t)(gaddr & 15u)) & 15u) / ES);
  if (head > n) head = n;
  L.nvec = (int)(((int64_t)(n - head) * ES) / 16);
  const int tail0 = head + L.nvec * A;
  const uint4* vb = reinterpret_cast<const uint4*>(rowp + lo + head);
  L.vb = vb;
  L.gid0 = P.voff + lo + head;
  const uint64_t pol = evict_first_policy();
#pragma unroll
  for (int u = 0; u < U; ++u) {
    const int j = tid + NT * u;
    L.q[u] = j < L.nvec ? ld_stream(vb + j, pol) : make_uint4(0u, 0u, 0u, 0u);
  }
  L.sid = -1;
  L.sy = -INFINITY;
  if (tid < head) {
    L.sid = lo + tid;
  } else if (tid >= 32 && tid - 32 < n - tail0) {
    L.sid = lo + tail0 + (tid - 32);
  }
  if (L.sid >= 0) {
    L.sy = E::ld(rowp, L.sid);
    L.sid += P.voff;
  }
}

// ---- warp-level sorting helpers (ascending 64-bit keys across the 32 lanes) -----------------
__device__ __forceinline__ unsigned long long warp_sort32(unsigned long long x) {
  const int lane = threadIdx.x & 31;
#pragma unroll
  for (int k = 2; k <= 32; k <<= 1) {
#pragma unroll
    for (int j = k >> 1; j > 0; j >>= 1) {
      const unsigned long long o = __shfl_xor_sync(FULLMASK, x, j);
      const bool lower = (lane & j) == 0, up = (lane & k) == 0;
      x = (lower == up) ? (o < x ? o : x) : (o > x ? o : x);
    }
  }
  return x;
}
// the 32 smallest of two ascending lane-sorted lists, ascending
__device__ __forceinline__ unsigned long long warp_merge32(unsigned long long a,
                                                           unsigned long long b) {
  const int lane = threadIdx.x & 31;
  const unsigned long long r = __shfl_sync(FULLMASK, b, 31 - lane);
  unsigned long long x = r < a ? r : a;  // a bitonic sequence holding the 32 smallest
#pragma unroll
  for (int j = 16; j > 0; j >>= 1) {
    const unsigned long long o = __shfl_xor_sync(FULLMASK, x, j);
    x = ((lane & j) == 0) ? (o < x ? o : x) : (o > x ? o : x);
  }
  return x;
}

// A first threshold for the run from this warp's first segment, with no CTA barrier: each lane
// takes the j-th largest of its vector maxima (j = ceil(K / 32)), and if q = ceil(K / j) lanes
// reach t then K distinct vectors do. t is the q-th largest lane value (a warp bitonic sort).
// With j = 1 a lane whose best vector holds a history id contributes nothing, so penalised
// tokens cannot lift the bound; with j > 1 they are not checked, and should penalties push
// the bound above the row's K-th largest processed value, the finishing kernel detects it and
// takes the exact search, so it only ever costs time. Published with atomicMax.
// ---- rows with 32 < K <= KMAX: their own instantiation of the streaming loop (the code below
// stays out of the K <= 32 loop's registers)

// The K-th largest of the 256 ordered keys Smem::ext holds (as floats), by one warp: a radix
// select bit by bit, each lane counting its eight keys and the warp summing the counts.
__device__ __forceinline__ uint32_t warp_kth_of_256(int K, Smem& S) {
  const int lane = threadIdx.x & 31;
  const volatile float* ext = S.ext;
  uint32_t key[NCW];
#pragma unroll
  for (int o = 0; o < NCW; ++o) key[o] = okey(ext[o * 32 + lane]);
  uint32_t prefix = 0u;
  int need = K;
#pragma unroll 1
  for (int bit = 31; bit >= 0; --bit) {
    const uint32_t mask = ~((1u << bit) - 1u), cand = prefix | (1u << bit);
    int c = 0;
#pragma unroll
    for (int o = 0; o < NCW; ++o) c += (key[o] & mask) == cand;
    c = (int)__reduce_add_sync(FULLMASK, (unsigned)c);
    if (c >= need) prefix = cand;
    else need -= c;
  }
  return prefix;
}

// Ascending sort of 64 keys held two per lane (a: element lane, b: element lane + 32), bitonic.
__device__ __forceinline__ void warp_sort64(unsigned long long& a, unsigned long long& b) {
  const int lane = threadIdx.x & 31;
#pragma unroll
  for (int k = 2; k <= 64; k <<= 1) {
#pragma unroll
    for (int j = k >> 1; j > 0; j >>= 1) {
      if (j == 32) {  // pairs (lane, lane + 32), ascending (k = 64)
        const unsigned long long lo = a < b ? a : b, hi = a < b ? b : a;
        a = lo;
        b = hi;
      } else {
        const unsigned long long pa = __shfl_xor_sync(FULLMASK, a, j);
        const unsigned long long pb = __shfl_xor_sync(FULLMASK, b, j);
        const bool low = (lane & j) == 0;  // the lower index of its pair
        const bool upa = (lane & k) == 0, upb = ((lane + 32) & k) == 0;
        a = (low == upa) ? (a < pa ? a : pa) : (a < pa ? pa : a);
        b = (low == upb) ? (b < pb ? b : pb) : (b < pb ? pb : b);
      }
    }
  }
}

// One block says little about a K-th largest with K > 32, so these rows keep the K best
// unflagged delegates seen so far (sorted, canonical order; Smem::bin_mass is free while
// streaming) and the warp that completes a block merges the block into them and raises the
// threshold to their K-th. One warp merges at a time; a block that finds the list busy is left
// out, which only leaves the bound looser (any K distinct elements bound the K-th largest).
static_assert(KMAX + TB <= 256, "the best list and a sorted block fit Smem::bin_mass");
__device__ __noinline__ void best_merge(const KParams& P, int b0, int K, float T, bool greedy,
                                        bool pen, int vec_len, Smem& S) {
  const int lane = threadIdx.x & 31;
  int got = 0;
  if (lane == 0) got = atomicCAS(&S.sc[SC_LOCK], 0, 1) == 0;
  if (!__shfl_sync(FULLMASK, got, 0)) return;
  __threadfence_block();
  unsigned long long* best = S.bin_mass;        // [KMAX]
  unsigned long long* blk = S.bin_mass + KMAX;  // [TB]
  auto ent = [&](int i) {
    unsigned long long v = list_entry(S, i);
    if (pen && v != ~0ull) {
      const RunHist h = hist_view(P, S);
      if (hist_any(h, (int)((uint32_t)v & DL_ID), ((uint32_t)v & DL_ONE) ? 1 : vec_len)) v = ~0ull;
    }
    return v;
  };
  unsigned long long a = ent(b0 + lane), b = ent(b0 + 32 + lane);
  warp_sort64(a, b);
  blk[lane] = a;
  blk[32 + lane] = b;
  const int na = *reinterpret_cast<volatile int*>(&S.sc[SC_NBEST]);
  const int nb = __popc(__ballot_sync(FULLMASK, a != ~0ull)) + __popc(__ballot_sync(FULLMASK, b != ~0ull));
  __syncwarp();
  // outputs o = lane + 32 t of the merge of best[0, na) and blk[0, nb): merge path
  const int nout = min(K, na + nb);
  unsigned long long out[(KMAX + 31) / 32];
#pragma unroll
  for (int t = 0; t < (KMAX + 31) / 32; ++t) {
    const int o = lane + 32 * t;
    out[t] = ~0ull;
    if (o < nout) {
      int lo = max(0, o - nb), hi = min(o, na);
      while (lo < hi) {  // elements of best among the first o outputs
        const int mid = (lo + hi) >> 1;
        if (best[mid] < blk[o - 1 - mid]) lo = mid + 1; else hi = mid;
      }
      const int j = o - lo;
      out[t] = (j >= nb || (lo < na && best[lo] < blk[j])) ? best[lo] : blk[j];
    }
  }
  __syncwarp();
#pragma unroll
  for (int t = 0; t < (KMAX + 31) / 32; ++t) {
    const int o = lane + 32 * t;
    if (o < nout) best[o] = out[t];
  }
  unsigned long long kth = ~0ull;
#pragma unroll
  for (int t = 0; t < (KMAX + 31) / 32; ++t)
    if (nout == K && t == ((K - 1) >> 5)) kth = __shfl_sync(FULLMASK, out[t], (K - 1) & 31);
  __syncwarp();
  if (lane == 0) *reinterpret_cast<volatile int*>(&S.sc[SC_NBEST]) = nout;
  if (kth != ~0ull) {
    RowCfg c{};
    c.T = T;
    c.greedy = greedy;
    const float y = ylo_for(vf(dele_max(kth), c), c);
    if (lane == 0) atomicMax(&S.ylo_key, okey(y));
  }
  __threadfence_block();
  __syncwarp();
  if (lane == 0) atomicExch(&S.sc[SC_LOCK], 0);
}

// First bounds of a large-K row, from the first segment. At once, per warp: the q-th largest
// of its lanes' j-th largest vector maxima (j = ceil(K / 32), q = ceil(K / j): q lanes with j
// vectors each reach it). Then, by the last warp to publish: the K-th largest of the 256 lanes'
// largest vector maxima (a lane's is left out when that vector holds a history id), which is
// much tighter. Both are bounds on the row's K-th largest.
template <typename TIn>
__device__ __forceinline__ void wide_first_bound(const KParams& P, const SegLoad<TIn>& L,
                                                 const float* vm, int K, float T, bool greedy,
                                                 bool pen, Smem& S) {
  constexpr int A = Elem<TIn>::A;
  const int tid = threadIdx.x, lane = tid & 31;
  const int j = (K + 31) / 32;
  float v[U];
#pragma unroll
  for (int u = 0; u < U; ++u) v[u] = vm[u];
  float l1 = -INFINITY, lv = -INFINITY;
  int u1 = -1;
  for (int r = 0; r < j; ++r) {  // the lane's r-th largest vector maximum
    float m = -INFINITY;
    int mu = -1;
#pragma unroll
    for (int u = 0; u < U; ++u)
      if (v[u] > m) {
        m = v[u];
        mu = u;
      }
    lv = m;
    if (r == 0) {
      l1 = m;
      u1 = mu;
    }
#pragma unroll
    for (int u = 0; u < U; ++u)
      if (u == mu) v[u] = -INFINITY;
  }
  float x = lv;
#pragma unroll
  for (int k = 2; k <= 32; k <<= 1) {  // descending bitonic sort of the 32 lane values
#pragma unroll
    for (int jj = k >> 1; jj > 0; jj >>= 1) {
      const float o = __shfl_xor_sync(FULLMASK, x, jj);
      const bool lower = (lane & jj) == 0, up = (lane & k) == 0;
      x = (lower == up) ? fmaxf(x, o) : fminf(x, o);
    }
  }
  const float tw = __shfl_sync(FULLMASK, x, (K + j - 1) / j - 1);
  if (tw > -INFINITY) {
    RowCfg c{};
    c.T = T;
    c.greedy = greedy;
    const float y = ylo_for(vf(tw, c), c);
    if (lane == 0) atomicMax(&S.ylo_key, okey(y));
  }
  if (pen && u1 >= 0 &&
      hist_any(hist_view(P, S), (int)(L.gid0 + (int64_t)(tid + NT * u1) * A), A))
    l1 = -INFINITY;
  S.ext[tid] = l1;
  __threadfence_block();
  __syncwarp();
  int last = 0;
  if (lane == 0) last = atomicAdd(&S.sc[SC_FB], 1) == NCW - 1;
  if (__shfl_sync(FULLMASK, last, 0)) {
    __threadfence_block();
    const float tc = from_okey(warp_kth_of_256(K, S));
    if (tc > -INFINITY) {
      RowCfg c{};
      c.T = T;
      c.greedy = greedy;
      const float y = ylo_for(vf(tc, c), c);
      if (lane == 0) atomicMax(&S.ylo_key, okey(y));
    }
  }
  __syncwarp();
}

template <typename TIn>
__device__ __forceinline__ void warp_first_bound(const KParams& P, const SegLoad<TIn>& L,
                                                 const float* vm, int K, float T, bool greedy,
                                                 bool pen, Smem& S) {
  constexpr int A = Elem<TIn>::A;
  const int tid = threadIdx.x, lane = tid & 31;
  const int j = (K + 31) / 32;
  float v[U];
#pragma unroll
  for (int u = 0; u < U; ++u) v[u] = vm[u];
  float lv = -INFINITY;
  int um = -1;
  for (int r = 0; r < j; ++r) {  // j-th largest of the lane's vector maxima
    float m = -INFINITY;
    int mu = -1;
#pragma unroll
    for (int u = 0; u < U; ++u)
      if (v[u] > m) {
        m = v[u];
        mu = u;
      }
    lv = m;
    um = mu;
#pragma unroll
    for (int u = 0; u < U; ++u)
      if (u == mu) v[u] = -INFINITY;
  }
  if (j == 1 && pen && um >= 0 &&
      hist_any(hist_view(P, S), (int)(L.gid0 + (int64_t)(tid + NT * um) * A), A))
    lv = -INFINITY;
  float x = lv;
#pragma unroll
  for (int k = 2; k <= 32; k <<= 1) {  // descending bitonic sort of the 32 lane values
#pragma unroll
    for (int jj = k >> 1; jj > 0; jj >>= 1) {
      const float o = __shfl_xor_sync(FULLMASK, x, jj);
      const bool lower = (lane & jj) == 0, up = (lane & k) == 0;
      x = (lower == up) ? fmaxf(x, o) : fminf(x, o);
    }
  }
  const int q = (K + j - 1) / j;
  const float t = __shfl_sync(FULLMASK, x, q - 1);
  RowCfg c{};
  c.T = T;
  c.greedy = greedy;
  if (t > -INFINITY) {
    const float y = ylo_for(vf(t, c), c);
    if (lane == 0) atomicMax(&S.ylo_key, okey(y));
  }
  // publish the sorted lane values; the last warp to do so derives the CTA-wide bound (the
  // q-th largest of all 256 lane values) without making any warp wait
  const int w = tid >> 5;
  S.ext[w * 32 + lane] = x;
  __threadfence_block();
  __syncwarp();
  int last = 0;
  if (lane == 0) last = atomicAdd(&S.sc[SC_FB], 1) == NCW - 1;
  if (__shfl_sync(FULLMASK, last, 0)) {
    __threadfence_block();
    const volatile float* ext = S.ext;
    auto key = [&](int o) {  // ascending keys = descending values, unique by position
      return ((unsigned long long)(~okey(ext[o * 32 + lane])) << 32) | (uint32_t)(o * 32 + lane);
    };
    unsigned long long m = key(0);
    for (int o = 1; o < NCW; ++o) m = warp_merge32(m, key(o));
    const unsigned long long kq = __shfl_sync(FULLMASK, m, q - 1);
    const float tc = from_okey(~(uint32_t)(kq >> 32));
    if (tc > -INFINITY) {
      const float y = ylo_for(vf(tc, c), c);
      if (lane == 0) atomicMax(&S.ylo_key, okey(y));
    }
  }
  __syncwarp();
}

// Mode 3: a row's top list from its sorted entries e[0, m) (the m largest processed values, in
// canonical order), each token with its log-probability under the distribution the preceding
// sampling call left in the row state: ln p = (v - m_v) - ln(s_kept), -inf outside the kept set
// (a greedy row's distribution is one-hot on its token). Slots past m get id -1 and -inf; a row
// without a sampling result gets -1 and NaN. The 32 lanes of one warp.
__device__ void write_top(const KParams& P, int row, const unsigned long long* e, int m) {
  const int lane = threadIdx.x & 31;
  const RowState st = P.rows[row];
  for (int j = lane; j < P.topn; j += 32) {
    int id = -1;
    float lp = -INFINITY;
    if (st.kind == 3) {
      lp = __int_as_float(0x7fc00000);
    } else if (j < m) {
      id = comp_id(e[j]);
      const uint32_t key = comp_key(e[j]);
      bool kept;
      if (st.kind == 2) kept = id == st.token;
      else if (st.kind == 1) kept = true;
      else kept = key > st.cut_key || (key == st.cut_key && id <= st.cut_id);
      if (kept) lp = st.kind == 2 ? 0.f : (from_okey(key) - st.m_v) - logf(st.s_kept);
    }
    P.top_ids[(size_t)row * P.topn + j] = id;
    P.top_lp[(size_t)row * P.topn + j] = lp;
  }
}

// ---------------------------------------------------------------------------------------------
// finishing a row inside the streaming kernel
// ---------------------------------------------------------------------------------------------
// The CTA that completes a row (or streams all of it) finishes the row itself when its
// candidates decide it: every kind of row except rows without top-k, whose softmax sum needs the
// penalised terms k_finish stages. Same decisions as k_finish: the K largest candidates with the
// ties of the K-th, the check that the K-th reaches every run's threshold (maxkey; all_in when
// no run raised one), then the cut and the draw (mode 0) or this rank's shard record (mode 1).
// cand[0, nc) are the row's candidates in shared memory, unsorted (nc <= CAND_BUF); the row's
// parameters are in Smem::prm. Called by the whole CTA; returns false (the same on every
// thread) when k_finish must finish the row.
__device__ __noinline__ bool fast_finish(const KParams& P, Smem& S, int row,
                                         unsigned long long* cand, int nc, uint32_t maxkey,
                                         bool all_in) {
  const int tid = threadIdx.x, lane = tid & 31, w = tid >> 5;
  const RowCfg c = S.cfg;  // made at the run's set-up
  const bool local = P.mode == 1;
  RecHdr* oh = local ? reinterpret_cast<RecHdr*>(P.shard_out + (size_t)row * P.shard_stride)
                     : nullptr;
  unsigned long long* oe = reinterpret_cast<unsigned long long*>(oh + 1);
  const int K = c.greedy ? 1 : c.K;
  if (c.greedy && !c.pen) {
    // one entry per run: the smallest composite key is the first index of the maximum
    if (P.mode == 3) {
      if (w == 0) {
        unsigned long long b = ~0ull;
        if (lane == 0)
          for (int i = 0; i < nc; ++i) b = cand[i] < b ? cand[i] : b;
        b = __shfl_sync(FULLMASK, b, 0);
        __syncwarp();
        if (lane == 0) cand[0] = b;
        __syncwarp();
        write_top(P, row, cand, b != ~0ull ? 1 : 0);
      }
      return true;
    }
    if (tid == 0) {
      unsigned long long b = ~0ull;
      for (int i = 0; i < nc; ++i) b = cand[i] < b ? cand[i] : b;
      const int nret = b != ~0ull;
      if (local) {
        const uint32_t rfl = (nret && P.V > 1) ? REC_UNRETAINED : 0u;
        if (nret) oe[0] = b;
        oh->m_y = -INFINITY;
        oh->s = 0.f;
        oh->n = nret;
        oh->t_key = rfl ? comp_key(b) : 0u;
        oh->flags = rfl;
      } else if (nret) {
        write_state(P, row, 2, comp_id(b), 0.f, 0.f, 0u, 0);
      } else {
        write_state(P, row, 3, -1, 0.f, 0.f, 0u, 0);
        status_or(P, VINFER_ST_NONFINITE);
      }
    }
    return true;
  }
  if (nc <= 64 && !c.greedy) {  // short lists: one warp sorts, selects, cuts and draws
    if (w == 0) {
      // sorted by counting ranks (entries are distinct): independent shared-memory reads
      // instead of a chain of shuffle stages
      unsigned long long a = lane < nc ? cand[lane] : ~0ull;
      unsigned long long b = lane + 32 < nc ? cand[lane + 32] : ~0ull;
      int ra = 0, rb = 0;
#pragma unroll 8
      for (int j = 0; j < nc; ++j) {
        const unsigned long long x = cand[j];
        ra += x < a;
        rb += x < b;
      }
      unsigned long long* srt = S.scratch;  // free once the run's candidates are made
      if (lane < nc) srt[ra] = a;
      if (lane + 32 < nc) srt[rb] = b;
      __syncwarp();
      a = lane < nc ? srt[lane] : ~0ull;
      b = lane + 32 < nc ? srt[lane + 32] : ~0ull;
      cand[lane] = a;
      cand[lane + 32] = b;
      __syncwarp();
      uint32_t tk = 0u;
      if (nc >= K) tk = comp_key(__shfl_sync(FULLMASK, K - 1 < 32 ? a : b, (K - 1) & 31));
      const int nr = nc >= K ? __popc(__ballot_sync(FULLMASK, lane < nc && comp_key(a) >= tk)) +
                                   __popc(__ballot_sync(FULLMASK, lane + 32 < nc && comp_key(b) >= tk))
                             : nc;
      int res = 0;
      if (all_in || (nc >= K && tk >= maxkey)) {  // the top-K cut is known
        const bool more = !(all_in && nr == nc);
        const uint32_t dkey = max(nc >= K ? tk : 0u, maxkey);
        const uint32_t rflags = more ? REC_UNRETAINED : 0u;
        res = 1;
        if (P.mode == 3) {
          write_top(P, row, cand, nr);
        } else if (local) {
          if (nr > P.shard_cap) {
            if (lane == 0) write_flag_hdr(oh, REC_OVERFLOW, -INFINITY, 0.f);
          } else {
            for (int j = lane; j < nr; j += 32) oe[j] = cand[j];
            if (lane == 0) {
              oh->m_y = -INFINITY;
              oh->s = 0.f;
              oh->n = nr;
              oh->t_key = rflags ? dkey : 0u;
              oh->flags = rflags;
            }
          }
        } else if (nr == 0) {
          if (lane == 0) {
            write_state(P, row, 3, -1, 0.f, 0.f, 0u, 0);
            status_or(P, VINFER_ST_NONFINITE);
          }
        } else {
          MergeIn mi;
          mi.m_y = -INFINITY;
          mi.s = 0.f;
          mi.d_key = dkey;
          mi.flags = rflags;
          mi.n = nr;
          res = finalize_warp(P, c, row, mi, cand) ? 1 : 0;
        }
      }
      if (lane == 0) S.sc[SC_X1] = res;
    }
    cbar();
    return S.sc[SC_X1] != 0;
  }
  int nret;
  uint32_t tkey;
  if (nc <= 32) {  // one warp sorts the short list
    if (w == 0) {
      unsigned long long x = lane < nc ? cand[lane] : ~0ull;
      x = warp_sort32(x);
      cand[lane] = x;
      const unsigned long long kx = __shfl_sync(FULLMASK, x, min(K, 32) - 1);
      const uint32_t tk = nc >= K ? comp_key(kx) : 0u;
      const int nr =
          nc >= K ? __popc(__ballot_sync(FULLMASK, lane < nc && comp_key(x) >= tk)) : nc;
      if (lane == 0) {
        S.sc[SC_NRET] = nr;
        S.sc[SC_TKEY] = (int)tk;
      }
    }
    cbar();
    nret = S.sc[SC_NRET];
    tkey = (uint32_t)S.sc[SC_TKEY];
  } else {
    nret = select_inplace(cand, nc, K, &tkey, S);
  }
  // every element at or above each run's threshold is a candidate; the top-K cut is known only
  // when the K-th candidate reaches all of them
  const bool cut_ok = all_in || (nc >= K && tkey >= maxkey);
  if (!cut_ok) return false;
  const bool more = !(all_in && nret == nc);
  const uint32_t dkey = max(nc >= K ? tkey : 0u, maxkey);
  const uint32_t rflags = more ? REC_UNRETAINED : 0u;
  if (P.mode == 3) {
    if (w == 0) write_top(P, row, cand, nret);
    return true;
  }
  if (local) {  // this rank's shard record: the sorted entries and the completeness key
    if (nret > P.shard_cap) {
      if (tid == 0) write_flag_hdr(oh, REC_OVERFLOW, -INFINITY, 0.f);
      return true;
    }
    for (int j = tid; j < nret; j += NT) oe[j] = cand[j];
    if (tid == 0) {
      oh->m_y = -INFINITY;
      oh->s = 0.f;
      oh->n = nret;
      oh->t_key = rflags ? dkey : 0u;
      oh->flags = rflags;
    }
    return true;
  }
  MergeIn mi;
  mi.m_y = -INFINITY;
  mi.s = 0.f;
  mi.d_key = dkey;
  mi.flags = rflags;
  mi.n = nret;
  bool done;
  if (nret >= 1 && nret <= 64 && !c.greedy) {  // one warp, no CTA barriers
    if (w == 0) {
      const bool d = finalize_warp(P, c, row, mi, cand);
      if (lane == 0) S.sc[SC_X1] = d;
    }
    cbar();
    done = S.sc[SC_X1] != 0;
  } else {
    done = finalize_sorted(P, c, row, mi, cand, S);
  }
  cbar();
  return done;
}

// ---------------------------------------------------------------------------------------------
// k_stream: every row streamed once; each run leaves an unsorted candidate record
// ---------------------------------------------------------------------------------------------
// A run record (global workspace, one slot per row and run): the run's threshold on raw logits,
// its candidates (unsorted composite keys of every non-penalised element at or above the
// threshold), and for rows without top-k its maximum raw logit and the softmax sum of its raw
// logits relative to it. Greedy rows without penalties keep one entry instead: the run's
// smallest composite key.
struct RunRec {
  float m;           // largest raw logit of the run (rows without top-k)
  float s;           // sum of exp2((y - m) * log2(e) / T) over the run's raw logits
  uint32_t ylo_key;  // ordered key of the run's threshold on raw logits
  int32_t n;         // entries
  uint32_t flags;    // REC_*
  int32_t pad[3];
};
static_assert(sizeof(RunRec) == 32, "run record header is 32 bytes");

enum { MODE_GREEDY = 0, MODE_CANDS = 1, MODE_CANDS_SUM = 2 };

// The streaming loop of one run, specialised per kind of row so each variant keeps only its
// own state in registers: MODE 0 greedy (first index of the maximum), 1 candidates, 2
// candidates plus the online softmax sum of rows without top-k.
template <typename TIn, int MODE, bool BIGK = false>
__device__ __forceinline__ void stream_run(const KParams& P, Smem& S, int row, int seg_a,
                                           int seg_b, int K, float T, float c2, bool greedy,
                                           bool pen, SegLoad<TIn>& sa, float& m_t, float& s_t,
                                           unsigned long long& gbest) {
  using E = Elem<TIn>;
  constexpr int A = E::A;
  const int tid = threadIdx.x;
  const TIn* rowp = (const TIn*)P.logits + (int64_t)row * P.ld;
  float bestv = -INFINITY;
  auto process = [&](const SegLoad<TIn>& L, int seg) {
    float vm[U];
#pragma unroll
    for (int u = 0; u < U; ++u) vm[u] = (tid + NT * u < L.nvec) ? E::vmax(L.q[u]) : -INFINITY;
    if (MODE == MODE_CANDS_SUM) {  // online softmax sum over raw logits (corrected later)
#pragma unroll
      for (int u = 0; u < U; ++u) {
        if (tid + NT * u >= L.nvec) continue;
        if (vm[u] > m_t) {
          s_t *= ex2((m_t - vm[u]) * c2);
          m_t = vm[u];
        }
#pragma unroll
        for (int e = 0; e < A; ++e) s_t += ex2((E::at(L.q[u], e) - m_t) * c2);
      }
      if (L.sid >= 0) {
        if (L.sy > m_t) {
          s_t *= ex2((m_t - L.sy) * c2);
          m_t = L.sy;
        }
        s_t += ex2((L.sy - m_t) * c2);
      }
    }
    if (MODE == MODE_GREEDY) {  // first index of the maximum
#pragma unroll
      for (int u = 0; u < U; ++u) {
        if (vm[u] > bestv) {
          int e = 0;
          while (e < A - 1 && E::at(L.q[u], e) != vm[u]) ++e;
          const unsigned long long cc =
              comp(okey(vm[u]), (int)(L.gid0 + (int64_t)(tid + NT * u) * A + e));
          gbest = cc < gbest ? cc : gbest;
          bestv = vm[u];
        }
      }
      if (L.sid >= 0) {
        const unsigned long long cc = comp(okey(L.sy), (int)L.sid);
        gbest = cc < gbest ? cc : gbest;
      }
      return;
    }
    if (seg == seg_a) {
      if (BIGK) wide_first_bound<TIn>(P, L, vm, K, T, greedy, pen, S);
      else warp_first_bound<TIn>(P, L, vm, K, T, greedy, pen, S);
    }
    // the CTA's threshold as it stands: warps raise it as they go
    const float ylo = from_okey(*reinterpret_cast<volatile uint32_t*>(&S.ylo_key));
    int trig = -1;  // a block of the list this thread completed
#pragma unroll
    for (int u = 0; u < U; ++u) {
      if (tid + NT * u < L.nvec && vm[u] >= ylo) {  // rare
        const int id0 = (int)(L.gid0 + (int64_t)(tid + NT * u) * A);
        const int pos = dele_push(S, dele(vm[u], (uint32_t)id0), L.q[u]);
        if (pos % TB == TB - 1 && pos < CAND_BUF) trig = pos - (TB - 1);
      }
    }
    if (L.sid >= 0 && L.sy >= ylo) {
      const int pos = dele_push(S, dele(L.sy, DL_ONE | (uint32_t)L.sid),
                                make_uint4(__float_as_uint(L.sy), 0u, 0u, 0u));
      if (pos % TB == TB - 1 && pos < CAND_BUF) trig = pos - (TB - 1);
    }
    unsigned tb = __ballot_sync(FULLMASK, trig >= 0);
    while (tb) {  // rare: this warp completed a block of delegates
      const int src = __ffs(tb) - 1;
      tb &= tb - 1;
      const int b0 = __shfl_sync(FULLMASK, trig, src);
      if (BIGK) best_merge(P, b0, K, T, greedy, pen, A, S);
      else block_tighten(P, b0, K, T, greedy, pen, A, S);
    }
  };
  // one segment in flight per CTA (64 KiB): the other resident CTA of the SM keeps its loads
  // outstanding while this one processes
  for (int seg = seg_a; seg <= seg_b; ++seg) {
    if (seg > seg_a) load_segment<TIn>(P, rowp, seg, sa);  // the first was issued by run()
    process(sa, seg);
  }
}

// The row's history count of `id` among the staged entries (ascending ids); 0 when absent.
__device__ __forceinline__ int staged_count(const int* hid, const int* hcnt, int nh, int id) {
  int a = 0, b = nh;
  while (a < b) {
    const int mid = (a + b) >> 1;
    if (hid[mid] < id) a = mid + 1; else b = mid;
  }
  return (a < nh && hid[a] == id) ? hcnt[a] : 0;
}

// One run: segments seg_a..seg_b of `row`, streamed by the whole CTA. Its candidates end in
// shared memory (SSmem::rc). The CTA that completes the row (or streams all of it) finishes the
// row when the candidates decide it; otherwise the records go to the workspace and the row is
// marked ready for k_finish.
template <typename TIn>
__device__ __forceinline__ void run(const KParams& P, SSmem& X, int row, int seg_a, int seg_b) {
  Smem& S = X.s;
  const int tid = threadIdx.x;
  // the row's history span loads with its parameters (one round trip)
  const int64_t ia = P.hrow ? __ldg(P.hrow + row) : 0;
  const int64_t ib = P.hrow ? __ldg(P.hrow + row + 1) : 0;
  // the loop keeps only these scalars of the row's configuration
  bool greedy, pen, need_sum, active, mono;
  float T, c2;
  int K;
  uint32_t flags;
  {
    float prm[8];
#pragma unroll
    for (int i = 0; i < 8; ++i) prm[i] = load_param(P, row, i);
    if (tid == 0) {  // kept for the run's end (no global round trip there)
#pragma unroll
      for (int i = 0; i < 8; ++i) S.prm[i] = prm[i];
    }
    const RowCfg c = cfg_from(P, prm);
    if (tid == 0) S.cfg = c;
    greedy = c.greedy;
    pen = c.pen;
    need_sum = c.need_sum;
    active = !(c.bad || c.exact);
    flags = c.bad ? REC_BAD : (c.exact ? REC_EXACT : 0u);
    T = c.T;
    c2 = c.c2;
    K = c.greedy ? 1 : c.K;
    // penalties that never raise a logit: a penalised token reaches the threshold only if its
    // raw logit does, so the delegates hold it
    mono = c.rep >= 1.f && c.pres >= 0.f && c.freq >= 0.f;
  }
  const bool cands = !greedy || pen;  // greedy with penalties runs as top-1 candidates
  const int nh = (pen && active) ? (int)(ib - ia) : 0;
  const bool staged = pen && active && nh <= HCAP;
  // the history entries go out first, ahead of the segment's loads, straight to shared memory
  const int* hid = X.hid;
  const int* hcnt = X.hcnt;
  if (staged) {
    for (int j = tid; j < nh; j += NT) {
      cp_async4(&X.hid[j], P.hids + ia + j);
      cp_async4(&X.hcnt[j], P.hcnt + ia + j);
    }
  }
  SegLoad<TIn> first;
  if (active) load_segment<TIn>(P, (const TIn*)P.logits + (int64_t)row * P.ld, seg_a, first);
  // ---- a bitmap of the row's penalised ids of this shard (lookups: one shared-memory load)
  if (tid == 0) S.sc[SC_NH] = 0;
  if (pen && active) {
    uint32_t* bm = reinterpret_cast<uint32_t*>(S.scratch);
    const int words = (int)((P.V + 31) / 32);
    for (int i = tid; i < words; i += NT) bm[i] = 0u;
    if (tid == 0) {  // for the penalised candidates at the end of the run
      S.hpos = ia;
      S.sc[SC_NH] = nh;
    }
    if (staged) cp_async_wait_all();
    cbar();
    if (staged) {
      for (int j = tid; j < nh; j += NT) {
        const int64_t li = (int64_t)hid[j] - P.voff;
        if (hcnt[j] > 0 && li >= 0 && li < P.V) atomicOr(&bm[li >> 5], 1u << (li & 31));
      }
    } else {
      constexpr int PB = 8;  // entries per thread fetched together
      for (int j0 = 0; j0 < nh; j0 += PB * NT) {
        int id[PB], cn[PB];
#pragma unroll
        for (int k = 0; k < PB; ++k) {
          const int j = j0 + k * NT + tid;
          id[k] = j < nh ? __ldg(P.hids + ia + j) : 0;
          cn[k] = j < nh ? __ldg(P.hcnt + ia + j) : 0;
        }
#pragma unroll
        for (int k = 0; k < PB; ++k) {
          const int64_t li = (int64_t)id[k] - P.voff;
          if (cn[k] > 0 && li >= 0 && li < P.V) atomicOr(&bm[li >> 5], 1u << (li & 31));
        }
      }
    }
  }
  if (tid == 0) {
    S.sc[SC_NC] = 0;
    S.sc[SC_FB] = 0;
    S.sc[SC_NRET] = 0;
    S.ylo_key = okey(-INFINITY);
    S.dkth = ~0ull;
    S.sc[SC_LOCK] = 0;
    S.sc[SC_NBEST] = 0;
  }
  for (int i = tid; i < CAND_BUF; i += NT) S.cand[i] = ~0ull;
  float m_t = -FLT_MAX, s_t = 0.f;
  unsigned long long gbest = ~0ull;
  cbar();
  float m = -INFINITY, sum = 0.f;
  int n = 0;
  if (active) {
    if (!cands)
      stream_run<TIn, MODE_GREEDY>(P, S, row, seg_a, seg_b, K, T, c2, greedy, pen, first, m_t,
                                   s_t, gbest);
    else if (need_sum)
      stream_run<TIn, MODE_CANDS_SUM>(P, S, row, seg_a, seg_b, K, T, c2, greedy, pen, first,
                                      m_t, s_t, gbest);
    else if (K > 32)
      stream_run<TIn, MODE_CANDS, true>(P, S, row, seg_a, seg_b, K, T, c2, greedy, pen, first,
                                        m_t, s_t, gbest);
    else
      stream_run<TIn, MODE_CANDS>(P, S, row, seg_a, seg_b, K, T, c2, greedy, pen, first, m_t,
                                  s_t, gbest);
    cbar();
    // ---- the run's candidates: the delegates, the threshold, the sum of rows without top-k
    if (need_sum) {
      const uint32_t mk = cta_max_u32(okey(m_t == -FLT_MAX ? -INFINITY : m_t), S);
      m = from_okey(mk);
      const float part = (m_t == -FLT_MAX) ? 0.f : s_t * ex2((m_t - m) * c2);
      cta_excl_scan_f(part, &sum, S);
    }
    if (!cands) {
      const unsigned long long b = cta_min_u64(gbest, S);
      if (b != ~0ull) {
        if (tid == 0) S.cand[0] = b;
        n = 1;
      }
    } else if (S.sc[SC_NC] > CAND_BUF) {
      flags |= REC_OVERFLOW;  // ties of the threshold flooded the list: exact search
    } else {
      // the delegates at or above the final threshold are expanded (their 16 bytes were kept
      // in shared memory; past DV_CAP they are read again, from cache) and every element at or
      // above it is a candidate. Penalised elements: with penalties that never raise a logit,
      // their exact values here (count from the staged history); otherwise top-k rows gather
      // all their penalised tokens below, and rows without top-k leave them to k_finish, which
      // also corrects the softmax sum with them.
      using E = Elem<TIn>;
      const float ylo = from_okey(S.ylo_key);
      const int nd = S.sc[SC_NC];
      const TIn* rowp = (const TIn*)P.logits + (int64_t)row * P.ld;
      const RunHist h = hist_view(P, S);
      RowCfg cq{};
      cq.T = T;
      cq.greedy = greedy;
      const bool pen_here = pen && !need_sum && mono && staged;
      RowCfg cp{};  // what penalize() needs
      cp.rep = S.prm[3];
      cp.pres = S.prm[4];
      cp.freq = S.prm[5];
      // (1) every element of the delegates at or above the threshold whose raw logit reaches it,
      //     as (raw bits, id) in SSmem::rc
      if (tid == 0) S.sc[SC_X1] = 0;
      cbar();
      for (int i = tid; i < nd; i += NT) {
        const unsigned long long x = S.cand[i];
        if (!(dele_max(x) >= ylo)) continue;
        const uint32_t xb = (uint32_t)x;
        const int id0 = (int)(xb & DL_ID);
        uint4 q;
        if (i < DV_CAP) {
          q = S.dv[i];
        } else {
          const int64_t li = (int64_t)id0 - P.voff;
          if (xb & DL_ONE) q = make_uint4(__float_as_uint(E::ld(rowp, li)), 0u, 0u, 0u);
          else q = __ldg(reinterpret_cast<const uint4*>(rowp + li));
        }
        const int ne = (xb & DL_ONE) ? 1 : E::A;
#pragma unroll 1
        for (int e = 0; e < ne; ++e) {
          const float y = (xb & DL_ONE) ? __uint_as_float(q.x) : E::at(q, e);
          if (y >= ylo) {
            const int pos = atomicAdd(&S.sc[SC_X1], 1);
            if (pos < CAND_CAP)
              X.rc[pos] = ((unsigned long long)__float_as_uint(y) << 32) | (uint32_t)(id0 + e);
          }
        }
      }
      cbar();
      // (2) one element per thread: penalties, the processed value, the candidate entry; the
      //     delegate list is spent, so the candidates go to Smem::cand (warp-aggregated slots)
      const int nq = S.sc[SC_X1];
      if (nq > CAND_CAP) {
        flags |= REC_OVERFLOW;
      } else {
        for (int j0 = 0; j0 < nq; j0 += NT) {
          const int j = j0 + tid;
          bool keep = false;
          unsigned long long ce = 0ull;
          if (j < nq) {
            const unsigned long long r = X.rc[j];
            float y = __uint_as_float((uint32_t)(r >> 32));
            const int id = (int)(uint32_t)r;
            keep = true;
            if (pen && hist_count(h, id) > 0) {
              keep = pen_here;  // otherwise gathered below (or, without top-k, by k_finish)
              if (keep) {
                y = penalize(y, staged_count(hid, hcnt, nh, id), cp);
                keep = y >= ylo;
              }
            }
            if (keep) ce = comp(okey(vf(y, cq)), id);
          }
          const unsigned bal = __ballot_sync(FULLMASK, keep);
          int base = 0;
          if ((tid & 31) == 0 && bal) base = atomicAdd(&S.sc[SC_NRET], __popc(bal));
          base = __shfl_sync(FULLMASK, base, 0);
          if (keep) S.cand[base + __popc(bal & ((1u << (tid & 31)) - 1u))] = ce;
        }
      }
      if (pen && !need_sum && !pen_here) {
        // the penalised tokens of this run's ids at or above the threshold, with their exact
        // values (their logits were just streamed, so from cache)
        const int64_t idlo = P.voff + (int64_t)seg_a * P.seg_len;
        const int64_t idhi = P.voff + min(P.V, (int64_t)(seg_b + 1) * P.seg_len);
        constexpr int PB = 8;  // entries per thread fetched together
        for (int j0 = 0; j0 < nh; j0 += PB * NT) {
          int id[PB], cn[PB];
          float raw[PB];
#pragma unroll
          for (int k = 0; k < PB; ++k) {
            const int j = j0 + k * NT + tid;
            id[k] = j < nh ? (staged ? hid[j] : __ldg(P.hids + ia + j)) : 0;
            cn[k] = j < nh ? (staged ? hcnt[j] : __ldg(P.hcnt + ia + j)) : 0;
          }
#pragma unroll
          for (int k = 0; k < PB; ++k) {
            if (id[k] < idlo || id[k] >= idhi) cn[k] = 0;  // another run's, or outside the shard
            raw[k] = cn[k] > 0 ? E::ld(rowp, (int64_t)id[k] - P.voff) : 0.f;
          }
#pragma unroll
          for (int k = 0; k < PB; ++k) {
            if (cn[k] <= 0) continue;
            const float yt = penalize(raw[k], cn[k], cp);
            if (yt >= ylo) {
              const int pos = atomicAdd(&S.sc[SC_NRET], 1);
              if (pos < CAND_BUF) S.cand[pos] = comp(okey(vf(yt, cq)), id[k]);
            }
          }
        }
      }
      cbar();
      n = S.sc[SC_NRET];
      if (n > CAND_CAP) {
        flags |= REC_OVERFLOW;
        n = 0;
      }
    }
  }
  cbar();
  // ---- publish: finish the row here, or leave the record for the CTA completing the row / k_finish
  const uint32_t ylo_key = S.ylo_key;
  const int r0 = seg_owner(P, row * P.nseg);
  const int nruns = seg_owner(P, row * P.nseg + P.nseg - 1) - r0 + 1;
  unsigned char* base = P.recs + (size_t)row * P.nseg * REC_STRIDE;
  unsigned char* rec = base + (size_t)(blockIdx.x - r0) * REC_STRIDE;
  RunRec* hd = reinterpret_cast<RunRec*>(rec);
  unsigned long long* ent = reinterpret_cast<unsigned long long*>(rec + sizeof(RunRec));
  RowCfg cq{};
  cq.T = T;
  cq.greedy = greedy;
  auto write_record = [&]() {
    for (int j = tid; j < n; j += NT) ent[j] = S.cand[j];
    if (tid == 0) {
      hd->m = m;
      hd->s = sum;
      hd->ylo_key = ylo_key;
      hd->n = n;
      hd->flags = flags;
    }
  };
  bool done = false;
  if (nruns == 1) {  // this CTA streamed the whole row
    if (flags == 0 && !need_sum) {
      const float y = from_okey(ylo_key);
      const bool all_in = !(y > -INFINITY);
      done = fast_finish(P, S, row, S.cand, n, all_in ? 0u : okey(vf(y, cq)), all_in);
    }
    if (!done) write_record();
    // the barrier orders every thread's writes before thread 0's fence, whose release covers
    // them. A finished row needs no fence: k_finish reads nothing of it, and waits for this grid
    // to complete before it exits itself.
    cbar();
    if (tid == 0) {
      if (done && !P.slot_ids) {
        *reinterpret_cast<volatile int*>(P.counters + row) = CNT_DONE;
      } else {  // records, or (decode) the row's id that k_finish counts into its slot
        __threadfence();
        st_release(P.counters + row, done ? CNT_DONE : CNT_READY);
      }
    }
    return;
  }
  write_record();
  cbar();
  if (tid == 0) {
    __threadfence();
    S.sc[SC_LAST] = atom_add_acq_rel(P.counters + row, 1) == nruns - 1;
  }
  cbar();
  if (!S.sc[SC_LAST]) return;
  // the CTA completing the row: every run's header, then (when they allow it) their candidates
  RunRec* rh = reinterpret_cast<RunRec*>(S.mh);
  if (tid < nruns) {
    const RunRec* src = reinterpret_cast<const RunRec*>(base + (size_t)tid * REC_STRIDE);
    RunRec r;
    r.ylo_key = __ldcg(&src->ylo_key);
    r.n = __ldcg(&src->n);
    r.flags = __ldcg(&src->flags);
    rh[tid] = r;
  }
  cbar();
  if (tid == 0) {
    uint32_t fl = 0, maxkey = 0;
    int tot = 0, all_in = 1;
    for (int r = 0; r < nruns; ++r) {
      fl |= rh[r].flags;
      S.moff[r] = tot;
      tot += rh[r].n;
      const float y = from_okey(rh[r].ylo_key);
      if (y > -INFINITY) {
        all_in = 0;
        maxkey = max(maxkey, okey(vf(y, cq)));
      }
    }
    S.moff[nruns] = tot;
    S.sc[SC_X0] = (fl == 0 && !need_sum && tot <= CAND_BUF) ? tot : -1;
    S.sc[SC_J] = (int)maxkey;
    S.sc[SC_B] = all_in;
  }
  cbar();
  const int tot = S.sc[SC_X0];
  if (tot >= 0) {
    for (int idx = tid; idx < tot; idx += NT) {
      int r = 0;
      while (S.moff[r + 1] <= idx) ++r;
      const unsigned long long* re = reinterpret_cast<const unsigned long long*>(
          base + (size_t)r * REC_STRIDE + sizeof(RunRec));
      S.cand[idx] = __ldcg(re + (idx - S.moff[r]));
    }
    cbar();
    done = fast_finish(P, S, row, S.cand, tot, (uint32_t)S.sc[SC_J], S.sc[SC_B] != 0);
  }
  cbar();
  if (tid == 0) {
    if (done && !P.slot_ids) {
      *reinterpret_cast<volatile int*>(P.counters + row) = CNT_DONE;
    } else {
      __threadfence();
      st_release(P.counters + row, done ? CNT_DONE : CNT_READY);
    }
  }
}

template <typename TIn>
__global__ void __launch_bounds__(NT, 2) k_stream(const __grid_constant__ KParams P) {
  extern __shared__ __align__(128) unsigned char smraw[];
  SSmem& X = *reinterpret_cast<SSmem*>(smraw);
  // k_finish may be scheduled as soon as SMs free up; it waits for this grid's records itself
  asm volatile("griddepcontrol.launch_dependents;" ::: "memory");
  const int s0 = seg_begin(P, blockIdx.x), s1 = seg_begin(P, blockIdx.x + 1);
  int sg = s0;
  while (sg < s1) {
    const int row = sg / P.nseg;
    const int seg_a = sg - row * P.nseg;
    const int seg_b = min(s1 - row * P.nseg, P.nseg) - 1;
    run<TIn>(P, X, row, seg_a, seg_b);
    cbar();
    sg = row * P.nseg + seg_b + 1;
  }
}

// ---------------------------------------------------------------------------------------------
// slotted histories (decode loop): one slot's in-place update
// ---------------------------------------------------------------------------------------------
constexpr int HIST_NT = 256;

// padding id of position p of a slot with cap entries (ascending, above every vocabulary id)
__device__ __forceinline__ int hist_pad_id(int cap, int p) {
  return VINFER_HIST_PAD_ID - (cap - 1 - p);
}

// Counts token t once more in slot s, or inserts it in id order (entries from its place on move
// up by one: read all, then written, when they fit the CTA's registers; otherwise chunk by chunk
// from the top, so no entry is overwritten before it is read). The whole CTA (HIST_NT threads).
__device__ __forceinline__ void slot_append(int* ids, int* cnts, int* lens, int cap, int s, int t,
                                            int* status) {
  const int tid = threadIdx.x;
  int* sid = ids + (int64_t)s * cap;
  int* sc = cnts + (int64_t)s * cap;
  const int n = min(max(lens[s], 0), cap);
  __shared__ int pos_s, found_s;
  if (tid < 32) {
    // the first entry whose id is >= t: a warp-wide search, 32 probes per round (each round
    // narrows [lo, hi] to a 33rd); the predicate sid[q] < t is monotone in q
    int lo = 0, hi = n;
    while (hi - lo > 32) {
      const int step = (hi - lo + 32) / 33;
      const int q = min(lo + (tid + 1) * step, hi) - 1;
      const int k = __popc(__ballot_sync(FULLMASK, sid[q] < t));
      const int nlo = min(lo + k * step, hi);
      if (k < 32) hi = min(lo + (k + 1) * step, hi);
      lo = nlo;
    }
    const int q = lo + tid;
    const int pos = lo + __popc(__ballot_sync(FULLMASK, q < hi && sid[q] < t));
    if (tid == 0) {
      pos_s = pos;
      found_s = pos < n && sid[pos] == t;
    }
  }
  __syncthreads();
  const int pos = pos_s;
  if (found_s) {
    if (tid == 0) sc[pos] += 1;
    return;
  }
  if (n >= cap) {
    if (tid == 0 && status) atomicOr(reinterpret_cast<unsigned int*>(status), VINFER_ST_HIST_FULL);
    return;
  }
  constexpr int PER = 8;  // entries a thread moves in the one-pass shift
  if (n - pos <= PER * HIST_NT) {
    // one pass: every entry of [pos, n) read into registers, then written one place up
    int a[PER], c[PER];
#pragma unroll
    for (int k = 0; k < PER; ++k) {
      const int i = pos + k * HIST_NT + tid;
      a[k] = i < n ? sid[i] : 0;
      c[k] = i < n ? sc[i] : 0;
    }
    __syncthreads();
#pragma unroll
    for (int k = 0; k < PER; ++k) {
      const int i = pos + k * HIST_NT + tid;
      if (i < n) {
        sid[i + 1] = a[k];
        sc[i + 1] = c[k];
      }
    }
  } else {
    for (int hi = n; hi > pos; hi -= HIST_NT) {  // entries [lo, hi) move to [lo + 1, hi + 1)
      const int lo = max(pos, hi - HIST_NT);
      const int i = lo + tid;
      int a = 0, c = 0;
      if (i < hi) {
        a = sid[i];
        c = sc[i];
      }
      __syncthreads();
      if (i < hi) {
        sid[i + 1] = a;
        sc[i + 1] = c;
      }
      __syncthreads();
    }
  }
  __syncthreads();
  if (tid == 0) {
    sid[pos] = t;
    sc[pos] = 1;
    lens[s] = n + 1;
  }
}

// ---------------------------------------------------------------------------------------------
// k_finish: one CTA per row gathers its runs' records, selects, cuts and draws (or writes this
// rank's shard record), falling back to the exact search when the candidates cannot decide the
// row
// ---------------------------------------------------------------------------------------------

// A row the streaming kernel left ready (its records are complete): the whole CTA.
template <typename TIn>
__device__ __forceinline__ void finish_ready(const KParams& P, Smem& S) {
  using E = Elem<TIn>;
  const int tid = threadIdx.x, lane = tid & 31, w = tid >> 5;
  const int row = blockIdx.x;
  const RowCfg c = load_row(P, row);
  const int r0 = seg_owner(P, row * P.nseg);
  const int nruns = seg_owner(P, row * P.nseg + P.nseg - 1) - r0 + 1;
  const unsigned char* base = P.recs + (size_t)row * P.nseg * REC_STRIDE;
  const TIn* rowp = (const TIn*)P.logits + (int64_t)row * P.ld;
  RunRec* rh = reinterpret_cast<RunRec*>(S.mh);  // the run headers (32 bytes each)
  static_assert(sizeof(RunRec) == sizeof(RecHdr), "run headers fit Smem::mh");
  // the candidate list lives in the first half of scratch, the row's history in the second:
  // ids, then the penalised value of each entry (NaN when its count is not positive)
  unsigned long long* cand = S.scratch;
  constexpr int FCAP = SCRATCH / 2;  // candidates; also history entries staged
  int* hid = reinterpret_cast<int*>(S.scratch + FCAP);
  float* htv = reinterpret_cast<float*>(hid + FCAP);
  if (tid < nruns) {
    // the end of run tid: its CTA's last segment of this row
    const int se = min(seg_begin(P, r0 + tid + 1) - row * P.nseg, P.nseg);
    S.rhi[tid] = (int)(P.voff + min(P.V, (int64_t)se * P.seg_len));
  }
  if (tid == 0) S.sc[SC_NH] = 0;
  // rows with top-k (and greedy rows) find their penalised tokens in the run records; rows
  // without top-k stage the history here to correct the softmax sum
  const bool hist_here = c.pen && c.need_sum;
  if (hist_here && tid < 32) {  // the row's history entries inside this shard
    const int64_t a = __ldg(P.hrow + row), b = __ldg(P.hrow + row + 1);
    int64_t ia = a, ib = b;
    if (P.voff != 0 || P.V != P.vtotal) {  // a shard: search its part of the row
      ia = warp_lower_bound(P.hids, a, b, P.voff, lane);
      ib = warp_lower_bound(P.hids, ia, b, P.voff + P.V, lane);
    }
    if (lane == 0) {
      S.hpos = ia;
      S.sc[SC_NH] = (int)(ib - ia);
    }
  }
  cbar();
  const bool greedy_plain = c.greedy && !c.pen;
  const int K = c.greedy ? 1 : c.K;
  const int nh = S.sc[SC_NH];
  const bool hshared = nh <= FCAP;
  // ---- the penalised values of the history entries
  if (hist_here && hshared) {
    constexpr int PB = 8;  // entries per thread whose ids and logits are fetched together
    for (int j0 = 0; j0 < nh; j0 += PB * NT) {
      int id[PB], cn[PB];
      float raw[PB];
#pragma unroll
      for (int k = 0; k < PB; ++k) {
        const int j = j0 + k * NT + tid;
        id[k] = j < nh ? __ldg(P.hids + S.hpos + j) : 0;
        cn[k] = j < nh ? __ldg(P.hcnt + S.hpos + j) : 0;
      }
#pragma unroll
      for (int k = 0; k < PB; ++k) {
        const int64_t li = (int64_t)id[k] - P.voff;
        if (li < 0 || li >= P.V) cn[k] = 0;  // not a token of this shard (or of the vocabulary)
        raw[k] = cn[k] > 0 ? E::ld(rowp, li) : 0.f;
      }
#pragma unroll
      for (int k = 0; k < PB; ++k) {
        const int j = j0 + k * NT + tid;
        if (j < nh) {
          hid[j] = id[k];
          htv[j] = cn[k] > 0 ? penalize(raw[k], cn[k], c) : __int_as_float(0x7fc00000);
        }
      }
    }
  }
  if (tid < nruns) {
    const RunRec* src = reinterpret_cast<const RunRec*>(base + (size_t)tid * REC_STRIDE);
    RunRec r;
    r.m = __ldcg(&src->m);
    r.s = __ldcg(&src->s);
    r.ylo_key = __ldcg(&src->ylo_key);
    r.n = __ldcg(&src->n);
    r.flags = __ldcg(&src->flags);
    rh[tid] = r;
  }
  if (tid == 0) P.counters[row] = 0;  // ready for the next call (stream-ordered after this one)
  cbar();
  if (tid == 0) {
    uint32_t fl = 0;
    float m = -INFINITY;
    int tot = 0;
    for (int r = 0; r < nruns; ++r) {
      fl |= rh[r].flags;
      m = fmaxf(m, rh[r].m);
      S.moff[r] = tot;
      tot += rh[r].n;
    }
    S.moff[nruns] = tot;
    float sum = 0.f;
    if (c.need_sum)
      for (int r = 0; r < nruns; ++r)
        if (rh[r].m > -INFINITY) sum += rh[r].s * ex2((rh[r].m - m) * c.c2);
    S.sc[SC_X0] = (int)fl;
    S.sf[SF_M] = m;
    S.sf[SF_SK] = sum;
    S.sc[SC_NC] = 0;
    S.dkth = ~0ull;
  }
  cbar();
  uint32_t flags = (uint32_t)S.sc[SC_X0];
  const float m_y = S.sf[SF_M];
  float s_run = S.sf[SF_SK];
  const int ntot = S.moff[nruns];
  const bool local = P.mode == 1;
  unsigned char* shard = local ? P.shard_out + (size_t)row * P.shard_stride : nullptr;
  if (flags & REC_BAD) {
    if (P.mode == 3) {
      if (w == 0) write_top(P, row, cand, 0);
      return;
    }
    if (tid == 0) {
      if (local) {
        write_flag_hdr(reinterpret_cast<RecHdr*>(shard), REC_BAD, m_y, s_run);
      } else {
        write_state(P, row, 3, -1, 0.f, 0.f, 0u, 0);
        status_or(P, VINFER_ST_BAD_PARAM);
      }
    }
    return;
  }
  // with more history entries than the staging area holds, the row takes the exact search
  bool exact = (flags & (REC_EXACT | REC_OVERFLOW)) != 0 || ntot > CAND_BUF ||
               (hist_here && !hshared);
  int nret = 0;
  uint32_t dkey = 0, rflags = 0;
  RowCfg cq{};  // what vf() needs
  cq.T = c.T;
  cq.greedy = c.greedy;
  // the run of global id `id` (of this shard)
  auto run_of = [&](int id) {
    int r = 0;
    while (r < nruns - 1 && id >= S.rhi[r]) ++r;
    return r;
  };
  bool sorted_done = false;  // the candidates are sorted and cut (short-list path)
  if (!exact) {
    // ---- the runs' candidates (or greedy entries)
    for (int idx = tid; idx < ntot; idx += NT) {
      int r = 0;
      while (S.moff[r + 1] <= idx) ++r;
      const unsigned long long* re = reinterpret_cast<const unsigned long long*>(
          base + (size_t)r * REC_STRIDE + sizeof(RunRec));
      cand[idx] = __ldcg(re + (idx - S.moff[r]));
    }
    if (tid == 0) S.sc[SC_NC] = ntot;
    cbar();
    if (greedy_plain) {
      // one entry per run: the smallest composite key is the first index of the maximum
      unsigned long long b = ~0ull;
      for (int i = 0; i < ntot; ++i) b = cand[i] < b ? cand[i] : b;
      cbar();
      if (tid == 0) cand[0] = b;
      nret = b != ~0ull;
      rflags = (nret && P.V > 1) ? REC_UNRETAINED : 0u;
      dkey = nret ? comp_key(b) : 0u;
      cbar();
    } else {
      // ---- the penalised tokens with their exact values (computed before the wait)
      if (hist_here) {
        for (int j = tid; j < nh; j += NT) {
          const float yt = htv[j];
          if (!(yt == yt)) continue;
          if (yt >= from_okey(rh[run_of(hid[j])].ylo_key)) {
            const int pos = atomicAdd(&S.sc[SC_NC], 1);
            if (pos < FCAP) cand[pos] = comp(okey(vf(yt, c)), hid[j]);
          }
        }
        if (c.need_sum) {  // their terms in the softmax sum replaced
          float draw = 0.f, dtrue = 0.f;
          for (int j = tid; j < nh; j += NT) {
            const float yt = htv[j];
            if (!(yt == yt)) continue;
            const float raw = E::ld(rowp, (int64_t)hid[j] - P.voff);
            draw += ex2((raw - m_y) * c.c2);
            dtrue += ex2((yt - m_y) * c.c2);
          }
          float dr, dt;
          cta_excl_scan_f(draw, &dr, S);
          cta_excl_scan_f(dtrue, &dt, S);
          if (dr > 0.5f * s_run) exact = true;  // cancellation: the exact search decides
          s_run = s_run - dr + dt;
        }
      }
      cbar();
      const int nc = S.sc[SC_NC];
      uint32_t maxkey = 0;
      bool all_in = true;
      for (int r = 0; r < nruns; ++r) {
        const float y = from_okey(rh[r].ylo_key);
        if (y > -INFINITY) {
          all_in = false;
          maxkey = max(maxkey, okey(vf(y, cq)));
        }
      }
      if (nc > FCAP) {
        exact = true;
      } else if (nc <= 32) {
        // short list: one warp sorts it and applies the cut (no CTA barrier)
        if (w == 0) {
          unsigned long long x = lane < nc ? cand[lane] : ~0ull;
          x = warp_sort32(x);
          cand[lane] = x;
          const unsigned long long kx = __shfl_sync(FULLMASK, x, min(K, 32) - 1);
          const uint32_t tkey = nc >= K ? comp_key(kx) : 0u;
          const int nr = nc >= K ? __popc(__ballot_sync(FULLMASK, lane < nc &&
                                                                  comp_key(x) >= tkey))
                                 : nc;
          if (lane == 0) {
            S.sc[SC_NRET] = nr;
            S.sc[SC_TKEY] = (int)tkey;
          }
        }
        cbar();
        nret = S.sc[SC_NRET];
        const uint32_t tkey = (uint32_t)S.sc[SC_TKEY];
        const bool cut_ok = all_in || (nc >= K && tkey >= maxkey);
        if ((c.topk || c.greedy) && !cut_ok) exact = true;
        const bool more = !(all_in && nret == nc);
        dkey = max(nc >= K ? tkey : 0u, maxkey);
        rflags = more ? REC_UNRETAINED : 0u;
        sorted_done = true;
      } else {
        uint32_t tkey;
        nret = select_inplace(cand, nc, K, &tkey, S);
        // every element at or above each run's threshold is a candidate; the top-K cut is
        // known only when the K-th candidate reaches all of them
        const bool cut_ok = all_in || (nc >= K && tkey >= maxkey);
        if ((c.topk || c.greedy) && !cut_ok) exact = true;
        const bool more = !(all_in && nret == nc);
        dkey = max(nc >= K ? tkey : 0u, maxkey);
        rflags = more ? REC_UNRETAINED : 0u;
      }
    }
  }
  (void)sorted_done;
  if (P.mode == 3) {  // rows the candidates cannot decide (ties flooding a list) report none
    if (w == 0) write_top(P, row, cand, exact ? 0 : nret);
    return;
  }
  if (local) {  // this rank's shard record: the sorted entries and the completeness key
    RecHdr* oh = reinterpret_cast<RecHdr*>(shard);
    unsigned long long* oe = reinterpret_cast<unsigned long long*>(shard + sizeof(RecHdr));
    if (exact || nret > P.shard_cap) {
      if (tid == 0) write_flag_hdr(oh, REC_OVERFLOW, m_y, s_run);
      return;
    }
    for (int j = tid; j < nret; j += NT) oe[j] = cand[j];
    if (tid == 0) {
      oh->m_y = m_y;
      oh->s = s_run;
      oh->n = nret;
      oh->t_key = rflags ? dkey : 0u;
      oh->flags = rflags;
    }
    return;
  }
  bool done = false;
  if (!exact) {
    MergeIn mi;
    mi.m_y = m_y;
    mi.s = s_run;
    mi.d_key = dkey;
    mi.flags = rflags;
    mi.n = nret;
    if (nret >= 1 && nret <= 64 && !c.greedy) {  // one warp, no CTA barriers
      if (tid < 32) {
        const bool d = finalize_warp(P, c, row, mi, cand);
        if (tid == 0) S.sc[SC_X1] = d;
      }
      cbar();
      done = S.sc[SC_X1] != 0;
    } else {
      done = finalize_sorted(P, c, row, mi, cand, S);
    }
  }
  cbar();
  if (!done) exact_row<TIn>(P, c, row, S, reinterpret_cast<unsigned char*>(S.scratch));
}

// One CTA per row. The row's counter carries a mark once the streaming kernel is through with
// the row (CNT_DONE: finished there; CNT_READY: records complete); a bounded wait for it first,
// and should it run out, the wait for the whole streaming grid (which always ends). Every CTA
// also waits for the streaming grid before it exits, so this grid completes after it: work
// queued behind the sampler may read every row's outputs.
template <typename TIn>
__global__ void __launch_bounds__(NT, 3) k_finish(const __grid_constant__ KParams P) {
  extern __shared__ __align__(128) unsigned char smraw[];
  Smem& S = *reinterpret_cast<Smem*>(smraw);
  const int tid = threadIdx.x, row = blockIdx.x;
  if (tid == 0) {
    int v = 0;
    for (int it = 0; it < 20000; ++it) {
      v = ld_acquire(P.counters + row);
      if (v >= CNT_READY) break;
      __nanosleep(128);
    }
    S.sc[SC_LAST] = v;
  }
  cbar();
  if (S.sc[SC_LAST] < CNT_READY) {
    asm volatile("griddepcontrol.wait;" ::: "memory");
    cbar();
    if (tid == 0) S.sc[SC_LAST] = ld_acquire(P.counters + row);
    cbar();
  }
  if (S.sc[SC_LAST] & CNT_DONE) {
    if (tid == 0) P.counters[row] = 0;  // ready for the next call (stream-ordered after this one)
  } else {
    finish_ready<TIn>(P, S);
  }
  if (P.slot_ids) {
    // decode: the row's id, final now (written by this CTA, or by the streaming kernel before
    // its release of the mark this CTA acquired), counted into the row's slot; every read of
    // the slot's history for this step is over
    cbar();
    if (tid == 0) S.sc[SC_J] = __ldcg(P.out_ids + row);
    cbar();
    const int t = S.sc[SC_J];
    if (t >= 0) slot_append(P.slot_ids, P.slot_cnt, P.hlen, P.hcap, row, t, P.status);
  }
  asm volatile("griddepcontrol.wait;" ::: "memory");
}

// ---------------------------------------------------------------------------------------------
// kernels: sharded merge and probabilities
// ---------------------------------------------------------------------------------------------
// merge of gathered shard records: one CTA per row
template <typename TIn>
__global__ void __launch_bounds__(NT, 1) k_merge(const __grid_constant__ KParams P, const unsigned char* recs,
                                              int world, int* unresolved) {
  extern __shared__ __align__(128) unsigned char smraw[];
  Smem& S = *reinterpret_cast<Smem*>(smraw);
  const int row = blockIdx.x;
  finish_row<TIn>(P, S, (unsigned char*)S.scratch, row, recs + (size_t)row * P.shard_stride,
                  (size_t)P.B * P.shard_stride, world, false, unresolved);
}

// final probabilities [B, V] from the row states (parity checks only)
template <typename TIn>
__global__ void __launch_bounds__(256) k_probs(const __grid_constant__ KParams P) {
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

// log-probability of each row's sampled token under the row's final distribution (penalties,
// temperature, top-k / top-p / min-p, renormalised), from the row state the finishing step
// left: ln p = (v_token - m_v) - ln(s_kept), where v_token is the token's processed logit.
// One thread per row; greedy rows give 0 (their distribution is one-hot), rows without a
// result NaN.
template <typename TIn>
__global__ void __launch_bounds__(128) k_logprobs(const __grid_constant__ KParams P, float* out) {
  const int row = blockIdx.x * blockDim.x + threadIdx.x;
  if (row >= P.B) return;
  const RowState st = P.rows[row];
  if (st.kind == 3 || st.token < 0) {
    out[row] = __int_as_float(0x7fc00000);
    return;
  }
  if (st.kind == 2) {
    out[row] = 0.f;
    return;
  }
  const RowCfg c = load_row(P, row);
  const int64_t li = (int64_t)st.token - P.voff;
  float y = Elem<TIn>::ld((const TIn*)P.logits + (int64_t)row * P.ld, li);
  if (c.pen) {
    const int64_t ha = __ldg(P.hrow + row), hb = __ldg(P.hrow + row + 1);
    const int64_t q = lower_bound_ids(P.hids, ha, hb, st.token);
    if (q < hb && __ldg(P.hids + q) == st.token && __ldg(P.hcnt + q) > 0)
      y = penalize(y, __ldg(P.hcnt + q), c);
  }
  out[row] = (vf(y, c) - st.m_v) - logf(st.s_kept);
}

// ---------------------------------------------------------------------------------------------
// slotted histories: in-place count updates between decode steps
// ---------------------------------------------------------------------------------------------
// One CTA per slot: tokens[s] counted once more in slot s (slot_append).
__global__ void __launch_bounds__(HIST_NT, 2) k_hist_append(const int* tokens, int* ids, int* cnts,
                                                         int* lens, int cap, int* status) {
  // launched as a programmatic dependent of the sampler: its ids are final once the kernel
  // before this one has completed
  asm volatile("griddepcontrol.wait;" ::: "memory");
  const int t = tokens[blockIdx.x];
  if (t < 0) return;  // no token this step (an invalid row's id is -1)
  slot_append(ids, cnts, lens, cap, blockIdx.x, t, status);
}

// One CTA per listed slot: every entry back to padding, the length to zero.
__global__ void __launch_bounds__(HIST_NT) k_hist_reset(const int* slot_list, int64_t slots,
                                                        int* ids, int* cnts, int* lens, int cap) {
  const int s = __ldg(slot_list + blockIdx.x);
  if (s < 0 || s >= slots) return;
  for (int p = threadIdx.x; p < cap; p += HIST_NT) {
    ids[(int64_t)s * cap + p] = hist_pad_id(cap, p);
    cnts[(int64_t)s * cap + p] = 0;
  }
  if (threadIdx.x == 0) lens[s] = 0;
}

// ---------------------------------------------------------------------------------------------
// host side
// ---------------------------------------------------------------------------------------------
struct Shape {
  int nseg, seg_len, grid;
};

// Segments per row and CTAs for a batch. A row is cut into at least enough segments of at most
// SEG_BYTES. When the batch has fewer rows than the device has resident CTAs, each row is cut
// into c = ctas / B runs of whole segments (nseg a multiple of c, segments of at least 2048
// tokens), so every CTA streams one run. With as many rows as CTAs or more, each CTA takes r =
// ceil(B / ctas) whole rows (the fewest CTAs that hold the batch; the CTAs share the row-major
// list of segments in equal contiguous ranges, which are whole rows when r divides B): a row
// then is one run, finished by its own CTA, instead of a run split over two CTAs whose second
// must gather the first's record (measured on configuration 4: 198 against 216 us a batch).
Shape plan(int64_t B, int64_t V, int dtype, int ctas) {
  const int es = dtype == VINFER_DTYPE_BF16 ? 2 : 4;
  const int A = 16 / es;
  const int64_t min_seg = (V * es + SEG_BYTES - 1) / SEG_BYTES;
  int64_t c = 1;
  if (B < ctas) c = std::min<int64_t>(ctas / B, MAX_NSEG);
  c = std::max<int64_t>(1, std::min<int64_t>(c, V / 2048));
  int64_t nseg = std::max<int64_t>(min_seg, c);
  nseg = (nseg + c - 1) / c * c;
  nseg = std::min<int64_t>(nseg, MAX_NSEG);
  int64_t len = (V + nseg - 1) / nseg;
  len = (len + A - 1) / A * A;
  nseg = (V + len - 1) / len;
  Shape s;
  s.nseg = (int)nseg;
  s.seg_len = (int)len;
  if (B < ctas) {
    s.grid = (int)std::min<int64_t>(B * nseg, B * c);
  } else {  // whole rows per CTA: r rows each, the fewest CTAs that hold the batch
    const int64_t r = (B + ctas - 1) / ctas;
    s.grid = (int)((B + r - 1) / r);
  }
  return s;
}

// An NVTX range over one entry point's host work (argument checks and launches), so profiler
// timelines group a call's kernels under its name (NVTX is header-only and costs nothing when no
// tool is attached).
struct NvtxRange {
  explicit NvtxRange(const char* name) { nvtxRangePushA(name); }
  ~NvtxRange() { nvtxRangePop(); }
  NvtxRange(const NvtxRange&) = delete;
  NvtxRange& operator=(const NvtxRange&) = delete;
};

constexpr size_t ALIGN = 256;
size_t align_up(size_t x) { return (x + ALIGN - 1) / ALIGN * ALIGN; }

// Every workspace starts with the per-row arrival counters for the largest batch, whose place
// and size do not depend on the shape: a workspace used for calls of different shapes never
// finds another call's records over its counters, and every call leaves them at zero.
constexpr size_t HDR_BYTES = ((size_t)VINFER_MAX_BATCH * 4 + ALIGN - 1) / ALIGN * ALIGN;

struct WsLayout {
  size_t counters, rows, recs, total;
};
// Records: one slot per (row, run); a row has at most nseg runs. Below the resident-CTA bound
// rows may be split up to MAX_NSEG ways, depending on the device; from it on, the segment size
// alone sets nseg. Either way the size does not depend on the device.
WsLayout ws_layout(int64_t B, int64_t V, int dtype) {
  const int64_t nseg = B < CTA_CAP ? MAX_NSEG : plan(B, V, dtype, CTA_CAP).nseg;
  WsLayout L;
  L.counters = 0;
  L.rows = HDR_BYTES;
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
// CTAs of it fit on the device at once (first calls from several host threads are serialised)
struct KernInfo {
  bool ready;
  int ctas;
};
std::mutex g_info_mu;
int kernel_info(const void* kern, int slot, int threads, size_t smem, int* ctas) {
  static KernInfo info[64][6] = {};
  int dev = 0;
  if (cudaGetDevice(&dev) != cudaSuccess || dev < 0 || dev >= 64) return VINFER_E_CUDA;
  std::lock_guard<std::mutex> lock(g_info_mu);
  KernInfo& k = info[dev][slot];
  if (!k.ready) {
    if (cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem) !=
        cudaSuccess)
      return VINFER_E_CUDA;
    int sms = 0, per_sm = 0;
    if (cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev) != cudaSuccess)
      return VINFER_E_CUDA;
    if (cudaOccupancyMaxActiveBlocksPerMultiprocessor(&per_sm, kern, threads, smem) !=
        cudaSuccess)
      return VINFER_E_CUDA;
    k.ctas = std::max(1, sms * per_sm);
    k.ready = true;
  }
  *ctas = k.ctas;
  return VINFER_OK;
}

// resident CTAs of k_stream on the current device (at most CTA_CAP)
int sample_ctas(int dtype, int* ctas) {
  const void* kern = dtype == VINFER_DTYPE_BF16 ? (const void*)k_stream<__nv_bfloat16>
                                                : (const void*)k_stream<float>;
  if (kernel_info(kern, dtype == VINFER_DTYPE_BF16 ? 0 : 1, NT, sizeof(SSmem), ctas) != VINFER_OK)
    return VINFER_E_CUDA;
  *ctas = std::min(*ctas, CTA_CAP);
  return VINFER_OK;
}
// k_stream, then k_finish (mode 0: every row's answer; mode 1: this rank's shard records)
int launch_sample(const KParams& P, int dtype, cudaStream_t st) {
  const bool bf = dtype == VINFER_DTYPE_BF16;
  const void* fin = bf ? (const void*)k_finish<__nv_bfloat16> : (const void*)k_finish<float>;
  int unused = 0;
  if (kernel_info(fin, bf ? 4 : 5, NT, sizeof(Smem), &unused) != VINFER_OK) return VINFER_E_CUDA;
  if (bf) k_stream<__nv_bfloat16><<<P.grid, NT, sizeof(SSmem), st>>>(P);
  else k_stream<float><<<P.grid, NT, sizeof(SSmem), st>>>(P);
  if (cudaGetLastError() != cudaSuccess) return VINFER_E_CUDA;
  // programmatic dependent launch: k_finish starts on SMs as k_stream frees them and does its
  // input-only set-up before waiting for k_stream's records
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[0].val.programmaticStreamSerializationAllowed = 1;
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3((unsigned)P.B);
  cfg.blockDim = dim3(NT);
  cfg.dynamicSmemBytes = sizeof(Smem);
  cfg.stream = st;
  cfg.attrs = attr;
  cfg.numAttrs = 1;
  const cudaError_t e = bf ? cudaLaunchKernelEx(&cfg, k_finish<__nv_bfloat16>, P)
                           : cudaLaunchKernelEx(&cfg, k_finish<float>, P);
  return e == cudaSuccess ? VINFER_OK : VINFER_E_CUDA;
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
  NvtxRange nvtx_range("vinfer_sample");
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
  NvtxRange nvtx_range("vinfer_sample_local");
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
  NvtxRange nvtx_range("vinfer_sample_merge");
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
  if (kernel_info(kern, a->dtype == VINFER_DTYPE_BF16 ? 2 : 3, NT, sizeof(Smem), &ctas) !=
      VINFER_OK)
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

int vinfer_sample_top_logprobs(const VinferSampleArgs* a, int32_t n, int32_t* out_ids,
                               float* out_logprobs, void* workspace, size_t workspace_bytes,
                               void* stream) {
  NvtxRange nvtx_range("vinfer_sample_top_logprobs");
  int rc = check_args(a);
  if (rc != VINFER_OK) return rc;
  if (a->vocab_offset != 0 || a->vocab_total != a->vocab) return VINFER_E_ARG;
  if (!workspace || !out_ids || !out_logprobs || n < 1 || (int64_t)n >= a->vocab)
    return VINFER_E_ARG;
  if (n > VINFER_TOP_LOGPROBS_MAX) return VINFER_E_LIMIT;
  if (workspace_bytes < ws_layout(a->batch, a->vocab, a->dtype).total) return VINFER_E_LIMIT;
  int ctas = 0;
  if (sample_ctas(a->dtype, &ctas) != VINFER_OK) return VINFER_E_CUDA;
  const Shape s = plan(a->batch, a->vocab, a->dtype, ctas);
  KParams P = make_params(a, s, workspace);
  P.mode = 3;
  P.topn = n;
  P.top_ids = out_ids;
  P.top_lp = out_logprobs;
  return launch_sample(P, a->dtype, (cudaStream_t)stream);
}

int vinfer_sample_decode(const VinferSampleArgs* a, int32_t* hist_len, int32_t cap,
                         void* workspace, size_t workspace_bytes, void* stream) {
  NvtxRange nvtx_range("vinfer_sample_decode");
  int rc = check_args(a);
  if (rc != VINFER_OK) return rc;
  if (a->vocab_offset != 0 || a->vocab_total != a->vocab) return VINFER_E_ARG;
  if (!workspace || !hist_len || !a->hist_row_ptr || a->out_probs || cap < 1) return VINFER_E_ARG;
  if (cap > VINFER_HIST_MAX_CAP) return VINFER_E_LIMIT;
  if (workspace_bytes < ws_layout(a->batch, a->vocab, a->dtype).total) return VINFER_E_LIMIT;
  int ctas = 0;
  if (sample_ctas(a->dtype, &ctas) != VINFER_OK) return VINFER_E_CUDA;
  const Shape s = plan(a->batch, a->vocab, a->dtype, ctas);
  KParams P = make_params(a, s, workspace);
  P.mode = 0;
  P.slot_ids = const_cast<int*>(a->hist_ids);  // the caller's slotted arrays, updated in place
  P.slot_cnt = const_cast<int*>(a->hist_counts);
  P.hlen = hist_len;
  P.hcap = cap;
  return launch_sample(P, a->dtype, (cudaStream_t)stream);
}

int vinfer_sample_logprobs(const VinferSampleArgs* a, float* out_logprobs, void* workspace,
                           size_t workspace_bytes, void* stream) {
  NvtxRange nvtx_range("vinfer_sample_logprobs");
  int rc = check_args(a);
  if (rc != VINFER_OK) return rc;
  if (a->vocab_offset != 0 || a->vocab_total != a->vocab) return VINFER_E_ARG;
  if (!workspace || !out_logprobs) return VINFER_E_ARG;
  if (workspace_bytes < ws_layout(a->batch, a->vocab, a->dtype).total) return VINFER_E_LIMIT;
  const Shape s = plan(a->batch, a->vocab, a->dtype, 1);
  KParams P = make_params(a, s, workspace);
  const unsigned grid = (unsigned)((a->batch + 127) / 128);
  if (a->dtype == VINFER_DTYPE_BF16)
    k_logprobs<__nv_bfloat16><<<grid, 128, 0, (cudaStream_t)stream>>>(P, out_logprobs);
  else
    k_logprobs<float><<<grid, 128, 0, (cudaStream_t)stream>>>(P, out_logprobs);
  return cudaGetLastError() == cudaSuccess ? VINFER_OK : VINFER_E_CUDA;
}

int vinfer_hist_append(const int32_t* tokens, int64_t slots, int32_t* hist_ids,
                       int32_t* hist_counts, int32_t* hist_len, int32_t cap, int32_t* status,
                       void* stream) {
  NvtxRange nvtx_range("vinfer_hist_append");
  if (!tokens || !hist_ids || !hist_counts || !hist_len || slots < 1 || cap < 1)
    return VINFER_E_ARG;
  if (slots > VINFER_MAX_BATCH || cap > VINFER_HIST_MAX_CAP) return VINFER_E_LIMIT;
  // programmatic dependent launch: scheduled while the kernel before it finishes, it waits on
  // the device for that kernel's completion before it reads the ids
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[0].val.programmaticStreamSerializationAllowed = 1;
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3((unsigned)slots);
  cfg.blockDim = dim3(HIST_NT);
  cfg.stream = (cudaStream_t)stream;
  cfg.attrs = attr;
  cfg.numAttrs = 1;
  const cudaError_t e = cudaLaunchKernelEx(&cfg, k_hist_append, tokens, hist_ids, hist_counts,
                                           hist_len, cap, status);
  return e == cudaSuccess ? VINFER_OK : VINFER_E_CUDA;
}

int vinfer_hist_reset(const int32_t* slot_list, int64_t n, int64_t slots, int32_t* hist_ids,
                      int32_t* hist_counts, int32_t* hist_len, int32_t cap, void* stream) {
  NvtxRange nvtx_range("vinfer_hist_reset");
  if (!slot_list || !hist_ids || !hist_counts || !hist_len || n < 1 || slots < 1 || cap < 1)
    return VINFER_E_ARG;
  if (n > VINFER_MAX_BATCH || slots > VINFER_MAX_BATCH || cap > VINFER_HIST_MAX_CAP)
    return VINFER_E_LIMIT;
  k_hist_reset<<<(unsigned)n, HIST_NT, 0, (cudaStream_t)stream>>>(slot_list, slots, hist_ids,
                                                                 hist_counts, hist_len, cap);
  return cudaGetLastError() == cudaSuccess ? VINFER_OK : VINFER_E_CUDA;
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
// (with that device current, as cudaGetSymbolAddress requires). The address is kept for the life
// of the process: the library does not survive a cudaDeviceReset (or any other teardown of the
// device's primary context) in the same process.
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
  // The per-row arrival counters must start at zero; the array keeps whatever the previous call
  // left, so clear this call's counters.
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

/*
 * vinfer_sampler.h — C ABI of the B200 (sm_100a) token sampler.
 *
 * One fused, memory-bound pass per batch of logits rows: repetition / presence / frequency
 * penalties from per-row token-count histograms, temperature, top-k, softmax, top-p, min-p,
 * and an inverse-CDF draw from a caller-supplied uniform. A vocab-sharded mode reduces each
 * rank's shard to a fixed-size candidate record for an all-gather and a merge.
 *
 * Every pointer is caller-owned memory. Device pointers unless stated otherwise; no pointer
 * is retained after a call returns. Calls are stream-ordered on the given CUDA stream
 * (`void*` is a `cudaStream_t`; NULL is the legacy default stream). Functions return
 * VINFER_OK or a VINFER_E_* code and never throw; a device-side problem is reported by OR-ing
 * VINFER_ST_* bits into `*status` (a device int32, may be NULL) and writing -1 as the row's id.
 *
 * The entry points replace these reference interfaces (vinfer, pure PyTorch):
 *   vinfer_sample        <- `sample(logits, params, seed, position) -> int`
 *                           (src/vinfer/runtime/sampler.py:68-77, called per decode step at
 *                           src/vinfer/runtime/generate.py:129), batched over rows, and
 *                           `filtered_probs(logits, params)` (sampler.py:50-65) through
 *                           the optional `out_probs`.
 *   vinfer_sampler_workspace_bytes / _init
 *                        <- per-device workspaces a backend sets up when the engine builds it
 *                           (src/vinfer/kernels/registry.py:9-11, BackendRegistry.resolve
 *                           registry.py:84-88 constructs it once).
 *   vinfer_sample_local / vinfer_sample_merge
 *                        <- no counterpart: the reference has no distributed code. They are
 *                           the vocab-sharded form of `vinfer_sample` (logits split along the
 *                           vocab as a tensor-parallel lm_head produces them,
 *                           src/vinfer/models/qwen/model.py:230-233).
 */
#ifndef VINFER_SAMPLER_H
#define VINFER_SAMPLER_H

#include <stddef.h>
#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

#define VINFER_SAMPLER_ABI_VERSION 1

/* logits element types */
#define VINFER_DTYPE_F32 0
#define VINFER_DTYPE_BF16 1

/* return codes */
#define VINFER_OK 0
#define VINFER_E_ARG 1      /* a null pointer, a bad size, a dtype or stride out of range */
#define VINFER_E_LIMIT 2    /* a documented limit exceeded (vocab, batch, workspace too small) */
#define VINFER_E_CUDA 3     /* a CUDA runtime call failed (launch, attribute) */

/* bits OR-ed into *status by the device */
#define VINFER_ST_BAD_PARAM 1u   /* a row's parameters are invalid; its id is -1 */
#define VINFER_ST_NONFINITE 2u   /* a row has no finite maximum after processing */
#define VINFER_ST_HIST_FULL 4u   /* vinfer_hist_append: a slot had no room for a new token */
#define VINFER_ST_INTERNAL 8u    /* an internal consistency check failed */

/* args.flags */
#define VINFER_FLAG_EXACT_ALL 1u /* resolve every row with the exact multi-pass search */

/* limits */
#define VINFER_MAX_VOCAB 262144   /* per call (per shard in sharded mode) and in total */
#define VINFER_MAX_BATCH 65535

typedef struct VinferSampleArgs {
  const void* logits;          /* [batch, ld] row-major; the first `vocab` columns are used */
  int32_t dtype;               /* VINFER_DTYPE_F32 or VINFER_DTYPE_BF16 */
  uint32_t flags;              /* VINFER_FLAG_* */
  int64_t batch;               /* rows */
  int64_t vocab;               /* columns processed (the local shard in sharded mode) */
  int64_t ld;                  /* row stride, in elements (>= vocab) */
  int64_t vocab_offset;        /* global id of column 0 (0 unless sharded) */
  int64_t vocab_total;         /* global vocabulary size (== vocab unless sharded) */
  /* per-row parameters, device float32 / int32 [batch]; NULL selects the default */
  const float* temperature;    /* 0 = greedy; default 1 */
  const int32_t* top_k;        /* 0 = off; default 0 */
  const float* top_p;          /* (0, 1], 1 = off; default 1 */
  const float* min_p;          /* [0, 1], 0 = off; default 0 */
  const float* repetition_penalty; /* > 0, 1 = off; default 1 */
  const float* presence_penalty;   /* 0 = off; default 0 */
  const float* frequency_penalty;  /* 0 = off; default 0 */
  /* token-count histograms, CSR over rows, global token ids; NULL row_ptr = no histories */
  const int64_t* hist_row_ptr; /* [batch + 1] */
  const int32_t* hist_ids;     /* [nnz], strictly ascending within each row */
  const int32_t* hist_counts;  /* [nnz]; entries with count <= 0 are ignored */
  const float* uniforms;       /* [batch] in [0, 1); required unless every row is greedy */
  int32_t* out_ids;            /* [batch] sampled global token ids */
  float* out_probs;            /* optional [batch, vocab] final probabilities (parity checks) */
  int32_t* status;             /* optional, one device int32 */
} VinferSampleArgs;

/* ABI version of the loaded library (VINFER_SAMPLER_ABI_VERSION). */
int vinfer_sampler_abi_version(void);

/* Workspace bytes `vinfer_sample` needs for this shape (independent of the device). A workspace
 * of N bytes serves every shape whose size is at most N: it starts with a header whose place and
 * size do not depend on the shape (per-row arrival counters for VINFER_MAX_BATCH rows), which
 * every call leaves at zero. */
size_t vinfer_sampler_workspace_bytes(int64_t batch, int64_t vocab, int32_t dtype);

/* Zero a workspace once after allocating it; calls leave it ready for the next call, of any
 * shape that fits. */
int vinfer_sampler_workspace_init(void* workspace, size_t bytes, void* stream);

/* Sample one token per row. One workspace serves one call at a time. */
int vinfer_sample(const VinferSampleArgs* args, void* workspace, size_t workspace_bytes,
                  void* stream);

/* Log-probability of each row's sampled token under the row's final distribution (after
 * penalties, temperature, top-k / top-p / min-p and renormalisation): the `logprobs` that
 * src/vinfer/server/protocol.py:131-132 rejects today. Call after vinfer_sample with the same
 * args and workspace (it reads the row results that call left there), before the next call on
 * that workspace. out_logprobs: float [batch]; greedy rows get 0 (a one-hot distribution),
 * rows without a result (invalid parameters, no finite logit) NaN. Unsharded calls only. */
int vinfer_sample_logprobs(const VinferSampleArgs* args, float* out_logprobs, void* workspace,
                           size_t workspace_bytes, void* stream);

/* The n most likely tokens of each row's final distribution with their log-probabilities: the
 * `top_logprobs` that src/vinfer/server/protocol.py:131-132 rejects today. Call after
 * vinfer_sample with the same args and workspace, before the next call on that workspace; it
 * streams the logits once more (the n largest processed values, by the candidate path) and
 * prices each token with the row's result that call left: out_ids / out_logprobs are
 * [batch, n] in descending probability (ties by ascending id); a token outside the kept set
 * gets -inf, a slot with no token id -1; a greedy row lists its token with 0 (its distribution
 * is one-hot); a row without a result (invalid parameters) gets -1 and NaN, and a row whose top
 * list ties flood (more than 1,024 equal values) gets -1. 1 <= n <= VINFER_TOP_LOGPROBS_MAX,
 * n < vocab. Unsharded calls only. */
#define VINFER_TOP_LOGPROBS_MAX 32
int vinfer_sample_top_logprobs(const VinferSampleArgs* args, int32_t n, int32_t* out_ids,
                               float* out_logprobs, void* workspace, size_t workspace_bytes,
                               void* stream);

/* ---- vocab-sharded mode -------------------------------------------------------------------
 * Each rank calls vinfer_sample_local on its shard (vocab_offset / vocab_total set), which
 * writes one fixed-size candidate record per row into `records` (this rank's slice of the
 * all-gather buffer). After an all-gather of those buffers in rank order, every rank calls
 * vinfer_sample_merge on the gathered [world][batch] records with identical parameters and
 * uniforms, and gets identical ids. A row whose cut or draw falls outside the candidates is
 * marked in `unresolved` (id -1); the caller resolves it with vinfer_sample on the full row.
 */
size_t vinfer_sample_record_bytes(int32_t record_cap);  /* bytes of one row's record */
int vinfer_sample_local(const VinferSampleArgs* args, int32_t record_cap, void* records,
                        void* workspace, size_t workspace_bytes, void* stream);
int vinfer_sample_merge(const VinferSampleArgs* args, int32_t record_cap, const void* records,
                        int32_t world_size, int32_t* unresolved, void* workspace,
                        size_t workspace_bytes, void* stream);

/* ---- allocation-free variant ---------------------------------------------------------------
 * No counterpart in the reference: an addition of this library. Some callers cannot allocate
 * device memory when they sample: a serving engine that has handed nearly all of HBM to its
 * KV-cache pool at start-up (a cudaMalloc then fails, or waits for the device), or a host
 * that links only this C library and owns no device allocator (a Go, Java or C runtime).
 * vinfer_sample_static is vinfer_sample without the workspace argument: its scratch is a
 * fixed array of VINFER_STATIC_SCRATCH_BYTES compiled into the library, which every device
 * that loads the library holds until the process exits. It allocates nothing.
 *  - Limit: the call returns VINFER_E_LIMIT when vinfer_sampler_workspace_bytes(batch, vocab,
 *    dtype) exceeds VINFER_STATIC_SCRATCH_BYTES (at least 63 rows fit at any vocabulary).
 *  - The first call on a device looks up the array's device address on that device (which
 *    may load the library's device code); make it before any stream capture. The address is
 *    kept for the life of the process: the library does not survive a cudaDeviceReset (or any
 *    other teardown of the device's primary context) in the same process.
 *  - All calls on one device share the array: calls that can overlap on the GPU (different
 *    streams or host threads without ordering) race and corrupt each other's results.
 */
#define VINFER_STATIC_SCRATCH_BYTES (32u << 20)
int vinfer_sample_static(const VinferSampleArgs* args, void* stream);

/* ---- slotted histories for a batched decode loop ----------------------------------------------
 * Replaces the host-side loop of src/vinfer/runtime/generate.py:127-143 (one sample() per step,
 * an int() host sync per token, no token counts kept) for a batch of decode slots, each owned
 * by one request as in src/vinfer/state/pool.py:70-82 (alloc / free of per-request state).
 * Slot s owns entries [s * cap, (s + 1) * cap) of hist_ids / hist_counts (int32): its first
 * hist_len[s] entries are its tokens (ids strictly ascending, counts > 0); the others are
 * padding with count 0 and id VINFER_HIST_PAD_ID - (cap - 1 - position), ascending and above
 * every vocabulary id. With row_ptr[s] = s * cap (int64 [slots + 1]) the arrays are a CSR
 * history that vinfer_sample reads as it is (padding entries are outside every vocabulary),
 * so sample -> append -> sample never leaves the device.
 *  - vinfer_hist_append: for every slot s with tokens[s] >= 0, count tokens[s] once more in
 *    slot s, or insert it in id order. A full slot (hist_len[s] == cap) keeps its counts and
 *    sets VINFER_ST_HIST_FULL in *status (may be NULL). tokens is typically the previous
 *    vinfer_sample's out_ids (an invalid row's id -1 changes nothing).
 *  - vinfer_hist_reset: empty the n slots listed in slot_list (a request leaving its slot);
 *    entries outside [0, slots) are skipped.
 * Both are stream-ordered, one CTA per slot, and allocate nothing. cap <= VINFER_HIST_MAX_CAP.
 *  - vinfer_sample_decode: vinfer_sample and vinfer_hist_append in one call. args' history
 *    is the slotted arrays (row_ptr[s] = s * cap) and is updated in place with each row's
 *    sampled id by the finishing kernel, after every read of it for this step; no out_probs.
 *    A log-probability call (which prices tokens with the counts of the step) must instead
 *    use vinfer_sample, vinfer_sample_logprobs, then vinfer_hist_append.
 */
#define VINFER_HIST_PAD_ID 0x7FFFFFFF
#define VINFER_HIST_MAX_CAP (1 << 20)
int vinfer_hist_append(const int32_t* tokens, int64_t slots, int32_t* hist_ids,
                       int32_t* hist_counts, int32_t* hist_len, int32_t cap, int32_t* status,
                       void* stream);
int vinfer_hist_reset(const int32_t* slot_list, int64_t n, int64_t slots, int32_t* hist_ids,
                      int32_t* hist_counts, int32_t* hist_len, int32_t cap, void* stream);
int vinfer_sample_decode(const VinferSampleArgs* args, int32_t* hist_len, int32_t cap,
                         void* workspace, size_t workspace_bytes, void* stream);

#ifdef __cplusplus
}
#endif

#endif /* VINFER_SAMPLER_H */

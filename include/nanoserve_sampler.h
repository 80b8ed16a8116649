/*
 * nanoserve_sampler.h -- C ABI of the B200 (sm_100a) token-sampling op.
 *
 * This library replaces one Python method of NanoServe:
 *
 *   nanoserve/scheduler/sampler.py:21-89   Sampler.sample(logits,
 *       sampling_params_list, history_token_ids, generators=None)
 *
 * The reference runs a chain of ATen ops per row (repetition penalty
 * sampler.py:31-38, temperature sampler.py:40-51, top-k sampler.py:53-58,
 * top-p sampler.py:60-73, softmax + NaN guard sampler.py:75-80, greedy
 * argmax sampler.py:82-83, multinomial sampler.py:84-89).  Here the whole
 * chain is one kernel launch per call with one HBM pass per vocabulary row:
 * batches of 32 or more aligned rows take the row kernel (one block per SM
 * streams whole rows through a bulk-copy ring and finishes each row while
 * the next one streams); smaller batches take an 8-CTA thread-block cluster
 * per row that holds it in distributed shared memory.
 *
 * Everything in this header is plain C: raw pointers, sizes and a stream
 * handle.  All pointers named "device" must be CUDA device (or managed)
 * memory of the current device; nothing here allocates device memory.
 *
 * Per-row parameters are the reference's DERIVED quantities, so that the
 * host does the Python-double comparisons exactly as the reference does:
 *   temperature   = float32(max(t, 1e-6)) if t > 0 else 1.0   (sampler.py:41-46)
 *   NS_ROW_GREEDY = (t == 0.0)                                  (sampler.py:47-50)
 *   top_k         = k if 0 < k < vocab else 0 (0 = off)         (sampler.py:55)
 *   NS_ROW_TOP_P  = (top_p < 1.0); top_p = float32(top_p)       (sampler.py:63)
 *   NS_ROW_PENALTY= (rp != 1.0 and history non-empty);          (sampler.py:33)
 *                   repetition_penalty = float32(rp)
 */
#ifndef NANOSERVE_SAMPLER_H_
#define NANOSERVE_SAMPLER_H_

#include <stddef.h>
#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

#define NS_ABI_VERSION 3

/* status codes returned by every entry point */
#define NS_OK 0
#define NS_ERR_INVALID_ARG 1   /* bad pointer / shape / dtype / stride   */
#define NS_ERR_UNSUPPORTED 2   /* e.g. vocab too large for one cluster   */
#define NS_ERR_CUDA 3          /* a CUDA runtime call failed             */

/* logits element types */
#define NS_DTYPE_F32 0
#define NS_DTYPE_BF16 1

/* output token types */
#define NS_OUT_I64 0
#define NS_OUT_I32 1

/* NsSampleArgs.kernel: which kernel serves the call ("split": the row
 * kernel, which splits a batch's rows over persistent blocks, one per SM) */
#define NS_KERNEL_AUTO 0     /* the row kernel for batches of >= 32 aligned rows,
                                the cluster kernel otherwise              */
#define NS_KERNEL_CLUSTER 1  /* always the cluster kernel                 */
#define NS_KERNEL_SPLIT 2    /* the row kernel where its layout
                                conditions hold (aligned rows, vocabulary
                                in [24576, 196608]), else the cluster one */

/* NsRowParams.flags bits */
#define NS_ROW_GREEDY 0x1u   /* temperature == 0.0: argmax token          */
#define NS_ROW_TOP_P 0x2u    /* top_p < 1.0: nucleus filter on            */
#define NS_ROW_PENALTY 0x4u  /* repetition penalty on for this row        */
#define NS_ROW_SEED 0x8u     /* use NsRowParams.seed as this row's key    */

/* device-side status word bits (NsSampleArgs.status, optional) */
#define NS_STATUS_BAD_SAMPLE_INDEX 0x1u /* sample_indices[i] out of range */
#define NS_STATUS_BAD_HISTORY_ID 0x2u   /* history id outside [0, vocab)  */
#define NS_STATUS_WAIT_TIMEOUT 0x4u     /* a bounded wait gave up         */
#define NS_STATUS_CAP_OVERFLOW 0x8u     /* a top-p boundary fell among more
                                           members than the kernel ranks
                                           exactly (distinct logits within
                                           one fp32 mass value); the row
                                           kept them in index order       */
#define NS_STATUS_BAD_ROW_ORDER 0x10u   /* row_order[t] outside [0, S): that
                                           slot took row t instead        */
#define NS_STATUS_BAD_POOL_RANGE 0x20u  /* ns_history_gather / _append: a
                                           range or slot outside the pool */

/* One row's sampling parameters (32 bytes, device array [num_rows]).
 * Mirrors nanoserve/config.py:68-79 SamplingParams (temperature :72,
 * top_p :73, top_k :74, repetition_penalty :75, seed :79), pre-derived as
 * described at the top of this file. */
typedef struct NsRowParams {
  float temperature;        /* divisor applied to the logits             */
  float top_p;              /* nucleus mass, used when NS_ROW_TOP_P      */
  float repetition_penalty; /* used when NS_ROW_PENALTY                  */
  int32_t top_k;            /* 0 = off                                   */
  uint32_t flags;           /* NS_ROW_* bits                             */
  uint32_t seed_step;       /* NS_ROW_SEED: the request's own step index
                               (e.g. its token count), the Philox counter */
  uint64_t seed;            /* per-row Philox key when NS_ROW_SEED       */
} NsRowParams;

/* Arguments of one sampling step (replaces sampler.py:21-27's signature).
 *
 * Row i of the output samples logits row sample_indices[i] (or row i when
 * sample_indices is NULL).  Histories are CSR: row i's prior token ids are
 * history_ids[history_offsets[i] .. history_offsets[i+1]).
 *
 * Randomness: when uniforms is non-NULL, row i draws with the caller's
 * uniform uniforms[i] in [0,1); otherwise from Philox4x32-10: key
 * philox_seed and counter (philox_offset, row_offset + i), or, for a row
 * with NS_ROW_SEED, key row_params[i].seed and counter
 * (row_params[i].seed_step, 0), so that a seeded request draws the same
 * stream whatever batch or position it is sampled in.  The draw is an
 * inverse CDF over the filtered probabilities in vocabulary order.
 *
 * Debug outputs (NULL = not written), all [num_rows, vocab] fp32:
 *   out_penalized : the logits after the repetition penalty, i.e. what the
 *                   reference leaves in its mutated input (sampler.py:38)
 *   out_filtered  : scaled logits after top-k/top-p masking, -inf where
 *                   masked (the tensor softmaxed at sampler.py:76)
 *   out_probs     : the final probabilities (sampler.py:76-80)
 * The input logits are never modified. */
typedef struct NsSampleArgs {
  const void* logits;          /* device [num_logit_rows, row_stride]      */
  int32_t logits_dtype;        /* NS_DTYPE_*                               */
  int32_t vocab_size;          /* V                                        */
  int64_t num_logit_rows;      /* rows in logits                           */
  int64_t logits_row_stride;   /* elements between rows (>= V)             */
  int32_t num_rows;            /* S = rows to sample                       */
  int32_t out_dtype;           /* NS_OUT_*                                 */
  const int64_t* sample_indices;     /* device [S] or NULL                 */
  const NsRowParams* row_params;     /* device [S]                         */
  const int64_t* history_offsets;    /* device [S+1] or NULL (no history)  */
  const int32_t* history_ids;        /* device [history_offsets[S]]        */
  const float* uniforms;             /* device [S] or NULL                 */
  uint64_t philox_seed;
  uint64_t philox_offset;
  int64_t row_offset;                /* global index of row 0 (sharding)   */
  void* out_tokens;                  /* device [S], int64 or int32         */
  float* out_penalized;              /* device [S, V] or NULL              */
  float* out_filtered;               /* device [S, V] or NULL              */
  float* out_probs;                  /* device [S, V] or NULL              */
  uint32_t* status;                  /* device [1] or NULL: NS_STATUS_* bits
                                        OR-ed in by the kernel             */
  const int32_t* row_order;          /* device [S] or NULL: the order in
                                        which the kernel takes rows, a
                                        permutation of [0, S).  A scheduling
                                        hint only: outputs do not depend on
                                        it.  Taking the rows with the
                                        longest finishing work (top-p
                                        without top-k) first shortens mixed
                                        batches. */
  int32_t kernel;                    /* NS_KERNEL_* (0: automatic choice)   */
  int32_t reserved;                  /* must be 0                          */
  void* workspace;                   /* device scratch of workspace_bytes
                                        bytes (ns_workspace_bytes(): the row
                                        kernel's row-ticket counter), all
                                        zero before its first use; every
                                        call leaves it all zero again.  Calls
                                        that may overlap on the GPU need
                                        separate workspaces. */
  int64_t workspace_bytes;
} NsSampleArgs;

/* Enqueue one sampling step on `stream` (a cudaStream_t; NULL = legacy
 * default stream): one kernel launch.  Host-side checks only; no host
 * synchronisation, no allocation.  Calls that take the row kernel hand out
 * their rows through a counter in args->workspace (required for them:
 * NS_ERR_INVALID_ARG without one); cluster-kernel calls need none.
 * Replaces sampler.py:21-89 (Sampler.sample). */
int ns_sample(const NsSampleArgs* args, void* stream);

/* Bytes of NsSampleArgs.workspace for calls of up to num_rows rows (128:
 * the same for every call).  No counterpart in the reference. */
int64_t ns_workspace_bytes(int32_t num_rows);

/* Bytes of ns_sample_noalloc's static workspace. */
#define NS_NOALLOC_WORKSPACE_BYTES 128

/* ns_sample for callers that must not allocate device memory: an engine that
 * hands all of the GPU's memory to its own pool at start-up and makes no
 * cudaMalloc afterwards, or a host that embeds this library under a fixed
 * memory budget.  It allocates nothing on any call and ignores
 * args->workspace: its scratch is a file-scope static device array of the
 * library (NS_NOALLOC_WORKSPACE_BYTES bytes, the row kernel's row-ticket
 * counter), zero when the library loads, which every GPU that loads the
 * library holds until the process exits.  The array's size does not depend
 * on the call, so it limits no call; calls it cannot serve at all (a
 * vocabulary beyond ns_max_vocab) fail with NS_ERR_UNSUPPORTED and a
 * message, as ns_sample's do.  Every call looks up the array's device address
 * on the current device (cudaGetSymbolAddress, a host-side query); the first
 * one on a device may load the library's GPU code, so make it outside any
 * stream capture.  Every call shares the array and leaves it zero, as it
 * found it; calls that overlap on the GPU (different streams, or several host
 * threads at once) race on it.  Same arguments (but the workspace) and same
 * outputs as ns_sample.  No counterpart in the reference
 * (nanoserve/scheduler/sampler.py allocates through torch). */
int ns_sample_noalloc(const NsSampleArgs* args, void* stream);

/* Device-resident histories.  The reference rebuilds each request's prior
 * token ids as a Python list every step (nanoserve/engine.py:242-246, prompt
 * + output) and the sampler indexes with them (sampler.py:34).  These two
 * calls keep the ids in one append-only int32 device pool instead (a region
 * per request, laid out by the caller) and build a step's CSR histories
 * (NsSampleArgs.history_offsets / history_ids) on the device.  No
 * counterpart in the reference.  Both only enqueue one small kernel on
 * `stream`: no host synchronisation, no allocation.  `status` (device [1] or
 * NULL) gets NS_STATUS_BAD_POOL_RANGE OR-ed in for ranges outside the pool.
 *
 * ns_history_gather: for r < num_rows, out_ids[offsets[r] + j] =
 *   pool[row_src[r] + j] for j < offsets[r+1] - offsets[r].  A row whose
 *   source range leaves [0, pool_size) gets ids of -1 instead (ns_sample
 *   then reports NS_STATUS_BAD_HISTORY_ID).  row_src, offsets: device int64
 *   [num_rows] and [num_rows + 1]; out_ids: device int32 [offsets[num_rows]].
 * ns_history_append: pool[row_dst[r]] = tokens[r] for r < num_rows with
 *   row_dst[r] >= 0 (negative: skip the row).  tokens: device [num_rows],
 *   int64 or int32 as tokens_dtype (NS_OUT_I64 / NS_OUT_I32) says -- the
 *   out_tokens of an ns_sample call.  Destinations at or past pool_size are
 *   not written. */
int ns_history_gather(const int32_t* pool, int64_t pool_size, const int64_t* row_src, const int64_t* offsets,
                      int32_t num_rows, int32_t* out_ids, uint32_t* status, void* stream);
int ns_history_append(int32_t* pool, int64_t pool_size, const int64_t* row_dst, const void* tokens,
                      int32_t tokens_dtype, int32_t num_rows, uint32_t* status, void* stream);

/* Message for the last non-OK status returned on this host thread. */
const char* ns_last_error(void);

/* NS_ABI_VERSION of the loaded library. */
int ns_abi_version(void);

/* Largest vocabulary one cluster can hold for the given dtype. */
int32_t ns_max_vocab(int32_t logits_dtype);

#ifdef __cplusplus
}
#endif

#endif /* NANOSERVE_SAMPLER_H_ */

/*
 * flashgen_sampler.h — C ABI of the B200 (sm_100a) decode-step token sampler.
 *
 * This is the drop-in boundary for FlashGen's sampling path. Every entry point
 * takes plain device pointers and sizes; nothing here depends on torch or on
 * CUDA headers (streams are passed as `void*` holding a `cudaStream_t`).
 *
 * Reference interfaces replaced (paths inside the FlashGen project):
 *   - flashgen/sampling/sampler.py:57-88    Sampler.sample(logits[B,V], params) -> int64[B]
 *   - flashgen/sampling/sampler.py:102-121  Sampler._sample_one (B = 1 call of fg_sample)
 *   - flashgen/sampling/sampler.py:90-100   Sampler.sample_batch (shared params)
 *   - flashgen/sampling/sampler.py:123-147  Sampler.apply_repetition_penalty (in place)
 *   - csrc/runtime/pipeline.cpp:267-342     InferenceEngine::sample_tokens (host sampler
 *                                           after a full D2H copy; decl pipeline.hpp:125-127)
 *   - csrc/include/kernels.cuh:77-94        kernels::softmax_temperature / top_k_filter /
 *                                           top_p_filter / argmax (kernels.cu:244-306,422-446)
 *
 * Conventions
 *   - Ownership: the caller owns every buffer. No entry point allocates device
 *     memory, frees it, or synchronises the stream. All work is enqueued on
 *     `stream`; results are valid once the stream reaches that point.
 *   - Errors: return codes (FG_OK ...). Per-row problems (NaN rows, bad history
 *     ids, bad parameters) are reported through the optional `out_status` array
 *     and never abort the process, trap or assert on the device.
 *   - Threading: every entry point is re-entrant. Calls on different streams may
 *     run concurrently; the host does no work proportional to B*V.
 */
#ifndef FLASHGEN_SAMPLER_H_
#define FLASHGEN_SAMPLER_H_

#include <stddef.h>
#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

/* ---- return codes --------------------------------------------------------- */
#define FG_OK          0  /* work enqueued                                        */
#define FG_EINVAL      1  /* bad argument (null pointer, shape, dtype, alignment) */
#define FG_ELAUNCH     2  /* the CUDA launch failed (cudaGetLastError)            */
#define FG_ENOTSUP     3  /* shape valid but beyond this build's on-chip limits   */
#define FG_EDEVICE     4  /* querying or configuring the current device failed    */
#define FG_ESCRATCH    5  /* request exceeds fg_sample_noalloc's fixed scratch    */

/* ---- logits element types ------------------------------------------------- */
#define FG_DTYPE_F32   0
#define FG_DTYPE_F16   1
#define FG_DTYPE_BF16  2

/* ---- per-row status bits (out_status[row]) -------------------------------- */
#define FG_ROW_NAN          0x0001 /* row contains NaN (sampling rows: id = -1)    */
#define FG_ROW_POS_INF      0x0002 /* +inf logit in a sampling row (id = -1)        */
#define FG_ROW_ALL_MASKED   0x0004 /* every logit is -inf in a sampling row (-1)    */
#define FG_ROW_BAD_HISTORY  0x0008 /* a history id outside [0, vocab_total) was
                                      skipped; the id is still drawn             */
#define FG_ROW_BAD_PARAM    0x0010 /* temperature < 0, top_p outside (0,1], NaN (-1) */
#define FG_ROW_BAD_UNIFORM  0x0020 /* uniform outside [0,1) or NaN (id = -1)        */
#define FG_ROW_TIMEOUT      0x0040 /* an on-chip pipeline wait gave up (id = -1)    */
#define FG_ROW_CAND_TRUNC   0x0080 /* candidates mode: the top-k set (with ties) did
                                      not fit in cand_max                        */
#define FG_ROW_ERROR_MASK   0x00FF /* conditions under which FlashGen's sampler
                                      raises (torch indexing / multinomial)      */
/* informational bits (the id is valid) */
#define FG_ROW_GENERAL_PATH 0x0100 /* row was finished by the multi-pass path      */
#define FG_ROW_GREEDY       0x0200 /* row was decoded greedily                     */

/*
 * Arguments of one batched sampling call (a decode step).
 *
 * Logits: `batch` rows of `vocab` elements, row r at logits + r*row_stride
 * elements. The pointer must be aligned to the element size; rows need not be
 * 16-byte aligned.
 *
 * Per-row parameters are structure-of-arrays device vectors of length `batch`
 * (the fields of FlashGen's SamplingParams, flashgen/core/config.py:37-43 and
 * csrc/include/request.hpp:14-22, plus presence/frequency penalties).
 * Optional arrays may be NULL, meaning: repetition 1, presence 0, frequency 0,
 * greedy false.
 *
 * Chain per row, in order: repetition penalty on the unique history ids
 * (x > 0 ? x / rep : x * rep), then presence and frequency
 * (x - freq * count - presence), then — unless the row is greedy
 * (greedy != 0 or temperature == 0), which takes the first argmax —
 * temperature (x / T when T != 1), top-k (keep every logit >= the k-th
 * largest; k <= 0 disables), top-p (keep the descending prefix whose exclusive
 * mass is <= top_p, ties at the cut in ascending id order; top_p >= 1
 * disables), softmax, and an inverse-CDF draw over the kept set walked in
 * descending-probability order (ties in ascending id order), the order of
 * csrc/runtime/pipeline.cpp:311-340: the first token whose inclusive mass
 * exceeds u * total.
 *
 * Histories: CSR token lists. Row r's ids are hist_ids[hist_offsets[r] ..
 * hist_offsets[r+1]). Ids are global vocabulary ids in [0, vocab_total);
 * repeats are allowed (they are the frequency counts). Both pointers NULL
 * means no history. `hist_max_len` must bound every row's history length (it
 * sizes the on-chip history tables; at most 65535 unique ids per row).
 *
 * Vocabulary sharding: `vocab_offset` is the global id of column 0 and
 * `vocab_total` the full vocabulary size (0 means vocab_total = vocab). Output
 * ids are global (column + vocab_offset).
 */
typedef struct FgSampleArgs {
    const void*    logits;
    int32_t        dtype;               /* FG_DTYPE_*                              */
    int32_t        batch;               /* B >= 0                                  */
    int32_t        vocab;               /* V >= 1 columns in this call             */
    int32_t        hist_max_len;        /* >= every row's history length           */
    int64_t        row_stride;          /* elements between rows, >= vocab         */
    int64_t        vocab_offset;        /* global id of column 0                   */
    int64_t        vocab_total;         /* global vocabulary size (0 = vocab)      */
    const int32_t* hist_ids;            /* CSR ids (device) or NULL                */
    const int64_t* hist_offsets;        /* [B+1] (device) or NULL                  */
    const float*   temperature;         /* [B]                                     */
    const float*   top_p;               /* [B]                                     */
    const int32_t* top_k;               /* [B]                                     */
    const float*   repetition_penalty;  /* [B] or NULL                             */
    const float*   presence_penalty;    /* [B] or NULL                             */
    const float*   frequency_penalty;   /* [B] or NULL                             */
    const uint8_t* greedy;              /* [B] or NULL                             */
    const float*   uniforms;            /* [B] in [0,1)                            */
    int64_t*       out_ids;             /* [B]                                     */
    int32_t*       out_status;          /* [B] or NULL                             */
    float*         out_probs;           /* [B, vocab] kept-set probabilities, 0
                                           elsewhere (debug/oracle mode) or NULL   */
    void*          workspace;           /* device scratch, zero before the first
                                           call (see below)                         */
    size_t         workspace_bytes;     /* size of `workspace` in bytes            */
} FgSampleArgs;

/*
 * Workspace: rows are handed to the GPU's persistent CTAs through counters in
 * the first FG_SAMPLE_WORKSPACE_MIN_BYTES of this device buffer. The caller
 * zeroes the buffer once (cudaMemset) before its first use; every fg_sample
 * call leaves the counters zero again. Bytes beyond the counters hold, for
 * large batches, a block per row written and read within the call (history
 * lists and candidate sets of the batch kernels): that path runs only when
 * workspace_bytes covers fg_sample_workspace_size(batch, vocab, dtype,
 * hist_max_len), so a smaller buffer is always safe and only gives up that
 * path. workspace_bytes below FG_SAMPLE_WORKSPACE_MIN_BYTES returns
 * FG_EINVAL. Calls that may run concurrently on the GPU (different streams)
 * need separate workspaces.
 */
#define FG_SAMPLE_WORKSPACE_MIN_BYTES 256

/*
 * Batched fused sampling (one decode step). Replaces Sampler.sample
 * (flashgen/sampling/sampler.py:57-88), Sampler._sample_one (:102-121) and
 * InferenceEngine::sample_tokens (csrc/runtime/pipeline.cpp:267-342).
 * `stream` is a cudaStream_t (NULL = legacy default stream).
 */
int fg_sample(const FgSampleArgs* args, void* stream);

/*
 * Bytes of workspace with which fg_sample takes its fastest path for a batch
 * of this shape: the batch kernels keep a block per row (the row's history
 * list and candidates) after the counters. hist_max_len as in FgSampleArgs
 * (0 without history). A smaller workspace (at least
 * FG_SAMPLE_WORKSPACE_MIN_BYTES) is still valid: fg_sample then samples
 * every row with the cluster kernel, which needs only the counters.
 * 0 for an invalid shape or dtype. Host-only; no device call.
 * No reference counterpart (FlashGen's sampler allocates on the host).
 */
size_t fg_sample_workspace_size(int32_t batch, int32_t vocab, int32_t dtype, int32_t hist_max_len);

/*
 * Local stage of vocabulary-sharded sampling (tensor-parallel LM heads).
 * `args` describes one shard: columns [vocab_offset, vocab_offset + vocab) of
 * a vocabulary of vocab_total ids; history ids are global and only the
 * shard's own columns are penalised. Instead of drawing, each row writes its
 * top-k set after penalties and temperature: every element whose value y
 * (= penalised logit / T) is at least the shard's k-th largest, ties
 * included, as vals[r*cand_max + i] = y and gids[...] = global id, i <
 * counts[r]; unused slots hold -inf / INT32_MAX. Greedy rows write their
 * first maximum (y = penalised logit). Rows with top-k off get
 * FG_ROW_BAD_PARAM (the full distribution would be needed); a top-k set
 * larger than cand_max gets FG_ROW_CAND_TRUNC. out_ids is written with the
 * greedy id or -1. The owner of a row merges the shards' sets — top-k of the
 * union equals the global top-k — and draws with fg_sample on them
 * (flashgen_b200.sampling.sharded). Replaces the top-k half of
 * Sampler._sample_one (flashgen/sampling/sampler.py:110-117) on a shard.
 */
int fg_sample_candidates(const FgSampleArgs* args, float* vals, int32_t* gids,
                         int32_t* counts, int32_t cand_max, void* stream);

/*
 * Small-batch mode of fg_sample (no reference counterpart; FlashGen samples
 * one row per call on the CPU). A batch of a few rows would leave most SMs
 * idle with one CTA per row, so fg_sample samples it with the cluster kernel
 * instead: one thread-block cluster of G CTAs (G <= 16) per row, each CTA
 * keeping a slice of the row's keys in shared memory, the decisions reduced
 * across the cluster through distributed shared memory. Same kept set, draw
 * order and integer masses as the batch path. mode 0 never takes it for a
 * whole batch, 1 (default) takes it when B * G <= SMs with G >= 4, 2 takes it
 * for every batch (tests). Calls that want kept-set probabilities (out_probs)
 * and rows the batch path hands on always use the cluster kernel.
 * Process-wide (an atomic, read once per call); returns FG_EINVAL for other
 * modes.
 */
int fg_sample_set_split(int mode);

/*
 * fg_sample without a caller workspace: args->workspace must be NULL, and the
 * row-queue counters live in a 256-byte static device array (one per device).
 * No reference counterpart: FlashGen has no native sampler entry point; this
 * one serves callers that cannot allocate device memory on the decode path
 * (an engine loop that must not allocate, a plain-FFI host with no device
 * allocator). The first call on a device looks up and clears the array on
 * `stream` — make it before any stream capture. Calls that overlap on the GPU
 * race on the array: serialise them. batch above 2^30 returns FG_ESCRATCH.
 */
int fg_sample_noalloc(const FgSampleArgs* args, void* stream);

/*
 * In-place repetition penalty on a [batch, vocab] logits buffer: for every
 * row, each unique history id's logit x becomes x / penalty if x > 0 else
 * x * penalty (computed in fp32, stored back in the buffer's dtype).
 * penalty == NULL or penalty[r] == 1 leaves the row unchanged.
 * Replaces Sampler.apply_repetition_penalty (flashgen/sampling/sampler.py:123-147).
 */
int fg_apply_repetition_penalty(void* logits, int32_t dtype, int32_t batch,
                                int32_t vocab, int64_t row_stride,
                                const int32_t* hist_ids,
                                const int64_t* hist_offsets,
                                const float* penalty, void* stream);

/*
 * Row-wise argmax (first index of the maximum; NaN counts as the maximum, as
 * in torch.argmax). Replaces kernels::argmax (csrc/include/kernels.cuh:92-94,
 * csrc/kernels/kernels.cu:279-306,442-446) and the all-greedy fast path of
 * Sampler.sample (flashgen/sampling/sampler.py:74-75).
 */
int fg_argmax(const void* logits, int32_t dtype, int32_t batch, int32_t vocab,
              int64_t row_stride, int64_t* out_ids, void* stream);

/* Human-readable name of a return code. */
const char* fg_strerror(int code);

/* ABI version: major * 10000 + minor * 100 + patch. */
int fg_version(void);

#ifdef __cplusplus
}
#endif
#endif /* FLASHGEN_SAMPLER_H_ */

/*
 * navsampler — sm_100a decode-time logits processing and token sampling.
 *
 * C ABI of the library (libnavsampler.so). Plain pointers and sizes only; the
 * conventions follow the reference's native library Neuraval.Cuda.Native:
 *   - exported symbols are `extern "C"` with default visibility
 *     (Neuraval.Cuda.Native/src/navcuda.cu:9-13);
 *   - status codes 0..7 keep NcbStatus's values (navcuda.cu:19-29), each entry
 *     point returns its status AND records it for ncb_sampler_last_status()
 *     (the g_lastStatus model, navcuda.cu:31-39, read by CudaDevice.ThrowIfError,
 *     Neuraval.Cuda/CudaDevice.cs:70-91);
 *   - `_device` entry points take device pointers and are asynchronous on the
 *     given stream; host-array entry points copy in, launch, synchronise and
 *     copy out (the navcuda.cu:702-734 pattern, without per-call allocation).
 *
 * Each sampling entry point replaces, for a [rows, vocab] fp32 batch, one call
 * per row of TokenSampler.SampleNext (Neuraval/Generation/TokenSampler.cs:10);
 * the LogitsProcessor entry points replace LogitsProcessor.* per row
 * (Neuraval/Generation/LogitsProcessor.cs:8-114). There is no CPU fallback.
 *
 * A sibling library of navcuda by design: the sampler keeps its own last
 * status (ncb_sampler_last_status, not navcuda's ncb_cuda_last_status), so a
 * C# caller checks it through its own ThrowIfError twin rather than through
 * CudaDevice.ThrowIfError; the symbol names (ncb_sampler_*, ncb_sample_*,
 * ncb_logits_*, ncb_vocab_shard_*, ncb_row_gather_*) do not collide with
 * navcuda's, so the two can also be linked into one shared object.
 */
#ifndef NAVSAMPLER_H
#define NAVSAMPLER_H

#include <stddef.h>
#include <stdint.h>

#if defined(_WIN32)
#define NCB_API __declspec(dllexport)
#else
#define NCB_API __attribute__((visibility("default")))
#endif

#ifdef __cplusplus
extern "C" {
#endif

/* ---- status codes --------------------------------------------------------
 * 0..7 are NcbStatus (navcuda.cu:19-29). 8 is new: a size beyond what the
 * handle was created for. */
#define NCB_OK 0
#define NCB_ERROR_NO_DEVICE 1
#define NCB_ERROR_INIT_FAILED 2
#define NCB_ERROR_ALLOC_FAILED 3
#define NCB_ERROR_COPY_FAILED 4
#define NCB_ERROR_LAUNCH_FAILED 5
#define NCB_ERROR_NOT_INITIALIZED 6
#define NCB_ERROR_INVALID_ARGUMENT 7
#define NCB_ERROR_CAPACITY 8

/* ---- per-row result flags (uint32 per row) -------------------------------
 * Parity contract: a row's token equals the reference's unless one of the
 * first three bits is set. */
#define NCB_FLAG_DRAW_BOUNDARY 0x1u   /* u*retained within 1e-6*retained of S_j or S_{j-1} */
#define NCB_FLAG_CUTOFF_BOUNDARY 0x2u /* top-p test S_i >= total*topP within 1e-6 relative */
#define NCB_FLAG_TIE_AT_DRAW 0x4u     /* drawn position in a group of equal values: the C#
                                         unstable sort (TokenSampler.cs:95) picks the id */
#define NCB_FLAG_NONFINITE 0x8u       /* NaN/+inf value or no finite maximum: token -1 */
/* API change from the reference, deliberate: for a row holding a NaN or +inf
 * value (after the penalties and 1/T), or no finite value at all, the C#
 * TokenSampler still returns an id, decided by how NaN compares inside its
 * heap and sort and by the NaN weights that exp(inf - inf) produces
 * (TokenSampler.cs:69-134); no test of the reference pins that id. This
 * library returns -1 with NCB_FLAG_NONFINITE for the row instead and samples
 * every other row normally, so the caller decides (the C# host class in the
 * integration notes throws, which ends a generation loop that would have run
 * on with an arbitrary id). Greedy rows are not affected: SampleGreedy's
 * first strict maximum is well defined with NaN and inf and is reproduced. */
#define NCB_FLAG_EXP_SLOW 0x10u       /* a weight needed the double-double exp path */
#define NCB_FLAG_BAD_HISTORY 0x20u    /* frequency counting over a history longer than the handle's max: token -1 */
#define NCB_FLAG_TIES_OVERFLOW 0x40u  /* ncb_sample_rows_noalloc_device and vocabulary-shard
                                         merges only: ties at the k-th value exceed the
                                         candidate buffers: token -1 */

/* ---- sampling options ----------------------------------------------------
 * Mirrors GenerationOptions (Neuraval/Generation/GenerationOptions.cs:5-19):
 * Greedy, Temperature, TopP, TopK, RepetitionPenalty. "No top-k" is any
 * top_k >= vocab (GenerationOptions.CreateGreedy uses int.MaxValue, :79).
 * frequency_penalty / presence_penalty are new (no reference counterpart):
 * v - count*frequency - [count>0]*presence, after the repetition penalty and
 * before the temperature scale; 0 disables them. */
typedef struct NcbSamplerParams {
    int32_t greedy;
    float temperature;
    float top_p;
    int32_t top_k;
    float repetition_penalty;
    float frequency_penalty;
    float presence_penalty;
} NcbSamplerParams;

typedef struct NcbSampler NcbSampler; /* opaque; owns device scratch only */

/* GenerationOptions.Create's validation (GenerationOptions.cs:56-72): returns
 * NCB_ERROR_INVALID_ARGUMENT for T<=0, top_p outside (0,1], top_k<=0,
 * repetition_penalty<=0 or a NaN penalty. Host only; needs no device. */
NCB_API int ncb_sampler_params_validate(const NcbSamplerParams* params);

/* Creates a sampler bound to `device` with scratch for up to max_rows rows of
 * up to max_vocab columns and histories of up to max_history ids per row.
 * Replaces the per-call state of the C# sampler (HashSet, PriorityQueue,
 * candidate list; TokenSampler.cs:61-95). The handle is single-stream: calls
 * on one handle are serialised by a per-handle lock. */
NCB_API int ncb_sampler_create(int device, int max_rows, int max_vocab, int max_history,
                               NcbSampler** out);
NCB_API int ncb_sampler_destroy(NcbSampler* sampler);

/* TokenSampler.SampleNext (TokenSampler.cs:10-30) for `rows` rows at once.
 *   d_logits      [rows, vocab] fp32, row-major, read only
 *   d_hist        generated ids of all rows, concatenated (any int32 value;
 *                 ids outside [0,vocab) never match, as with the C# HashSet)
 *   d_hist_offsets rows+1 int32 offsets into d_hist (CSR)
 *   d_uniforms    rows fp32 u in [0,1): the reference's (float)random.NextDouble()
 *                 (TokenSampler.cs:125); unread when params->greedy
 *   d_tokens      rows int32 out
 *   d_flags       rows uint32 out (NCB_FLAG_*), may be NULL
 *   d_probs       optional [rows, vocab] fp32 out: w_i/retained for the retained
 *                 candidates, 0 elsewhere (unused when greedy), may be NULL
 *   stream        cudaStream_t (NULL = legacy default stream)
 * Asynchronous; arguments are validated on the host before any launch. */
NCB_API int ncb_sample_rows_device(NcbSampler* sampler, const float* d_logits, int rows,
                                   int vocab, const int32_t* d_hist,
                                   const int32_t* d_hist_offsets, const float* d_uniforms,
                                   const NcbSamplerParams* params, int32_t* d_tokens,
                                   uint32_t* d_flags, float* d_probs, void* stream);

/* Same with host arrays: copies in, samples, synchronises, copies out. This is
 * the drop-in for TokenSampler.SampleNext(float[] logits, ...) with rows=1. */
NCB_API int ncb_sample_rows(NcbSampler* sampler, const float* h_logits, int rows, int vocab,
                            const int32_t* h_hist, const int32_t* h_hist_offsets,
                            const float* h_uniforms, const NcbSamplerParams* params,
                            int32_t* h_tokens, uint32_t* h_flags, float* h_probs);

/* Allocation-free variant of ncb_sample_rows_device, with no counterpart in the
 * reference. For callers that cannot allocate device memory when they sample:
 * a serving process whose device memory is all owned by its own pool or by
 * another allocator, or a latency-critical loop that cannot afford the device
 * synchronisation cudaMalloc implies. It needs no handle and allocates nothing:
 * its scratch (candidate lists of rows split across CTAs, per-row tickets and
 * marks) is one file-scope device array of 8 MiB, present on every GPU that
 * loads the library until the process exits.
 *   - Runs on the current device. The first call on a device looks up that
 *     array's device address (cudaGetSymbolAddress) and raises the kernels'
 *     shared-memory limits; make that first call before any stream capture.
 *   - Serves greedy rows and top-k <= 64 with top_k < vocab only (top_k >=
 *     vocab means "no top-k", the full-vocabulary nucleus, whose scratch
 *     grows with rows x vocab); other options return NCB_ERROR_CAPACITY, as
 *     do rows > 1024 and vocab > 2^24. A row whose
 *     frequency counting needs more than 4096 history ids comes back as
 *     token -1 with NCB_FLAG_BAD_HISTORY.
 *   - Every call reuses the same array (the parts that must start at zero are
 *     cleared on `stream` at the start of each call): calls that overlap on the
 *     GPU, from any stream or thread, race and corrupt each other's results.
 *   - Rows whose ties at the k-th value overflow the candidate buffers, which
 *     the handle-based entry point resolves with its large full-vocabulary
 *     scratch, come back as token -1 with NCB_FLAG_TIES_OVERFLOW.
 * Arguments, outputs and errors are otherwise those of ncb_sample_rows_device. */
NCB_API int ncb_sample_rows_noalloc_device(const float* d_logits, int rows, int vocab,
                                           const int32_t* d_hist, const int32_t* d_hist_offsets,
                                           const float* d_uniforms,
                                           const NcbSamplerParams* params, int32_t* d_tokens,
                                           uint32_t* d_flags, float* d_probs, void* stream);

/* The same five operations on host arrays, in place (LogitsProcessor.* take a
 * float[]): rows are copied in through the handle's staging buffers, processed
 * and copied back before returning. Histories are host CSR arrays. */
NCB_API int ncb_logits_repetition_penalty(NcbSampler* sampler, float* h_logits, int rows,
                                          int vocab, const int32_t* h_hist,
                                          const int32_t* h_hist_offsets, float penalty);
NCB_API int ncb_logits_frequency_presence_penalty(NcbSampler* sampler, float* h_logits, int rows,
                                                  int vocab, const int32_t* h_hist,
                                                  const int32_t* h_hist_offsets, float frequency,
                                                  float presence);
NCB_API int ncb_logits_temperature(NcbSampler* sampler, float* h_logits, int rows, int vocab,
                                   float temperature);
NCB_API int ncb_logits_filter_top_k(NcbSampler* sampler, float* h_logits, int rows, int vocab,
                                    int top_k);
NCB_API int ncb_logits_filter_top_p(NcbSampler* sampler, float* h_probs, int rows, int vocab,
                                    float top_p, uint32_t* h_flags);

/* ---- vocabulary shards -----------------------------------------------------
 * No counterpart in the reference (it samples on one CPU thread): a batch whose
 * vocabulary is split in contiguous column ranges over several GPUs (a
 * tensor-parallel LM head leaves each GPU its columns of the logits). Each GPU
 * reduces its columns of every row to one record of
 * ncb_vocab_shard_record_bytes() bytes; the caller gathers the records of all
 * shards on every GPU, in column order, as [shards][rows] records (one NCCL
 * all-gather); each GPU then merges them into the tokens that
 * ncb_sample_rows_device gives for the whole rows (TokenSampler.cs:10-143).
 * Served: greedy rows and top-k <= 64 (other options: NCB_ERROR_CAPACITY).
 * A row whose ties at the global k-th value were cut from a shard's record
 * (more than 128 - (k-1) equal values) comes back as token -1 with
 * NCB_FLAG_TIES_OVERFLOW. */
NCB_API int ncb_vocab_shard_record_bytes(void);

/* d_logits: [rows, ld] fp32 holding columns [col_begin, col_end) of the full
 * vocabulary `vocab` (ld >= col_end - col_begin); histories hold full-vocabulary
 * ids. Writes rows records to d_records. col_end - col_begin <= the handle's
 * max_vocab; rows <= its max_rows. Asynchronous on `stream`. */
NCB_API int ncb_vocab_shard_candidates_device(NcbSampler* sampler, const float* d_logits,
                                              int rows, int vocab, int col_begin, int col_end,
                                              int ld, const int32_t* d_hist,
                                              const int32_t* d_hist_offsets,
                                              const NcbSamplerParams* params, void* d_records,
                                              void* stream);

/* d_records: [shards][rows] records, shard s holding the s-th column range.
 * shards <= 16. Outputs as ncb_sample_rows_device (no probabilities). */
NCB_API int ncb_vocab_shard_merge_device(NcbSampler* sampler, const void* d_records, int shards,
                                         int rows, int vocab, const float* d_uniforms,
                                         const NcbSamplerParams* params, int32_t* d_tokens,
                                         uint32_t* d_flags, void* stream);

/* ---- LogitsProcessor, batched, in place on device [rows, vocab] ----------- */

/* LogitsProcessor.ApplyRepetitionPenalty (LogitsProcessor.cs:8-36), per row
 * with that row's CSR history. penalty<=0 -> NCB_ERROR_INVALID_ARGUMENT. */
NCB_API int ncb_logits_repetition_penalty_device(NcbSampler* sampler, float* d_logits,
                                                 int rows, int vocab, const int32_t* d_hist,
                                                 const int32_t* d_hist_offsets,
                                                 float penalty, void* stream);
/* New (no reference counterpart): v - count*frequency - [count>0]*presence. */
NCB_API int ncb_logits_frequency_presence_penalty_device(NcbSampler* sampler, float* d_logits,
                                                         int rows, int vocab,
                                                         const int32_t* d_hist,
                                                         const int32_t* d_hist_offsets,
                                                         float frequency, float presence,
                                                         void* stream);
/* LogitsProcessor.ApplyTemperature (LogitsProcessor.cs:38-51): divides by T. */
NCB_API int ncb_logits_temperature_device(NcbSampler* sampler, float* d_logits, int rows,
                                          int vocab, float temperature, void* stream);
/* LogitsProcessor.FilterTopK (LogitsProcessor.cs:53-73): values below the
 * top_k-th largest (with multiplicity) become -inf; no-op when top_k>=vocab. */
NCB_API int ncb_logits_filter_top_k_device(NcbSampler* sampler, float* d_logits, int rows,
                                           int vocab, int top_k, void* stream);
/* LogitsProcessor.FilterTopP (LogitsProcessor.cs:75-114) on probabilities:
 * keeps the smallest descending prefix whose sequential fp32 sum reaches top_p
 * and renormalises it; d_flags (optional, rows) gets NCB_FLAG_TIE_AT_DRAW when
 * the cutoff splits a group of equal probabilities. */
NCB_API int ncb_logits_filter_top_p_device(NcbSampler* sampler, float* d_probs, int rows,
                                           int vocab, float top_p, uint32_t* d_flags,
                                           void* stream);

/* The same exchange done by the library through peer memory, without a
 * collective (no reference counterpart). Each GPU's handle owns one exchange
 * area: ncb_vocab_shard_peer_setup allocates it and writes its CUDA IPC handle
 * with what the area is laid out for (ncb_peer_handle_bytes() bytes); the
 * caller gives every handle all handles in shard order
 * (ncb_vocab_shard_peer_connect; handles exported by the same process resolve
 * without IPC). Connect returns NCB_ERROR_INVALID_ARGUMENT unless every handle
 * was set up for the same shard count and the same max_rows. Per call, on
 * every GPU in the same order: ncb_vocab_shard_push_peer_device (the shard
 * kernel; each finished record is stored, every word tagged with the call's
 * epoch, into every GPU's area over NVLink) and
 * ncb_vocab_shard_merge_peer_device (waits until every shard's words of the
 * row carry the epoch, then merges). Every wait is bounded (about 2 s); a row
 * whose words do not all arrive returns token -1 with NCB_FLAG_PEER_TIMEOUT.
 * rows <= the handle's max_rows; all GPUs pass the same rows, vocab and
 * params. */
#define NCB_FLAG_PEER_TIMEOUT 0x80u
NCB_API int ncb_peer_handle_bytes(void);
NCB_API int ncb_vocab_shard_peer_setup(NcbSampler* sampler, int shards, int me, void* handle_out);
NCB_API int ncb_vocab_shard_peer_connect(NcbSampler* sampler, const void* handles);
NCB_API int ncb_vocab_shard_push_peer_device(NcbSampler* sampler, const float* d_logits, int rows,
                                             int vocab, int col_begin, int col_end, int ld,
                                             const int32_t* d_hist,
                                             const int32_t* d_hist_offsets,
                                             const NcbSamplerParams* params, void* stream);
NCB_API int ncb_vocab_shard_merge_peer_device(NcbSampler* sampler, int rows, int vocab,
                                              const float* d_uniforms,
                                              const NcbSamplerParams* params, int32_t* d_tokens,
                                              uint32_t* d_flags, void* stream);

/* ---- rows split over GPUs --------------------------------------------------
 * No reference counterpart (the reference samples one row per call on one CPU
 * thread). A batch split by rows over `ranks` GPUs, one process per GPU: each
 * GPU samples its own rows, and every GPU gets every row's token and flags,
 * gathered through peer memory instead of a collective. Each GPU's handle owns
 * one gather area: ncb_row_gather_setup allocates it for rows_total rows and
 * writes its CUDA IPC handle (ncb_peer_handle_bytes() bytes); the caller gives
 * every handle all handles in rank order (ncb_row_gather_connect, which returns
 * NCB_ERROR_INVALID_ARGUMENT unless every handle was set up for the same ranks
 * and rows_total). Per call,
 * on every GPU in the same order: ncb_sample_rows_gather_device samples this
 * GPU's rows [row_begin, row_begin + rows) (arguments as ncb_sample_rows_device,
 * rows <= max_rows; the GPUs' ranges together cover [0, rows_total) once),
 * stores their tokens and flags, tagged with the call's epoch, into every GPU's
 * area over NVLink, waits (bounded, about 2 s) until every row of its own area
 * carries the epoch and writes all rows_total tokens (and flags, may be NULL)
 * to d_tokens_all / d_flags_all. A row still missing when the wait gives up
 * (a peer that stopped, or a range no GPU covered) comes back as -1 with
 * NCB_FLAG_PEER_TIMEOUT. Asynchronous on `stream`. */
NCB_API int ncb_row_gather_setup(NcbSampler* sampler, int ranks, int me, int rows_total,
                                 void* handle_out);
NCB_API int ncb_row_gather_connect(NcbSampler* sampler, const void* handles);
NCB_API int ncb_sample_rows_gather_device(NcbSampler* sampler, const float* d_logits, int rows,
                                          int vocab, int row_begin, const int32_t* d_hist,
                                          const int32_t* d_hist_offsets,
                                          const float* d_uniforms,
                                          const NcbSamplerParams* params,
                                          int32_t* d_tokens_all, uint32_t* d_flags_all,
                                          void* stream);

/* ---- row softmax ----------------------------------------------------------
 * ncb_cuda_softmax_rows_device (Neuraval.Cuda.Native/src/navcuda.cu:673-700)
 * with the arithmetic of its kernel (:616-671), output bits equal: row max,
 * e = expf(x - max), 256 strided partial sums in element order and their
 * tree, e / sum. d_out may equal d_in. rows <= 0 or cols <= 0 ->
 * NCB_ERROR_INVALID_ARGUMENT (as the reference). Needs no handle;
 * asynchronous on `stream`. */
NCB_API int ncb_softmax_rows_device(const float* d_in, float* d_out, int rows, int cols,
                                    void* stream);

/* ---- diagnostics ----------------------------------------------------------
 * Rows this handle has redone on the exact full-sort kernel since it was
 * created: top-k rows whose ties overflowed the candidate buffers, and
 * full-vocabulary rows the bucketed kernel handed over (a running-sum
 * estimate outside its margin, a very large bucket of equal-looking values).
 * Synchronises the device. */
NCB_API int ncb_sampler_full_sort_rows(NcbSampler* sampler, uint64_t* out_rows);

/* Largest distance, in float steps, between the fast exponential the bucketed
 * kernel estimates with and the correctly rounded exp over every float x in
 * [x_lo, x_hi] (x_lo <= x_hi <= 0). The kernel relies on at most 21 steps on
 * [-17, 0]. Synchronous; runs on the current device. */
NCB_API int ncb_fast_exp_max_steps(float x_lo, float x_hi, uint32_t* out_steps);

/* ---- status --------------------------------------------------------------- */
/* ncb_cuda_last_status / ncb_cuda_status_message (navcuda.cu:982-1001). */
NCB_API int ncb_sampler_last_status(void);
NCB_API const char* ncb_sampler_status_message(int status);

#ifdef __cplusplus
}
#endif

#endif /* NAVSAMPLER_H */

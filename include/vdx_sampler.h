/*
 * vdx_sampler.h - C ABI of the B200 (sm_100a) token sampler.
 *
 * Drop-in for the sampling hot path of VindexLLM: TVdxSampler in
 * src/VindexLLM.Sampler.pas. The reference samples on the host after
 * TVdxInference.RunUnembedding (src/VindexLLM.Inference.pas:327-339) has mapped and
 * copied the fp32 logits row out of GPU memory (src/VindexLLM.Compute.pas:718-725).
 * This library samples directly from device-resident [batch, vocab] fp32 or bf16
 * logits, so only token IDs cross PCIe.
 *
 * Conventions
 *   - Every entry point is extern "C", cdecl, and takes plain pointers and sizes.
 *   - Functions return VDXS_OK (0) or a negative VDXS_E_* code; nothing traps or
 *     aborts. vdxs_last_error() returns a readable message for the last failure.
 *   - Pointers named d_* are device pointers on the context's device; h_* are host
 *     pointers. `stream` is a cudaStream_t (NULL = legacy default stream). Work on
 *     device buffers is enqueued on `stream` and is asynchronous unless stated.
 *   - The library never writes the caller's logits. The reference applies the
 *     repetition penalty in place (Sampler.pas:285-303); the result is the same.
 *   - One context per host thread (or serialise calls on a context yourself).
 */
#ifndef VDX_SAMPLER_H
#define VDX_SAMPLER_H

#include <stddef.h>
#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

#if defined(_WIN32)
#define VDXS_API __declspec(dllexport)
#else
#define VDXS_API __attribute__((visibility("default")))
#endif

#define VDXS_ABI_VERSION 1

/* ------------------------------------------------------------------------------
 * Configuration record.
 * Mirrors TVdxSamplerConfig (src/VindexLLM.Sampler.pas:26-34) field by field under
 * the reference's {$A8} record alignment (src/VindexLLM.Defines.inc:13): offsets
 * 0,4,8,12,16,20,24, size 32 bytes, so a Pascal record can be passed by pointer.
 * ---------------------------------------------------------------------------- */
typedef struct vdxs_config {
    float   temperature;    /* 0 = greedy argmax; > 0 = logits are divided by it   */
    int32_t top_k;          /* 0 (or >= vocab) = full-softmax path                 */
    float   top_p;          /* >= 1 = nucleus filter off                           */
    float   min_p;          /* 0 = off; > 0 = floor relative to the top probability */
    float   repeat_penalty; /* 1 = off; x>0 -> x/p, x<0 -> x*p per history entry    */
    int32_t repeat_window;  /* history ring length                                  */
    int64_t seed;           /* 0 = time seeded; > 0 = deterministic                 */
} vdxs_config;

/* Status codes. */
#define VDXS_OK              0
#define VDXS_E_INVALID_ARG  (-1)
#define VDXS_E_CUDA         (-2)
#define VDXS_E_NCCL         (-3)
#define VDXS_E_TIMEOUT      (-4)
#define VDXS_E_UNSUPPORTED  (-5)
#define VDXS_E_NO_MEMORY    (-6)
#define VDXS_E_DEVICE_STATE (-7)

/* Logits element types. bf16 is widened exactly to fp32, then fp32 semantics apply. */
#define VDXS_DTYPE_F32   0
#define VDXS_DTYPE_BF16  1

/* Tie modes.
 * FAITHFUL (default): the token equals what TVdxSampler.Process returns. Rows whose
 *   result depends on the reference's K-slot min-buffer order (a draw that lands in a
 *   run of equal probabilities, top_p >= 1 with top_k > 1, or a probability sum whose
 *   double rounding depends on order) are re-resolved on the GPU by an exact emulation
 *   of the min-buffer scan (Sampler.pas:341-383) and of its sequential double sums.
 * CANONICAL: top-k ties and equal-probability order are broken by lowest index; no
 *   emulation pass. This is the order used by the vocab-sharded path. */
#define VDXS_TIES_FAITHFUL   0
#define VDXS_TIES_CANONICAL  1

/* Per-row result flags (optional output of vdxs_sample_ex). */
#define VDXS_FLAG_GREEDY         (1u << 0)  /* temperature == 0: argmax, no uniform used   */
#define VDXS_FLAG_TOPK           (1u << 1)  /* 0 < top_k < vocab path                      */
#define VDXS_FLAG_FULL           (1u << 2)  /* full-softmax path                           */
#define VDXS_FLAG_BOUNDARY_TIE   (1u << 3)  /* more elements equal the k-th value than fit */
#define VDXS_FLAG_DRAW_TIE_RUN   (1u << 4)  /* drawn position lies in a run of equal probs */
#define VDXS_FLAG_NEAR_BOUNDARY  (1u << 5)  /* |t - CDF edge| <= 1e-6 * sum                */
#define VDXS_FLAG_INEXACT_SUM    (1u << 6)  /* a double sum could depend on summation order */
#define VDXS_FLAG_FALLBACK       (1u << 7)  /* no cumulative sum exceeded t: fallback token */
#define VDXS_FLAG_SLOT_ORDER     (1u << 8)  /* reference walks min-buffer slot order        */
#define VDXS_FLAG_FAITHFUL_PASS  (1u << 9)  /* row re-resolved by the min-buffer emulation  */

/* ------------------------------------------------------------------------------
 * Library and context.
 * ---------------------------------------------------------------------------- */
typedef struct vdxs_context vdxs_context;

/* Returns VDXS_ABI_VERSION. */
VDXS_API int32_t vdxs_abi_version(void);

/* TVdxSampler.DefaultConfig (Sampler.pas:100-109): 0 / 0 / 1 / 0 / 1 / 64 / 0. */
VDXS_API void vdxs_default_config(vdxs_config* out);

/* Creates a context bound to CUDA device `device`. The context owns a lazily grown
 * device workspace (TVdxSampler.EnsureWorkspace, Sampler.pas:250-263). */
VDXS_API int32_t vdxs_create(int32_t device, vdxs_context** out);
VDXS_API int32_t vdxs_destroy(vdxs_context* ctx);

/* Message for the last failing call on `ctx` (ctx may be NULL: message of the last
 * failing call on this thread). Never NULL; "" when there was no error. */
VDXS_API const char* vdxs_last_error(const vdxs_context* ctx);

/* VDXS_TIES_FAITHFUL or VDXS_TIES_CANONICAL (default FAITHFUL). */
VDXS_API int32_t vdxs_set_tie_mode(vdxs_context* ctx, int32_t mode);
VDXS_API int32_t vdxs_get_tie_mode(const vdxs_context* ctx, int32_t* mode);

/* ------------------------------------------------------------------------------
 * Stateless batched sampling: replaces TVdxSampler.Process (Sampler.pas:265-528)
 * for `batch` independent rows, with the penalty history and the uniform supplied
 * by the caller instead of the object's ring and PRNG.
 *
 *   d_logits        [batch, row_stride] fp32 or bf16, first `vocab` entries used
 *   d_history       [batch, history_stride] int32 token ids (ring slots 0..count-1)
 *                   or NULL; ids outside [0, vocab) are ignored (Sampler.pas:292)
 *   d_history_count [batch] int32 entries used per row (NULL = no history)
 *   d_uniform       [batch] fp32 in [0,1): the value NextFloat() would return
 *                   (Sampler.pas:243-248); ignored when temperature == 0
 *   d_out_tokens    [batch] int32
 * ---------------------------------------------------------------------------- */
VDXS_API int32_t vdxs_sample(vdxs_context* ctx, const vdxs_config* cfg,
                             const void* d_logits, int32_t dtype, int32_t batch,
                             int32_t vocab, int64_t row_stride,
                             const int32_t* d_history, int64_t history_stride,
                             const int32_t* d_history_count,
                             const float* d_uniform, int32_t* d_out_tokens,
                             void* stream);

/* As vdxs_sample, plus optional diagnostics (any may be NULL):
 *   d_out_flags  [batch] VDXS_FLAG_* bits
 *   d_out_idx    [batch, out_k] survivor token ids in draw-walk order (-1 padded)
 *   d_out_prob   [batch, out_k] their unnormalised probabilities after min-p and
 *                before the top-p cut (the values the reference sums, Sampler.pas:389)
 * On the full-softmax path d_out_idx/d_out_prob are filled with -1 / 0. */
VDXS_API int32_t vdxs_sample_ex(vdxs_context* ctx, const vdxs_config* cfg,
                                const void* d_logits, int32_t dtype, int32_t batch,
                                int32_t vocab, int64_t row_stride,
                                const int32_t* d_history, int64_t history_stride,
                                const int32_t* d_history_count,
                                const float* d_uniform, int32_t* d_out_tokens,
                                uint32_t* d_out_flags, int32_t* d_out_idx,
                                float* d_out_prob, int32_t out_k, void* stream);

/* Host-buffer variant with Process's calling shape: host logits/history/uniforms in,
 * host tokens out. Copies inputs to the context's device workspace on `stream`,
 * samples, copies the tokens back and synchronises `stream` before returning.
 * Pinned host memory gives the fastest copies. */
VDXS_API int32_t vdxs_sample_host(vdxs_context* ctx, const vdxs_config* cfg,
                                  const void* h_logits, int32_t dtype, int32_t batch,
                                  int32_t vocab, int64_t row_stride,
                                  const int32_t* h_history, int64_t history_stride,
                                  const int32_t* h_history_count,
                                  const float* h_uniform, int32_t* h_out_tokens,
                                  void* stream);

/* Allocation-free variant of vdxs_sample for callers that cannot allocate device
 * memory while sampling: for example a host that reserves all of its GPU memory when
 * the model loads and treats any later allocation as an error, or a decode loop that
 * must not take the implicit device-wide synchronisation of cudaMalloc/cudaFree.
 * No counterpart in the reference (its sampler runs on the host and allocates its
 * workspace lazily, Sampler.pas:250-263).
 *
 * Runs on the calling thread's current CUDA device and takes no context: its
 * workspace is a fixed 32 MiB device array built into the library, which every GPU
 * that loads the library holds until the process exits. Calls whose workspace would
 * exceed it return VDXS_E_UNSUPPORTED (batch 512 at vocab 262144 with top_k 64 fits;
 * batch 1024 with top_k 1024 does not). Where vdxs_sample would use long candidate
 * lists (small batches with top_k above 64) that do not fit, this call uses shorter
 * ones: the same tokens, rows whose lists overflow take a slower exact select. The
 * call never allocates: no cudaMalloc,
 * cudaFree or allocating library routine. Its first call on a device resolves the
 * array's device address (once per device, with that device current); make that
 * first call before any stream capture. All calls share the one array and it keeps
 * the last call's contents, so calls that overlap on the GPU (other streams, other
 * host threads) race: serialise them. `stream` must belong to the current device
 * (VDXS_E_INVALID_ARG otherwise). `tie_mode` is VDXS_TIES_FAITHFUL or
 * VDXS_TIES_CANONICAL; the other arguments are those of vdxs_sample. */
VDXS_API int32_t vdxs_sample_noalloc(const vdxs_config* cfg, int32_t tie_mode, const void* d_logits,
                                     int32_t dtype, int32_t batch, int32_t vocab,
                                     int64_t row_stride, const int32_t* d_history,
                                     int64_t history_stride, const int32_t* d_history_count,
                                     const float* d_uniform, int32_t* d_out_tokens, void* stream);

/* Status of the last vdxs_sample_noalloc call on the current device, for callers that
 * have no context to pass to vdxs_device_status. Waits for `stream` (the stream of that
 * call, on the current device), then reads the device error word that the call's
 * kernels set instead of trapping: VDXS_E_TIMEOUT when a bounded wait gave up,
 * VDXS_E_DEVICE_STATE when an internal selection check failed; the tokens of that call
 * are then not valid. The word lives in the fixed array and the next
 * vdxs_sample_noalloc call clears it, so check after each call whose tokens matter.
 * Allocates nothing (the word is copied into a host variable). No counterpart in the
 * reference, whose Process runs on the host and cannot fail. */
VDXS_API int32_t vdxs_noalloc_status(void* stream);

/* ------------------------------------------------------------------------------
 * Stateful mirror of TVdxSampler: one sampler state (config, xoshiro256** PRNG,
 * repeat-history ring) per batch row, kept on the host exactly as the reference
 * keeps it; Process draws the row uniforms from the PRNGs and samples on the GPU.
 * ---------------------------------------------------------------------------- */
typedef struct vdxs_sampler vdxs_sampler;

/* TVdxSampler.Create (Sampler.pas:111-122): default config, window 64, time seed. */
VDXS_API int32_t vdxs_sampler_create(vdxs_context* ctx, int32_t batch, vdxs_sampler** out);
VDXS_API int32_t vdxs_sampler_destroy(vdxs_sampler* s);
/* TVdxSampler.SetConfig (Sampler.pas:132-150) applied to every row: reseeds only
 * if the seed changed; resizes and clears the ring only if the window changed. */
VDXS_API int32_t vdxs_sampler_set_config(vdxs_sampler* s, const vdxs_config* cfg);
/* TVdxSampler.GetConfig (Sampler.pas:152-155). */
VDXS_API int32_t vdxs_sampler_get_config(const vdxs_sampler* s, vdxs_config* out);
/* TVdxSampler.AddToHistory (Sampler.pas:530-539) for one row, or for every row
 * (h_tokens[batch]). */
VDXS_API int32_t vdxs_sampler_add_to_history(vdxs_sampler* s, int32_t row, int32_t token);
VDXS_API int32_t vdxs_sampler_add_to_history_batch(vdxs_sampler* s, const int32_t* h_tokens);
/* TVdxSampler.ResetHistory (Sampler.pas:541-549); row = -1 resets every row. */
VDXS_API int32_t vdxs_sampler_reset_history(vdxs_sampler* s, int32_t row);
/* TVdxSampler.Process (Sampler.pas:265-528) for all rows on device logits
 * [batch, row_stride]. Writes the tokens to h_out_tokens (host) and returns after
 * `stream` has completed. One uniform per row is drawn unless temperature == 0. */
VDXS_API int32_t vdxs_sampler_process(vdxs_sampler* s, const void* d_logits,
                                      int32_t dtype, int32_t vocab, int64_t row_stride,
                                      int32_t* h_out_tokens, void* stream);
/* The same with host fp32 logits: the exact calling shape of Process(PSingle, V)
 * used by RunUnembedding today (Inference.pas:336-337). */
VDXS_API int32_t vdxs_sampler_process_host(vdxs_sampler* s, const float* h_logits,
                                           int32_t vocab, int64_t row_stride,
                                           int32_t* h_out_tokens);
/* PRNG access for resume and tests: NextFloat (Sampler.pas:243-248) of one row, and
 * the 4-word xoshiro256** state (Sampler.pas:42-45) of one row. */
VDXS_API int32_t vdxs_sampler_next_float(vdxs_sampler* s, int32_t row, float* out);
VDXS_API int32_t vdxs_sampler_get_prng_state(const vdxs_sampler* s, int32_t row, uint64_t out_state[4]);
VDXS_API int32_t vdxs_sampler_set_prng_state(vdxs_sampler* s, int32_t row, const uint64_t state[4]);
/* Copies one row's ring (slots 0..count-1 in slot order) into h_ids (capacity
 * `capacity`), sets *count and *pos (Sampler.pas:48-50). */
VDXS_API int32_t vdxs_sampler_get_history(const vdxs_sampler* s, int32_t row, int32_t* h_ids,
                                          int32_t capacity, int32_t* count, int32_t* pos);

/* ------------------------------------------------------------------------------
 * Device-resident decode state: the row PRNGs and history rings that the stateful
 * sampler keeps on the host (Sampler.pas:42-50, 157-248, 530-549), kept instead in
 * caller-owned device buffers, so that a decode loop samples without a host round trip
 * per token. The reference has no such interface (its sampler runs on the host).
 *   d_prng        [batch][4] uint64 xoshiro256** states, in the layout of
 *                 vdxs_sampler_get_prng_state (seed them there, or by the reference's
 *                 SplitMix64 rule, Sampler.pas:224-241, and copy them to the device)
 *   d_hist        [batch][window] int32 history rings; d_hist_pos and d_hist_count
 *                 [batch] int32 (zero for an empty ring, as after ResetHistory)
 * ---------------------------------------------------------------------------- */
/* NextFloat (Sampler.pas:243-248) of every row on the device: writes d_uniforms[batch]
 * and advances each row's state by one step, bit-identical to vdxs_sampler_next_float. */
VDXS_API int32_t vdxs_device_uniforms(uint64_t* d_prng, int32_t batch, float* d_uniforms, void* stream);
/* AddToHistory (Sampler.pas:530-539) of d_tokens[batch] into the rings (nothing when
 * window <= 0). When n_stop > 0, rows whose token is one of d_stop_ids[n_stop] get
 * d_stopped[row] = 1; other rows' flags are left as they are. */
VDXS_API int32_t vdxs_device_history_push(int32_t* d_hist, int32_t* d_hist_pos, int32_t* d_hist_count,
                                          int32_t window, const int32_t* d_tokens, int32_t batch,
                                          const int32_t* d_stop_ids, int32_t n_stop, int32_t* d_stopped,
                                          void* stream);
/* One decode step on `stream`, all on the device: the row uniforms from d_prng into
 * d_uniforms[batch] (unless temperature == 0: Process draws only then, Sampler.pas:448,
 * 514), vdxs_sample with the rings as the history (window = cfg->repeat_window), then
 * the tokens pushed into the rings and the stop check. It returns the tokens that
 * vdxs_sampler_process followed by vdxs_sampler_add_to_history_batch return on the same
 * host state. Asynchronous: call vdxs_device_status after a run of steps. After one
 * warm-up call with the same shapes (so the context's workspace no longer grows) the step
 * can be captured in a CUDA graph and replayed, each replay advancing the device state. */
VDXS_API int32_t vdxs_decode_step(vdxs_context* ctx, const vdxs_config* cfg, const void* d_logits,
                                  int32_t dtype, int32_t batch, int32_t vocab, int64_t row_stride,
                                  uint64_t* d_prng, float* d_uniforms, int32_t* d_hist,
                                  int32_t* d_hist_pos, int32_t* d_hist_count,
                                  const int32_t* d_stop_ids, int32_t n_stop, int32_t* d_stopped,
                                  int32_t* d_out_tokens, void* stream);

/* ------------------------------------------------------------------------------
 * Vocab-sharded sampling over several GPUs (one process or thread per GPU).
 * Each rank holds a contiguous vocab shard [vocab_offset, vocab_offset + vocab_shard)
 * of every row. Each rank selects its local top-k (lowest global index wins ties),
 * the (value, global index) candidates are all-gathered with NCCL, and every rank
 * runs the identical merge, top-p and draw, so all ranks return the same tokens.
 * Ties are canonical (lowest global index); history ids are global. The sharded call
 * serves 0 < top_k <= 1024 and greedy (temperature 0); other configurations return
 * VDXS_E_UNSUPPORTED.
 * NCCL is loaded at run time (libnccl.so.2) on the first communicator creation.
 * ---------------------------------------------------------------------------- */
typedef struct vdxs_comm vdxs_comm;

#define VDXS_NCCL_UNIQUE_ID_BYTES 128
#define VDXS_COMM_DEFAULT_TIMEOUT_MS 60000
/* Creates an NCCL unique id on one rank; broadcast the 128 bytes to the others. */
VDXS_API int32_t vdxs_comm_unique_id(uint8_t out_id[VDXS_NCCL_UNIQUE_ID_BYTES]);
/* vdxs_comm_create_ex with timeout_ms = VDXS_COMM_DEFAULT_TIMEOUT_MS. */
VDXS_API int32_t vdxs_comm_create(vdxs_context* ctx, int32_t nranks, int32_t rank,
                                  const uint8_t unique_id[VDXS_NCCL_UNIQUE_ID_BYTES],
                                  vdxs_comm** out);
/* Failure detection for the one collective this library adds (the reference has none;
 * its sampler runs on one host thread). The communicator is created non-blocking and
 * every host-side wait on it (its initialisation, each collective's enqueue, finalisation
 * and vdxs_comm_wait) runs under timeout_ms: when a rank does not join, stops, or NCCL
 * reports an asynchronous error, the communicator is aborted (ncclCommAbort, which also
 * ends NCCL kernels waiting for a peer) and the call returns VDXS_E_TIMEOUT or
 * VDXS_E_NCCL. An aborted communicator refuses every later call with VDXS_E_NCCL and
 * launches nothing; destroy it and create a new one. */
VDXS_API int32_t vdxs_comm_create_ex(vdxs_context* ctx, int32_t nranks, int32_t rank,
                                     const uint8_t unique_id[VDXS_NCCL_UNIQUE_ID_BYTES],
                                     int32_t timeout_ms, vdxs_comm** out);
/* Aborts the communicator now: for a caller that learns on the host (a heartbeat, a
 * store) that a peer left. */
VDXS_API int32_t vdxs_comm_abort(vdxs_comm* comm);
/* VDXS_OK while the communicator is usable; VDXS_E_NCCL after an asynchronous NCCL error
 * (for example a peer process that died) or an abort. Does not wait. */
VDXS_API int32_t vdxs_comm_status(vdxs_comm* comm);
/* Waits for `stream` (the stream of this rank's sharded calls) for at most timeout_ms
 * (<= 0: the communicator's timeout), watching the communicator for asynchronous errors;
 * on either failure the communicator is aborted, so NCCL kernels waiting for a peer
 * return, and VDXS_E_TIMEOUT or VDXS_E_NCCL is returned. */
VDXS_API int32_t vdxs_comm_wait(vdxs_comm* comm, void* stream, int32_t timeout_ms);
VDXS_API int32_t vdxs_comm_destroy(vdxs_comm* comm);

VDXS_API int32_t vdxs_sample_sharded(vdxs_context* ctx, vdxs_comm* comm,
                                     const vdxs_config* cfg,
                                     const void* d_logits_shard, int32_t dtype,
                                     int32_t batch, int32_t vocab_shard,
                                     int64_t row_stride, int64_t vocab_offset,
                                     int64_t vocab_total,
                                     const int32_t* d_history, int64_t history_stride,
                                     const int32_t* d_history_count,
                                     const float* d_uniform, int32_t* d_out_tokens,
                                     uint32_t* d_out_flags, void* stream);

/* ------------------------------------------------------------------------------
 * Status and diagnostics. None of these has a counterpart in the reference, whose
 * Process runs on the host and cannot fail (Sampler.pas:265-528).
 * ---------------------------------------------------------------------------- */

/* Waits for `stream` and reads the context's device error word, which the kernels
 * set instead of trapping when a bounded wait gives up (VDXS_E_TIMEOUT) or an
 * internal selection check fails (VDXS_E_DEVICE_STATE). A non-zero word means the
 * tokens of the calls since the last check may be wrong; the word and the kernels'
 * self-resetting counters are cleared before returning, so the context stays usable.
 * vdxs_sample_host and vdxs_sampler_process* perform this check themselves. */
VDXS_API int32_t vdxs_device_status(vdxs_context* ctx, void* stream);

/* Profiling hook: while set, every sampling call on `ctx` records `ev_begin`
 * (a cudaEvent_t created on the context's device) on the call's stream immediately
 * before its dominant pass over the logits and `ev_end` immediately after it, so
 * the caller can time that kernel alone. Pass NULL, NULL to stop. */
VDXS_API int32_t vdxs_set_stage_events(vdxs_context* ctx, void* ev_begin, void* ev_end);

/* Number of kernels launched by the library for calls on `ctx` since it was
 * created (NCCL's own kernels are not counted). */
VDXS_API int32_t vdxs_get_launch_count(const vdxs_context* ctx, int64_t* out);

/* ----------------------------------------------------------------------------
 * Unembedding in front of the sampler. Replaces TVdxModel.UnembedToLogits
 * (src/VindexLLM.Model.pas:1258-1271: the tied-embedding matvec of
 * shaders/matvec_q4_0.comp:45-88 on the normed hidden vector) followed by
 * TVdxSampler.Process, so the logits never leave the GPU. The weights are the
 * reference's Q4_0 blocks (18 bytes per 32 elements: fp16 scale, 16 bytes of
 * nibbles, element j low nibble of byte j, element j + 16 high nibble), row-major
 * [out_dim][in_dim / 32]. The logits equal the shader's bit for bit: per row 64
 * partial sums over elements t, t + 64, ... with every product and sum rounded to
 * fp32 (no fused multiply-add), then the pairwise tree over strides 32..1.
 * ---------------------------------------------------------------------------- */
typedef struct vdxs_q4_0_weights vdxs_q4_0_weights;
/* Repacks the device Q4_0 matrix once into the library's lane-major layout (the same
 * number of bytes) on the context's device; synchronises `stream`. in_dim must be a
 * multiple of 32. The source may be freed afterwards. No reference counterpart (the
 * reference uploads its GGUF blocks once, Model.pas:978-982). */
VDXS_API int32_t vdxs_q4_0_prepare(vdxs_context* ctx, const void* d_q4_0, int32_t in_dim,
                                   int32_t out_dim, void* stream, vdxs_q4_0_weights** out);
VDXS_API int32_t vdxs_q4_0_release(vdxs_q4_0_weights* w);
/* logits[batch][out_dim] = hidden[batch][in_dim] x weights^T (the shader's arithmetic).
 * Batches above 8 rows are computed 8 rows at a time. */
VDXS_API int32_t vdxs_unembed_q4_0(vdxs_context* ctx, const vdxs_q4_0_weights* w,
                                   const float* d_hidden, int32_t batch, float* d_logits,
                                   void* stream);
/* vdxs_unembed_q4_0 into a context-owned logits buffer, then vdxs_sample on it. */
VDXS_API int32_t vdxs_sample_unembed_q4_0(vdxs_context* ctx, const vdxs_config* cfg,
                                          const vdxs_q4_0_weights* w, const float* d_hidden,
                                          int32_t batch, const int32_t* d_history,
                                          int64_t history_stride, const int32_t* d_history_count,
                                          const float* d_uniform, int32_t* d_out_tokens,
                                          void* stream);

#ifdef __cplusplus
}
#endif

#endif /* VDX_SAMPLER_H */

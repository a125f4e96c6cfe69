/*
 * vdx_oracle.h - TEST INFRASTRUCTURE ONLY.
 *
 * CPU restatement of VindexLLM's TVdxSampler (src/VindexLLM.Sampler.pas:100-549),
 * used as the parity checker for the CUDA library and as the timed CPU baseline.
 * Only tests/, __graft_entry__.smoke() and bench.py (cpu_baseline leg and the
 * reference arm) may load it. The product library never links or calls it.
 *
 * Parity status: the reference is Delphi (Win64) and no Delphi/FreePascal compiler
 * exists here, so no reference-produced outputs exist. The oracle is pinned by the
 * reference's own unit tests (testbed/UTest.Sampler.pas, restated in tests/) and by
 * an independent pure-Python restatement (oracle/pyref.py). The System.Exp result and
 * the Win64 $EXCESSPRECISION setting are not pinned by any reference test: parity
 * unpinned at that level. Convention used: Single operands are evaluated in Double
 * (the Win64 default) and Exp is the C library double exp, rounded to Single on store.
 */
#ifndef VDX_ORACLE_H
#define VDX_ORACLE_H

#include <stdint.h>
#include "../include/vdx_sampler.h"

#ifdef __cplusplus
extern "C" {
#endif

#define VDXO_API __attribute__((visibility("default")))

/* Object API: one TVdxSampler. */
typedef struct vdxo_sampler vdxo_sampler;
VDXO_API vdxo_sampler* vdxo_create(void);
VDXO_API void vdxo_destroy(vdxo_sampler* s);
VDXO_API void vdxo_default_config(vdxs_config* out);
VDXO_API void vdxo_set_config(vdxo_sampler* s, const vdxs_config* cfg);
VDXO_API void vdxo_get_config(const vdxo_sampler* s, vdxs_config* out);
VDXO_API void vdxo_add_to_history(vdxo_sampler* s, int32_t token);
VDXO_API void vdxo_reset_history(vdxo_sampler* s);
VDXO_API int32_t vdxo_get_history(const vdxo_sampler* s, int32_t* ids, int32_t cap,
                                  int32_t* count, int32_t* pos);
/* Process exactly as the reference: mutates `logits` (penalty) and draws NextFloat. */
VDXO_API int32_t vdxo_process(vdxo_sampler* s, float* logits, int32_t vocab);
VDXO_API uint64_t vdxo_next_uint64(vdxo_sampler* s);
VDXO_API float vdxo_next_float(vdxo_sampler* s);
VDXO_API void vdxo_get_state(const vdxo_sampler* s, uint64_t out[4]);
VDXO_API void vdxo_set_state(vdxo_sampler* s, const uint64_t st[4]);
VDXO_API uint64_t vdxo_splitmix64(uint64_t* state);

/* One row with the uniform injected and a tie mode (VDXS_TIES_*). `logits` is
 * mutated by the penalty. Diagnostics (flags, walk-ordered survivors) are optional. */
VDXO_API int32_t vdxo_process_row(const vdxs_config* cfg, int32_t tie_mode, float* logits,
                                  int32_t vocab, const int32_t* history,
                                  int32_t history_count, float uniform,
                                  uint32_t* out_flags, int32_t* out_idx,
                                  float* out_prob, int32_t out_k);

/* Batch of rows (the oracle counterpart of vdxs_sample_ex), rows split over
 * `nthreads` host threads. Logits are not modified. Returns 0 or -1 on bad args. */
VDXO_API int32_t vdxo_sample_batch(const vdxs_config* cfg, int32_t tie_mode,
                                   const void* logits, int32_t dtype, int32_t batch,
                                   int32_t vocab, int64_t row_stride,
                                   const int32_t* history, int64_t history_stride,
                                   const int32_t* history_count, const float* uniform,
                                   int32_t* out_tokens, uint32_t* out_flags,
                                   int32_t* out_idx, float* out_prob, int32_t out_k,
                                   int32_t nthreads);

/* The tied-embedding unembedding of TVdxModel.UnembedToLogits (Model.pas:1258-1271) as
 * shaders/matvec_q4_0.comp computes it (:45-88): out[r] = row r of the Q4_0 matrix
 * (18-byte blocks: fp16 scale, 16 bytes of nibbles) times x, summed by 64 partial sums
 * (element e goes to partial e mod 64, in order) and a pairwise tree (strides 32..1).
 * `batch` input vectors of in_dim floats give batch rows of out_dim floats. in_dim must
 * be a multiple of 32. Returns 0, or -1 on bad arguments. */
VDXO_API int32_t vdxo_matvec_q4_0(const uint8_t* weights, const float* x, int32_t batch,
                                  int32_t in_dim, int32_t out_dim, float* out,
                                  int32_t nthreads);

#ifdef __cplusplus
}
#endif
#endif

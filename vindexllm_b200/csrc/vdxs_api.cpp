// vdxs_api.cpp - the C ABI declared in include/vdx_sampler.h.
//
// Validates arguments, resolves TVdxSamplerConfig into a kernel path (greedy /
// top-k / full softmax, Sampler.pas:305-327), owns the device workspace, and keeps
// the stateful per-row sampler state (xoshiro256** PRNG and repeat-history ring,
// Sampler.pas:41-50) on the host exactly as the reference does.
#include "../../include/vdx_sampler.h"
#include "vdxs_internal.h"

#include <cuda_runtime.h>
#include <dlfcn.h>
#include <nccl.h>

#include <algorithm>
#include <chrono>
#include <cstdarg>
#include <cstdio>
#include <cstring>
#include <mutex>
#include <string>
#include <thread>
#include <vector>

using namespace vdxs;

struct vdxs_context {
    int device = 0;
    int smem_optin = 0;
    int sm_count = 0;
    int tie_mode = VDXS_TIES_FAITHFUL;
    Workspace ws;
    std::string last_error;
    cudaEvent_t ev_begin = nullptr;  // profiling hook (vdxs_set_stage_events)
    cudaEvent_t ev_end = nullptr;
    int64_t launches = 0;            // kernels launched for this context
};

namespace {

thread_local std::string g_thread_error;

int32_t fail(vdxs_context* ctx, int32_t code, const char* fmt, ...) {
    char buf[512];
    va_list ap;
    va_start(ap, fmt);
    vsnprintf(buf, sizeof(buf), fmt, ap);
    va_end(ap);
    g_thread_error = buf;
    if (ctx) ctx->last_error = buf;
    return code;
}

int32_t cuda_fail(vdxs_context* ctx, cudaError_t e, const char* what) {
    return fail(ctx, VDXS_E_CUDA, "%s: %s (%s)", what, cudaGetErrorString(e), cudaGetErrorName(e));
}

void ok(vdxs_context* ctx) {
    g_thread_error.clear();
    if (ctx) ctx->last_error.clear();
}

// Switches to the context's device for the duration of a call.
struct DeviceGuard {
    int prev = -1;
    bool changed = false;
    explicit DeviceGuard(int dev) {
        if (cudaGetDevice(&prev) == cudaSuccess && prev != dev) {
            changed = cudaSetDevice(dev) == cudaSuccess;
        }
    }
    ~DeviceGuard() {
        if (changed) cudaSetDevice(prev);
    }
};

vdxs_config default_config() {  // Sampler.pas:100-109
    vdxs_config c;
    c.temperature = 0.0f;
    c.top_k = 0;
    c.top_p = 1.0f;
    c.min_p = 0.0f;
    c.repeat_penalty = 1.0f;
    c.repeat_window = 64;
    c.seed = 0;
    return c;
}

// Fills the configuration part of SampleArgs. vocab_total decides the path.
int32_t resolve_config(vdxs_context* ctx, const vdxs_config* cfg, int64_t vocab_total, SampleArgs* a) {
    if (cfg->temperature == 0.0f) {  // Sampler.pas:306
        a->path = kGreedy;
        a->K = 1;
    } else if (cfg->top_k > 0 && (int64_t)cfg->top_k < vocab_total) {  // :327
        a->path = kTopK;
        a->K = cfg->top_k;
    } else {
        a->path = kFull;
        a->K = 0;
    }
    a->inv_temp = (float)(1.0 / (double)cfg->temperature);  // :325
    a->min_p = cfg->min_p;
    a->top_p = cfg->top_p;
    a->penalty = cfg->repeat_penalty;
    return VDXS_OK;
}

int32_t validate_common(vdxs_context* ctx, const vdxs_config* cfg, const void* logits, int32_t dtype,
                        int32_t batch, int32_t vocab, int64_t row_stride, const int32_t* hist,
                        int64_t hist_stride, const int32_t* hist_count, int32_t* out_tokens) {
    if (!ctx) return fail(nullptr, VDXS_E_INVALID_ARG, "context is NULL");
    if (!cfg) return fail(ctx, VDXS_E_INVALID_ARG, "config is NULL");
    if (!logits) return fail(ctx, VDXS_E_INVALID_ARG, "logits pointer is NULL");
    if (!out_tokens) return fail(ctx, VDXS_E_INVALID_ARG, "output token pointer is NULL");
    if (dtype != VDXS_DTYPE_F32 && dtype != VDXS_DTYPE_BF16)
        return fail(ctx, VDXS_E_INVALID_ARG, "dtype %d is neither VDXS_DTYPE_F32 nor VDXS_DTYPE_BF16", dtype);
    if (batch < 1) return fail(ctx, VDXS_E_INVALID_ARG, "batch must be >= 1 (got %d)", batch);
    if (batch > 65535) return fail(ctx, VDXS_E_UNSUPPORTED, "batch %d exceeds 65535", batch);
    if (vocab < 1) return fail(ctx, VDXS_E_INVALID_ARG, "vocab must be >= 1 (got %d)", vocab);
    if (row_stride < vocab)
        return fail(ctx, VDXS_E_INVALID_ARG, "row_stride %lld is smaller than vocab %d", (long long)row_stride, vocab);
    if (hist && !hist_count)
        return fail(ctx, VDXS_E_INVALID_ARG, "history given without history counts");
    if (hist && hist_stride < 1) return fail(ctx, VDXS_E_INVALID_ARG, "history_stride must be >= 1");
    if (hist && hist_stride > kMaxHistory)
        return fail(ctx, VDXS_E_UNSUPPORTED, "history_stride %lld exceeds the supported maximum %d",
                    (long long)hist_stride, kMaxHistory);
    return VDXS_OK;
}

template <typename P>
cudaError_t grow_dev(P** ptr, size_t* cap, size_t want, cudaStream_t stream) {
    if (*ptr && *cap >= want) return cudaSuccess;
    if (*ptr) {
        cudaStreamSynchronize(stream);
        cudaFree(*ptr);
        *ptr = nullptr;
    }
    cudaError_t e = cudaMalloc((void**)ptr, std::max<size_t>(want, 1) * sizeof(P));
    if (e != cudaSuccess) {
        *ptr = nullptr;
        *cap = 0;
        return e;
    }
    *cap = want;
    return cudaSuccess;
}

// Maps a non-zero device error word to a status; clears the word and the kernels'
// self-resetting counters so the next call starts clean.
int32_t device_word_status(vdxs_context* ctx, int32_t word, cudaStream_t stream) {
    if (word == 0) return VDXS_OK;
    reset_device_state(ctx->ws, stream);
    cudaStreamSynchronize(stream);
    if (word == 3)
        return fail(ctx, VDXS_E_TIMEOUT, "a bounded device wait gave up (tensor-memory copy did not complete); "
                                         "the tokens of the affected call are not valid");
    return fail(ctx, VDXS_E_DEVICE_STATE, "device selection check failed (code %d); the tokens of the affected "
                                          "call are not valid", word);
}

// The allocation-free entry points pick the scratch array of the current device, so a
// stream created on another device would mix devices: refuse it with a clear error.
// The legacy and per-thread default streams follow the current device.
int32_t check_stream_device(cudaStream_t st) {
    if (st == nullptr || st == cudaStreamLegacy || st == cudaStreamPerThread) return VDXS_OK;
    int cur = 0, sdev = 0;
    cudaError_t e = cudaGetDevice(&cur);
    if (e != cudaSuccess) return cuda_fail(nullptr, e, "cudaGetDevice");
    if ((e = cudaStreamGetDevice(st, &sdev)) != cudaSuccess) return cuda_fail(nullptr, e, "cudaStreamGetDevice");
    if (sdev != cur)
        return fail(nullptr, VDXS_E_INVALID_ARG,
                    "the stream belongs to device %d but device %d is current; make the stream's device current", sdev,
                    cur);
    return VDXS_OK;
}

// Fills the diagnostics part of SampleArgs from the context.
void attach_diagnostics(vdxs_context* ctx, SampleArgs* a) {
    a->ev_begin = ctx->ev_begin;
    a->ev_end = ctx->ev_end;
    a->launches = &ctx->launches;
}

}  // namespace

extern "C" {

VDXS_API int32_t vdxs_abi_version(void) { return VDXS_ABI_VERSION; }

VDXS_API void vdxs_default_config(vdxs_config* out) {
    if (out) *out = default_config();
}

VDXS_API int32_t vdxs_create(int32_t device, vdxs_context** out) {
    if (!out) return fail(nullptr, VDXS_E_INVALID_ARG, "out pointer is NULL");
    *out = nullptr;
    int n = 0;
    cudaError_t e = cudaGetDeviceCount(&n);
    if (e != cudaSuccess) return cuda_fail(nullptr, e, "cudaGetDeviceCount");
    if (device < 0 || device >= n) return fail(nullptr, VDXS_E_INVALID_ARG, "device %d out of range [0,%d)", device, n);
    auto* ctx = new vdxs_context();
    ctx->device = device;
    DeviceGuard g(device);
    if ((e = cudaDeviceGetAttribute(&ctx->smem_optin, cudaDevAttrMaxSharedMemoryPerBlockOptin, device)) != cudaSuccess ||
        (e = cudaDeviceGetAttribute(&ctx->sm_count, cudaDevAttrMultiProcessorCount, device)) != cudaSuccess) {
        delete ctx;
        return cuda_fail(nullptr, e, "cudaDeviceGetAttribute");
    }
    int major = 0;
    cudaDeviceGetAttribute(&major, cudaDevAttrComputeCapabilityMajor, device);
    if (major < 10) {
        delete ctx;
        return fail(nullptr, VDXS_E_UNSUPPORTED, "device %d is compute capability %d.x; this library is built for sm_100a",
                    device, major);
    }
    *out = ctx;
    ok(ctx);
    return VDXS_OK;
}

VDXS_API int32_t vdxs_destroy(vdxs_context* ctx) {
    if (!ctx) return VDXS_OK;
    {
        DeviceGuard g(ctx->device);
        cudaDeviceSynchronize();
        free_workspace(ctx->ws);
    }
    delete ctx;
    return VDXS_OK;
}

VDXS_API const char* vdxs_last_error(const vdxs_context* ctx) {
    if (ctx) return ctx->last_error.c_str();
    return g_thread_error.c_str();
}

VDXS_API int32_t vdxs_set_tie_mode(vdxs_context* ctx, int32_t mode) {
    if (!ctx) return fail(nullptr, VDXS_E_INVALID_ARG, "context is NULL");
    if (mode != VDXS_TIES_FAITHFUL && mode != VDXS_TIES_CANONICAL)
        return fail(ctx, VDXS_E_INVALID_ARG, "unknown tie mode %d", mode);
    ctx->tie_mode = mode;
    ok(ctx);
    return VDXS_OK;
}

VDXS_API int32_t vdxs_get_tie_mode(const vdxs_context* ctx, int32_t* mode) {
    if (!ctx || !mode) return fail(nullptr, VDXS_E_INVALID_ARG, "NULL argument");
    *mode = ctx->tie_mode;
    return VDXS_OK;
}

VDXS_API int32_t vdxs_sample_ex(vdxs_context* ctx, const vdxs_config* cfg, const void* d_logits, int32_t dtype,
                                int32_t batch, int32_t vocab, int64_t row_stride, const int32_t* d_history,
                                int64_t history_stride, const int32_t* d_history_count, const float* d_uniform,
                                int32_t* d_out_tokens, uint32_t* d_out_flags, int32_t* d_out_idx,
                                float* d_out_prob, int32_t out_k, void* stream) {
    int32_t rc = validate_common(ctx, cfg, d_logits, dtype, batch, vocab, row_stride, d_history, history_stride,
                                 d_history_count, d_out_tokens);
    if (rc != VDXS_OK) return rc;
    if (out_k < 0) return fail(ctx, VDXS_E_INVALID_ARG, "out_k must be >= 0");
    if (out_k > 0 && !d_out_idx && !d_out_prob) out_k = 0;
    SampleArgs a;
    if ((rc = resolve_config(ctx, cfg, vocab, &a)) != VDXS_OK) return rc;
    if (a.path != kGreedy && !d_uniform)
        return fail(ctx, VDXS_E_INVALID_ARG, "uniform pointer is NULL but temperature != 0");
    a.logits = d_logits;
    a.dtype = dtype;
    a.B = batch;
    a.V = vocab;
    a.stride = row_stride;
    a.penalty_on = cfg->repeat_penalty != 1.0f && d_history != nullptr && d_history_count != nullptr;
    a.hist = d_history;
    a.hist_stride = history_stride;
    a.hist_count = d_history_count;
    a.uniform = d_uniform;
    a.tokens = d_out_tokens;
    a.flags = d_out_flags;
    a.out_idx = d_out_idx;
    a.out_prob = d_out_prob;
    a.out_k = out_k;
    a.tie_mode = ctx->tie_mode;
    a.vocab_total = vocab;
    a.stream = (cudaStream_t)stream;
    attach_diagnostics(ctx, &a);

    DeviceGuard g(ctx->device);
    LaunchPlan plan;
    std::string msg;
    cudaError_t e = a.path == kFull ? plan_full(a, &plan, &msg) : plan_topk(a, ctx->smem_optin, &plan, &msg);
    if (e != cudaSuccess) return fail(ctx, VDXS_E_UNSUPPORTED, "%s", msg.c_str());
    if ((e = ensure_workspace(ctx->ws, a, plan, 1, a.stream, &msg)) != cudaSuccess)
        return e == cudaErrorMemoryAllocation ? fail(ctx, VDXS_E_NO_MEMORY, "workspace allocation failed")
                                              : cuda_fail(ctx, e, "workspace");
    if ((e = launch_sample(a, plan, ctx->ws, &msg)) != cudaSuccess) return cuda_fail(ctx, e, "kernel launch");
    ok(ctx);
    return VDXS_OK;
}

VDXS_API int32_t vdxs_sample(vdxs_context* ctx, const vdxs_config* cfg, const void* d_logits, int32_t dtype,
                             int32_t batch, int32_t vocab, int64_t row_stride, const int32_t* d_history,
                             int64_t history_stride, const int32_t* d_history_count, const float* d_uniform,
                             int32_t* d_out_tokens, void* stream) {
    return vdxs_sample_ex(ctx, cfg, d_logits, dtype, batch, vocab, row_stride, d_history, history_stride,
                          d_history_count, d_uniform, d_out_tokens, nullptr, nullptr, nullptr, 0, stream);
}


// Device-resident decode state (no reference C interface: the reference keeps the PRNG
// and the ring on the host, Sampler.pas:157-248, 530-549).
VDXS_API int32_t vdxs_device_uniforms(uint64_t* d_prng, int32_t batch, float* d_uniforms, void* stream) {
    if (!d_prng || !d_uniforms) return fail(nullptr, VDXS_E_INVALID_ARG, "NULL argument");
    if (batch < 1 || batch > 65535) return fail(nullptr, VDXS_E_INVALID_ARG, "batch %d out of range [1,65535]", batch);
    const cudaError_t e = vdxs::launch_device_uniforms(d_prng, batch, d_uniforms, (cudaStream_t)stream);
    if (e != cudaSuccess) return cuda_fail(nullptr, e, "uniforms launch");
    ok(nullptr);
    return VDXS_OK;
}

VDXS_API int32_t vdxs_device_history_push(int32_t* d_hist, int32_t* d_hist_pos, int32_t* d_hist_count,
                                          int32_t window, const int32_t* d_tokens, int32_t batch,
                                          const int32_t* d_stop_ids, int32_t n_stop, int32_t* d_stopped,
                                          void* stream) {
    if (!d_tokens) return fail(nullptr, VDXS_E_INVALID_ARG, "NULL tokens");
    if (batch < 1 || batch > 65535) return fail(nullptr, VDXS_E_INVALID_ARG, "batch %d out of range [1,65535]", batch);
    if (window > 0 && (!d_hist || !d_hist_pos || !d_hist_count))
        return fail(nullptr, VDXS_E_INVALID_ARG, "history ring buffers are NULL");
    if (n_stop < 0 || (n_stop > 0 && (!d_stop_ids || !d_stopped)))
        return fail(nullptr, VDXS_E_INVALID_ARG, "stop list: n_stop %d with NULL buffers", n_stop);
    const cudaError_t e = vdxs::launch_history_push(d_hist, d_hist_pos, d_hist_count, window > 0 ? window : 0,
                                                    d_tokens, batch, d_stop_ids, n_stop, d_stopped,
                                                    (cudaStream_t)stream);
    if (e != cudaSuccess) return cuda_fail(nullptr, e, "history push launch");
    ok(nullptr);
    return VDXS_OK;
}

VDXS_API int32_t vdxs_decode_step(vdxs_context* ctx, const vdxs_config* cfg, const void* d_logits, int32_t dtype,
                                  int32_t batch, int32_t vocab, int64_t row_stride, uint64_t* d_prng,
                                  float* d_uniforms, int32_t* d_hist, int32_t* d_hist_pos, int32_t* d_hist_count,
                                  const int32_t* d_stop_ids, int32_t n_stop, int32_t* d_stopped,
                                  int32_t* d_out_tokens, void* stream) {
    if (!ctx || !cfg) return fail(ctx, VDXS_E_INVALID_ARG, "NULL argument");
    const bool greedy = cfg->temperature == 0.0f;
    if (!greedy && (!d_prng || !d_uniforms)) return fail(ctx, VDXS_E_INVALID_ARG, "PRNG state or uniforms are NULL");
    const int32_t W = cfg->repeat_window > 0 ? cfg->repeat_window : 0;
    if (W > 0 && (!d_hist || !d_hist_pos || !d_hist_count))
        return fail(ctx, VDXS_E_INVALID_ARG, "history ring buffers are NULL");
    if (n_stop < 0 || (n_stop > 0 && (!d_stop_ids || !d_stopped)))
        return fail(ctx, VDXS_E_INVALID_ARG, "stop list: n_stop %d with NULL buffers", n_stop);
    if (batch < 1 || batch > 65535) return fail(ctx, VDXS_E_INVALID_ARG, "batch %d out of range [1,65535]", batch);
    DeviceGuard g(ctx->device);
    const cudaStream_t st = (cudaStream_t)stream;
    cudaError_t e;
    int64_t n = 0;
    if (!greedy) {
        if ((e = vdxs::launch_device_uniforms(d_prng, batch, d_uniforms, st)) != cudaSuccess)
            return cuda_fail(ctx, e, "uniforms launch");
        ++n;
    }
    const bool pen = W > 0 && cfg->repeat_penalty != 1.0f;
    int32_t rc = vdxs_sample(ctx, cfg, d_logits, dtype, batch, vocab, row_stride, pen ? d_hist : nullptr,
                             pen ? (int64_t)W : 0, pen ? d_hist_count : nullptr, greedy ? nullptr : d_uniforms,
                             d_out_tokens, stream);
    if (rc != VDXS_OK) return rc;
    if (W > 0 || n_stop > 0) {
        if ((e = vdxs::launch_history_push(d_hist, d_hist_pos, d_hist_count, W, d_out_tokens, batch, d_stop_ids,
                                           n_stop, d_stopped, st)) != cudaSuccess)
            return cuda_fail(ctx, e, "history push launch");
        ++n;
    }
    ctx->launches += n;
    ok(ctx);
    return VDXS_OK;
}

VDXS_API int32_t vdxs_sample_host(vdxs_context* ctx, const vdxs_config* cfg, const void* h_logits, int32_t dtype,
                                  int32_t batch, int32_t vocab, int64_t row_stride, const int32_t* h_history,
                                  int64_t history_stride, const int32_t* h_history_count, const float* h_uniform,
                                  int32_t* h_out_tokens, void* stream) {
    int32_t rc = validate_common(ctx, cfg, h_logits, dtype, batch, vocab, row_stride, h_history, history_stride,
                                 h_history_count, h_out_tokens);
    if (rc != VDXS_OK) return rc;
    if (cfg->temperature != 0.0f && !h_uniform)
        return fail(ctx, VDXS_E_INVALID_ARG, "uniform pointer is NULL but temperature != 0");
    DeviceGuard g(ctx->device);
    cudaStream_t st = (cudaStream_t)stream;
    Workspace& ws = ctx->ws;
    const size_t esz = dtype == VDXS_DTYPE_BF16 ? 2 : 4;
    const size_t row_bytes = (size_t)vocab * esz;
    // Rows are packed with a 16-byte aligned pitch so the streaming loads stay vectorised.
    const size_t pitch_elems = ((row_bytes + 15) / 16 * 16) / esz;
    cudaError_t e;
    size_t cap_bytes = ws.d_logits_cap;
    unsigned char* dl = (unsigned char*)ws.d_logits;
    if ((e = grow_dev(&dl, &cap_bytes, (size_t)batch * pitch_elems * esz, st)) != cudaSuccess)
        return cuda_fail(ctx, e, "staging allocation");
    ws.d_logits = dl;
    ws.d_logits_cap = cap_bytes;
    size_t rows_cap = ws.d_rows_cap;
    if (!ws.d_unif || rows_cap < (size_t)batch) {
        size_t c1 = 0, c2 = 0, c3 = 0;
        if (ws.d_unif) {
            cudaStreamSynchronize(st);
            cudaFree(ws.d_unif);
            cudaFree(ws.d_tok);
            cudaFree(ws.d_hcnt);
            cudaFreeHost(ws.h_tok_pinned);
            ws.d_unif = nullptr;
            ws.d_tok = nullptr;
            ws.d_hcnt = nullptr;
            ws.h_tok_pinned = nullptr;
        }
        if ((e = grow_dev(&ws.d_unif, &c1, (size_t)batch, st)) != cudaSuccess ||
            (e = grow_dev(&ws.d_tok, &c2, (size_t)batch, st)) != cudaSuccess ||
            (e = grow_dev(&ws.d_hcnt, &c3, (size_t)batch, st)) != cudaSuccess ||
            (e = cudaMallocHost((void**)&ws.h_tok_pinned, sizeof(int32_t) * (batch + 1))) != cudaSuccess)
            return cuda_fail(ctx, e, "staging allocation");
        ws.d_rows_cap = batch;
    }
    if ((e = cudaMemcpy2DAsync(ws.d_logits, pitch_elems * esz, h_logits, (size_t)row_stride * esz, row_bytes, batch,
                               cudaMemcpyHostToDevice, st)) != cudaSuccess)
        return cuda_fail(ctx, e, "logits upload");
    if (cfg->temperature != 0.0f &&
        (e = cudaMemcpyAsync(ws.d_unif, h_uniform, sizeof(float) * batch, cudaMemcpyHostToDevice, st)) != cudaSuccess)
        return cuda_fail(ctx, e, "uniform upload");
    const int32_t* dh = nullptr;
    const int32_t* dhc = nullptr;
    if (h_history && cfg->repeat_penalty != 1.0f) {
        if ((e = grow_dev(&ws.d_hist, &ws.d_hist_cap, (size_t)batch * history_stride, st)) != cudaSuccess)
            return cuda_fail(ctx, e, "history allocation");
        if ((e = cudaMemcpyAsync(ws.d_hist, h_history, sizeof(int32_t) * batch * history_stride,
                                 cudaMemcpyHostToDevice, st)) != cudaSuccess ||
            (e = cudaMemcpyAsync(ws.d_hcnt, h_history_count, sizeof(int32_t) * batch, cudaMemcpyHostToDevice, st)) !=
                cudaSuccess)
            return cuda_fail(ctx, e, "history upload");
        dh = ws.d_hist;
        dhc = ws.d_hcnt;
    }
    rc = vdxs_sample(ctx, cfg, ws.d_logits, dtype, batch, vocab, (int64_t)pitch_elems, dh, history_stride, dhc,
                     cfg->temperature != 0.0f ? ws.d_unif : nullptr, ws.d_tok, stream);
    if (rc != VDXS_OK) return rc;
    if ((e = cudaMemcpyAsync(ws.h_tok_pinned, ws.d_tok, sizeof(int32_t) * batch, cudaMemcpyDeviceToHost, st)) !=
            cudaSuccess ||
        (e = cudaMemcpyAsync(ws.h_tok_pinned + batch, ws.err, sizeof(int32_t), cudaMemcpyDeviceToHost, st)) !=
            cudaSuccess)
        return cuda_fail(ctx, e, "token download");
    if ((e = cudaStreamSynchronize(st)) != cudaSuccess) return cuda_fail(ctx, e, "stream synchronize");
    if ((rc = device_word_status(ctx, ws.h_tok_pinned[batch], st)) != VDXS_OK) return rc;
    std::memcpy(h_out_tokens, ws.h_tok_pinned, sizeof(int32_t) * batch);
    ok(ctx);
    return VDXS_OK;
}

VDXS_API int32_t vdxs_sample_noalloc(const vdxs_config* cfg, int32_t tie_mode, const void* d_logits,
                                     int32_t dtype, int32_t batch, int32_t vocab, int64_t row_stride,
                                     const int32_t* d_history, int64_t history_stride,
                                     const int32_t* d_history_count, const float* d_uniform,
                                     int32_t* d_out_tokens, void* stream) {
    // Argument checks need a context only for their error text: use the thread's.
    if (!cfg) return fail(nullptr, VDXS_E_INVALID_ARG, "config is NULL");
    if (!d_logits || !d_out_tokens) return fail(nullptr, VDXS_E_INVALID_ARG, "NULL logits or token pointer");
    if (dtype != VDXS_DTYPE_F32 && dtype != VDXS_DTYPE_BF16)
        return fail(nullptr, VDXS_E_INVALID_ARG, "dtype %d is neither VDXS_DTYPE_F32 nor VDXS_DTYPE_BF16", dtype);
    if (batch < 1 || batch > 65535) return fail(nullptr, VDXS_E_INVALID_ARG, "batch %d out of range [1,65535]", batch);
    if (vocab < 1 || row_stride < vocab)
        return fail(nullptr, VDXS_E_INVALID_ARG, "vocab %d / row_stride %lld invalid", vocab, (long long)row_stride);
    if (d_history && (!d_history_count || history_stride < 1 || history_stride > kMaxHistory))
        return fail(nullptr, VDXS_E_INVALID_ARG, "history needs counts and 1 <= history_stride <= %d", kMaxHistory);
    if (tie_mode != VDXS_TIES_FAITHFUL && tie_mode != VDXS_TIES_CANONICAL)
        return fail(nullptr, VDXS_E_INVALID_ARG, "unknown tie mode %d", tie_mode);
    SampleArgs a;
    int32_t rc = resolve_config(nullptr, cfg, vocab, &a);
    if (rc != VDXS_OK) return rc;
    if (a.path != kGreedy && !d_uniform)
        return fail(nullptr, VDXS_E_INVALID_ARG, "uniform pointer is NULL but temperature != 0");
    a.logits = d_logits;
    a.dtype = dtype;
    a.B = batch;
    a.V = vocab;
    a.stride = row_stride;
    a.penalty_on = cfg->repeat_penalty != 1.0f && d_history != nullptr && d_history_count != nullptr;
    a.hist = d_history;
    a.hist_stride = history_stride;
    a.hist_count = d_history_count;
    a.uniform = d_uniform;
    a.tokens = d_out_tokens;
    a.tie_mode = tie_mode;
    a.vocab_total = vocab;
    a.stream = (cudaStream_t)stream;
    void* scratch = nullptr;
    int optin = 0;
    cudaError_t e = noalloc_scratch(&scratch, &optin);
    if (e != cudaSuccess) return cuda_fail(nullptr, e, "scratch address lookup");
    if ((rc = check_stream_device(a.stream)) != VDXS_OK) return rc;
    LaunchPlan plan;
    std::string msg;
    e = a.path == kFull ? plan_full(a, &plan, &msg) : plan_topk(a, optin, &plan, &msg);
    if (e != cudaSuccess) return fail(nullptr, VDXS_E_UNSUPPORTED, "%s", msg.c_str());
    Workspace ws;
    size_t need = carve_workspace(ws, (unsigned char*)scratch, kNoAllocScratchBytes, a, plan);
    if (need > kNoAllocScratchBytes && plan.stream && plan.cand_cap > 4096) {
        // Row lists sized for many stage-1 warps per row (small batches, wide top_k) may not
        // fit the array: shorter lists give the same tokens (a row whose list overflows is
        // selected from the whole row), only slower.
        const int base = (int)std::min<int64_t>(std::max<int64_t>(32LL * a.K, 4096), (int64_t)plan.cand_cap);
        if (base < plan.cand_cap) {
            plan.cand_cap = base;
            need = carve_workspace(ws, (unsigned char*)scratch, kNoAllocScratchBytes, a, plan);
        }
    }
    if (need > kNoAllocScratchBytes)
        return fail(nullptr, VDXS_E_UNSUPPORTED,
                    "this call needs %zu bytes of workspace; the allocation-free entry point has %zu "
                    "(use vdxs_sample with a context)",
                    need, kNoAllocScratchBytes);
    // The array keeps the previous call's contents: reset what must start at zero.
    if ((e = reset_device_state(ws, a.stream)) != cudaSuccess) return cuda_fail(nullptr, e, "scratch reset");
    if ((e = launch_sample(a, plan, ws, &msg)) != cudaSuccess) return cuda_fail(nullptr, e, "kernel launch");
    ok(nullptr);
    return VDXS_OK;
}

VDXS_API int32_t vdxs_noalloc_status(void* stream) {
    void* scratch = nullptr;
    int optin = 0;
    cudaError_t e = noalloc_scratch(&scratch, &optin);
    if (e != cudaSuccess) return cuda_fail(nullptr, e, "scratch address lookup");
    const cudaStream_t st = (cudaStream_t)stream;
    int32_t rc = check_stream_device(st);
    if (rc != VDXS_OK) return rc;
    if ((e = cudaStreamSynchronize(st)) != cudaSuccess) return cuda_fail(nullptr, e, "stream synchronize");
    // The error word is the first field carved out of the array (carve_workspace), so it
    // sits at offset 0 whatever the last call's shapes were. A synchronous copy into a
    // host variable: no device allocation.
    int32_t word = 0;
    if ((e = cudaMemcpy(&word, (const unsigned char*)scratch + kNoAllocErrOffset, sizeof(int32_t),
                        cudaMemcpyDeviceToHost)) != cudaSuccess)
        return cuda_fail(nullptr, e, "error word download");
    if (word == 0) {
        ok(nullptr);
        return VDXS_OK;
    }
    if (word == 3)
        return fail(nullptr, VDXS_E_TIMEOUT, "a bounded device wait gave up in the last allocation-free call; "
                                             "its tokens are not valid");
    return fail(nullptr, VDXS_E_DEVICE_STATE, "device selection check failed (code %d) in the last allocation-free "
                                              "call; its tokens are not valid", word);
}

VDXS_API int32_t vdxs_device_status(vdxs_context* ctx, void* stream) {
    if (!ctx) return fail(nullptr, VDXS_E_INVALID_ARG, "context is NULL");
    DeviceGuard g(ctx->device);
    cudaStream_t st = (cudaStream_t)stream;
    cudaError_t e = cudaStreamSynchronize(st);
    if (e != cudaSuccess) return cuda_fail(ctx, e, "stream synchronize");
    if (!ctx->ws.err) {
        ok(ctx);
        return VDXS_OK;
    }
    int32_t word = 0;
    if ((e = cudaMemcpy(&word, ctx->ws.err, sizeof(int32_t), cudaMemcpyDeviceToHost)) != cudaSuccess)
        return cuda_fail(ctx, e, "error word download");
    int32_t rc = device_word_status(ctx, word, st);
    if (rc == VDXS_OK) ok(ctx);
    return rc;
}

VDXS_API int32_t vdxs_set_stage_events(vdxs_context* ctx, void* ev_begin, void* ev_end) {
    if (!ctx) return fail(nullptr, VDXS_E_INVALID_ARG, "context is NULL");
    if ((ev_begin == nullptr) != (ev_end == nullptr))
        return fail(ctx, VDXS_E_INVALID_ARG, "give both events or neither");
    ctx->ev_begin = (cudaEvent_t)ev_begin;
    ctx->ev_end = (cudaEvent_t)ev_end;
    ok(ctx);
    return VDXS_OK;
}

VDXS_API int32_t vdxs_get_launch_count(const vdxs_context* ctx, int64_t* out) {
    if (!ctx || !out) return fail(nullptr, VDXS_E_INVALID_ARG, "NULL argument");
    *out = ctx->launches;
    return VDXS_OK;
}

}  // extern "C"

// =====================================================================================
// Stateful sampler: the TVdxSampler object API (Sampler.pas:37-91) for `batch` rows.
// =====================================================================================
namespace {

inline uint64_t rotl64(uint64_t x, int k) { return (x << k) | (x >> (64 - k)); }
uint64_t splitmix64(uint64_t& st) {  // Sampler.pas:194-201
    st += 0x9E3779B97F4A7C15ull;
    uint64_t r = st;
    r = (r ^ (r >> 30)) * 0xBF58476D1CE4E5B9ull;
    r = (r ^ (r >> 27)) * 0x94D049BB133111EBull;
    return r ^ (r >> 31);
}

struct RowState {
    uint64_t s[4] = {0, 0, 0, 0};
    std::vector<int32_t> history;  // FHistory
    int32_t pos = 0, count = 0;    // FHistoryPos, FHistoryCount
    void seed(int64_t seed, uint64_t salt) {  // Sampler.pas:224-241
        uint64_t st = seed == 0 ? (uint64_t)std::chrono::steady_clock::now().time_since_epoch().count() + salt
                                : (uint64_t)seed;
        for (int i = 0; i < 4; ++i) s[i] = splitmix64(st);
    }
    uint64_t next() {  // Sampler.pas:208-222 (xoshiro256**)
        const uint64_t result = rotl64(s[1] * 5, 7) * 9;
        const uint64_t t = s[1] << 17;
        s[2] ^= s[0];
        s[3] ^= s[1];
        s[1] ^= s[2];
        s[0] ^= s[3];
        s[2] ^= t;
        s[3] = rotl64(s[3], 45);
        return result;
    }
    float next_float() { return (float)((double)(next() >> 40) / 16777216.0); }  // :243-248
};

}  // namespace

struct vdxs_sampler {
    vdxs_context* ctx = nullptr;
    int32_t batch = 0;
    vdxs_config cfg;
    std::vector<RowState> rows;
    // device / pinned staging
    int32_t* d_hist = nullptr;
    size_t d_hist_cap = 0;
    int32_t* d_hcnt = nullptr;
    float* d_unif = nullptr;
    int32_t* d_tok = nullptr;
    float* h_unif = nullptr;
    int32_t* h_tok = nullptr;
    int32_t* h_hist = nullptr;
    size_t h_hist_cap = 0;
    int32_t* h_hcnt = nullptr;
    float* d_logits = nullptr;  // process_host staging
    size_t d_logits_cap = 0;
};

namespace {

int32_t sampler_stage_history(vdxs_sampler* s, cudaStream_t st, const int32_t** dh, const int32_t** dhc,
                              int64_t* hstride) {
    *dh = nullptr;
    *dhc = nullptr;
    *hstride = 1;
    const int W = std::max(0, s->cfg.repeat_window);
    if (s->cfg.repeat_penalty == 1.0f || W == 0) return VDXS_OK;
    bool any = false;
    for (auto& r : s->rows) any |= r.count > 0;
    if (!any) return VDXS_OK;
    if (W > kMaxHistory)
        return fail(s->ctx, VDXS_E_UNSUPPORTED, "repeat_window %d exceeds the supported maximum %d", W, kMaxHistory);
    const size_t need = (size_t)s->batch * W;
    cudaError_t e;
    if (s->h_hist_cap < need) {
        if (s->h_hist) cudaFreeHost(s->h_hist);
        s->h_hist = nullptr;
        if ((e = cudaMallocHost((void**)&s->h_hist, need * sizeof(int32_t))) != cudaSuccess)
            return cuda_fail(s->ctx, e, "pinned history staging");
        s->h_hist_cap = need;
    }
    if (s->d_hist_cap < need) {
        if (s->d_hist) {
            cudaStreamSynchronize(st);
            cudaFree(s->d_hist);
        }
        s->d_hist = nullptr;
        if ((e = cudaMalloc((void**)&s->d_hist, need * sizeof(int32_t))) != cudaSuccess)
            return cuda_fail(s->ctx, e, "history allocation");
        s->d_hist_cap = need;
    }
    for (int r = 0; r < s->batch; ++r) {
        const RowState& rs = s->rows[r];
        std::memcpy(s->h_hist + (size_t)r * W, rs.history.data(), sizeof(int32_t) * rs.count);
        s->h_hcnt[r] = rs.count;
    }
    if ((e = cudaMemcpyAsync(s->d_hist, s->h_hist, need * sizeof(int32_t), cudaMemcpyHostToDevice, st)) !=
            cudaSuccess ||
        (e = cudaMemcpyAsync(s->d_hcnt, s->h_hcnt, sizeof(int32_t) * s->batch, cudaMemcpyHostToDevice, st)) !=
            cudaSuccess)
        return cuda_fail(s->ctx, e, "history upload");
    *dh = s->d_hist;
    *dhc = s->d_hcnt;
    *hstride = W;
    return VDXS_OK;
}

int32_t sampler_run(vdxs_sampler* s, const void* d_logits, int32_t dtype, int32_t vocab, int64_t row_stride,
                    int32_t* h_out, cudaStream_t st) {
    cudaError_t e;
    const bool greedy = s->cfg.temperature == 0.0f;
    if (!greedy) {
        for (int r = 0; r < s->batch; ++r) s->h_unif[r] = s->rows[r].next_float();  // one draw per row (:448/:514)
        if ((e = cudaMemcpyAsync(s->d_unif, s->h_unif, sizeof(float) * s->batch, cudaMemcpyHostToDevice, st)) !=
            cudaSuccess)
            return cuda_fail(s->ctx, e, "uniform upload");
    }
    const int32_t* dh;
    const int32_t* dhc;
    int64_t hs;
    int32_t rc = sampler_stage_history(s, st, &dh, &dhc, &hs);
    if (rc != VDXS_OK) return rc;
    rc = vdxs_sample(s->ctx, &s->cfg, d_logits, dtype, s->batch, vocab, row_stride, dh, hs, dhc,
                     greedy ? nullptr : s->d_unif, s->d_tok, st);
    if (rc != VDXS_OK) return rc;
    if ((e = cudaMemcpyAsync(s->h_tok, s->d_tok, sizeof(int32_t) * s->batch, cudaMemcpyDeviceToHost, st)) !=
            cudaSuccess ||
        (e = cudaMemcpyAsync(s->h_tok + s->batch, s->ctx->ws.err, sizeof(int32_t), cudaMemcpyDeviceToHost, st)) !=
            cudaSuccess)
        return cuda_fail(s->ctx, e, "token download");
    if ((e = cudaStreamSynchronize(st)) != cudaSuccess) return cuda_fail(s->ctx, e, "stream synchronize");
    if ((rc = device_word_status(s->ctx, s->h_tok[s->batch], st)) != VDXS_OK) return rc;
    std::memcpy(h_out, s->h_tok, sizeof(int32_t) * s->batch);
    ok(s->ctx);
    return VDXS_OK;
}

}  // namespace

extern "C" {

VDXS_API int32_t vdxs_sampler_create(vdxs_context* ctx, int32_t batch, vdxs_sampler** out) {
    if (!ctx || !out) return fail(ctx, VDXS_E_INVALID_ARG, "NULL argument");
    if (batch < 1 || batch > 65535) return fail(ctx, VDXS_E_INVALID_ARG, "batch %d out of range [1,65535]", batch);
    *out = nullptr;
    DeviceGuard g(ctx->device);
    auto* s = new vdxs_sampler();
    s->ctx = ctx;
    s->batch = batch;
    s->cfg = default_config();  // Sampler.pas:114
    s->rows.resize(batch);
    for (int r = 0; r < batch; ++r) {
        s->rows[r].history.assign((size_t)s->cfg.repeat_window, 0);  // :120
        s->rows[r].seed(0, (uint64_t)r);                              // :121
    }
    cudaError_t e;
    if ((e = cudaMalloc((void**)&s->d_hcnt, sizeof(int32_t) * batch)) != cudaSuccess ||
        (e = cudaMalloc((void**)&s->d_unif, sizeof(float) * batch)) != cudaSuccess ||
        (e = cudaMalloc((void**)&s->d_tok, sizeof(int32_t) * batch)) != cudaSuccess ||
        (e = cudaMallocHost((void**)&s->h_unif, sizeof(float) * batch)) != cudaSuccess ||
        (e = cudaMallocHost((void**)&s->h_tok, sizeof(int32_t) * (batch + 1))) != cudaSuccess ||
        (e = cudaMallocHost((void**)&s->h_hcnt, sizeof(int32_t) * batch)) != cudaSuccess) {
        vdxs_sampler_destroy(s);
        return cuda_fail(ctx, e, "sampler allocation");
    }
    *out = s;
    ok(ctx);
    return VDXS_OK;
}

VDXS_API int32_t vdxs_sampler_destroy(vdxs_sampler* s) {
    if (!s) return VDXS_OK;
    DeviceGuard g(s->ctx->device);
    cudaDeviceSynchronize();
    cudaFree(s->d_hist);
    cudaFree(s->d_hcnt);
    cudaFree(s->d_unif);
    cudaFree(s->d_tok);
    cudaFree(s->d_logits);
    if (s->h_unif) cudaFreeHost(s->h_unif);
    if (s->h_tok) cudaFreeHost(s->h_tok);
    if (s->h_hist) cudaFreeHost(s->h_hist);
    if (s->h_hcnt) cudaFreeHost(s->h_hcnt);
    delete s;
    return VDXS_OK;
}

VDXS_API int32_t vdxs_sampler_set_config(vdxs_sampler* s, const vdxs_config* cfg) {  // Sampler.pas:132-150
    if (!s || !cfg) return fail(s ? s->ctx : nullptr, VDXS_E_INVALID_ARG, "NULL argument");
    const bool seed_changed = cfg->seed != s->cfg.seed;
    s->cfg = *cfg;
    const size_t want = (size_t)std::max(0, cfg->repeat_window);
    for (int r = 0; r < s->batch; ++r) {
        RowState& rs = s->rows[r];
        if (rs.history.size() != want) {
            rs.history.assign(want, 0);
            rs.pos = 0;
            rs.count = 0;
        }
        if (seed_changed) rs.seed(cfg->seed, (uint64_t)r);
    }
    ok(s->ctx);
    return VDXS_OK;
}

VDXS_API int32_t vdxs_sampler_get_config(const vdxs_sampler* s, vdxs_config* out) {
    if (!s || !out) return fail(nullptr, VDXS_E_INVALID_ARG, "NULL argument");
    *out = s->cfg;
    return VDXS_OK;
}

VDXS_API int32_t vdxs_sampler_add_to_history(vdxs_sampler* s, int32_t row, int32_t token) {  // Sampler.pas:530-539
    if (!s) return fail(nullptr, VDXS_E_INVALID_ARG, "sampler is NULL");
    if (row < 0 || row >= s->batch) return fail(s->ctx, VDXS_E_INVALID_ARG, "row %d out of range", row);
    const int W = s->cfg.repeat_window;
    if (W <= 0) return VDXS_OK;
    RowState& rs = s->rows[row];
    rs.history[rs.pos] = token;
    rs.pos = (rs.pos + 1) % W;
    if (rs.count < W) ++rs.count;
    return VDXS_OK;
}

VDXS_API int32_t vdxs_sampler_add_to_history_batch(vdxs_sampler* s, const int32_t* h_tokens) {
    if (!s || !h_tokens) return fail(s ? s->ctx : nullptr, VDXS_E_INVALID_ARG, "NULL argument");
    for (int r = 0; r < s->batch; ++r) vdxs_sampler_add_to_history(s, r, h_tokens[r]);
    return VDXS_OK;
}

VDXS_API int32_t vdxs_sampler_reset_history(vdxs_sampler* s, int32_t row) {  // Sampler.pas:541-549
    if (!s) return fail(nullptr, VDXS_E_INVALID_ARG, "sampler is NULL");
    if (row < -1 || row >= s->batch) return fail(s->ctx, VDXS_E_INVALID_ARG, "row %d out of range", row);
    for (int r = (row < 0 ? 0 : row); r < (row < 0 ? s->batch : row + 1); ++r) {
        RowState& rs = s->rows[r];
        rs.pos = 0;
        rs.count = 0;
        if (s->cfg.seed > 0) rs.seed(s->cfg.seed, (uint64_t)r);
    }
    return VDXS_OK;
}

VDXS_API int32_t vdxs_sampler_process(vdxs_sampler* s, const void* d_logits, int32_t dtype, int32_t vocab,
                                      int64_t row_stride, int32_t* h_out_tokens, void* stream) {
    if (!s || !d_logits || !h_out_tokens) return fail(s ? s->ctx : nullptr, VDXS_E_INVALID_ARG, "NULL argument");
    DeviceGuard g(s->ctx->device);
    return sampler_run(s, d_logits, dtype, vocab, row_stride, h_out_tokens, (cudaStream_t)stream);
}

VDXS_API int32_t vdxs_sampler_process_host(vdxs_sampler* s, const float* h_logits, int32_t vocab, int64_t row_stride,
                                           int32_t* h_out_tokens) {
    if (!s || !h_logits || !h_out_tokens) return fail(s ? s->ctx : nullptr, VDXS_E_INVALID_ARG, "NULL argument");
    if (vocab < 1 || row_stride < vocab) return fail(s->ctx, VDXS_E_INVALID_ARG, "bad vocab/row_stride");
    DeviceGuard g(s->ctx->device);
    const size_t pitch = ((size_t)vocab + 3) / 4 * 4;
    const size_t need = pitch * s->batch;
    cudaError_t e;
    if (s->d_logits_cap < need) {
        cudaFree(s->d_logits);
        s->d_logits = nullptr;
        if ((e = cudaMalloc((void**)&s->d_logits, need * sizeof(float))) != cudaSuccess)
            return cuda_fail(s->ctx, e, "logits staging");
        s->d_logits_cap = need;
    }
    if ((e = cudaMemcpy2DAsync(s->d_logits, pitch * sizeof(float), h_logits, (size_t)row_stride * sizeof(float),
                               (size_t)vocab * sizeof(float), s->batch, cudaMemcpyHostToDevice, nullptr)) !=
        cudaSuccess)
        return cuda_fail(s->ctx, e, "logits upload");
    return sampler_run(s, s->d_logits, VDXS_DTYPE_F32, vocab, (int64_t)pitch, h_out_tokens, nullptr);
}

VDXS_API int32_t vdxs_sampler_next_float(vdxs_sampler* s, int32_t row, float* out) {
    if (!s || !out) return fail(nullptr, VDXS_E_INVALID_ARG, "NULL argument");
    if (row < 0 || row >= s->batch) return fail(s->ctx, VDXS_E_INVALID_ARG, "row %d out of range", row);
    *out = s->rows[row].next_float();
    return VDXS_OK;
}

VDXS_API int32_t vdxs_sampler_get_prng_state(const vdxs_sampler* s, int32_t row, uint64_t out_state[4]) {
    if (!s || !out_state) return fail(nullptr, VDXS_E_INVALID_ARG, "NULL argument");
    if (row < 0 || row >= s->batch) return fail(s->ctx, VDXS_E_INVALID_ARG, "row %d out of range", row);
    std::memcpy(out_state, s->rows[row].s, sizeof(uint64_t) * 4);
    return VDXS_OK;
}

VDXS_API int32_t vdxs_sampler_set_prng_state(vdxs_sampler* s, int32_t row, const uint64_t state[4]) {
    if (!s || !state) return fail(nullptr, VDXS_E_INVALID_ARG, "NULL argument");
    if (row < 0 || row >= s->batch) return fail(s->ctx, VDXS_E_INVALID_ARG, "row %d out of range", row);
    std::memcpy(s->rows[row].s, state, sizeof(uint64_t) * 4);
    return VDXS_OK;
}

VDXS_API int32_t vdxs_sampler_get_history(const vdxs_sampler* s, int32_t row, int32_t* h_ids, int32_t capacity,
                                          int32_t* count, int32_t* pos) {
    if (!s || !count || !pos) return fail(nullptr, VDXS_E_INVALID_ARG, "NULL argument");
    if (row < 0 || row >= s->batch) return fail(s->ctx, VDXS_E_INVALID_ARG, "row %d out of range", row);
    const RowState& rs = s->rows[row];
    *count = rs.count;
    *pos = rs.pos;
    if (h_ids)
        for (int i = 0; i < std::min(capacity, rs.count); ++i) h_ids[i] = rs.history[i];
    return VDXS_OK;
}

}  // extern "C"

// =====================================================================================
// Vocab-sharded sampling with NCCL (resolved at run time with dlopen).
// =====================================================================================
namespace {

struct NcclApi {
    void* handle = nullptr;
    ncclResult_t (*GetUniqueId)(ncclUniqueId*) = nullptr;
    ncclResult_t (*CommInitRankConfig)(ncclComm_t*, int, ncclUniqueId, int, ncclConfig_t*) = nullptr;
    ncclResult_t (*CommGetAsyncError)(ncclComm_t, ncclResult_t*) = nullptr;
    ncclResult_t (*CommFinalize)(ncclComm_t) = nullptr;
    ncclResult_t (*CommDestroy)(ncclComm_t) = nullptr;
    ncclResult_t (*CommAbort)(ncclComm_t) = nullptr;
    ncclResult_t (*AllGather)(const void*, void*, size_t, ncclDataType_t, ncclComm_t, cudaStream_t) = nullptr;
    const char* (*GetErrorString)(ncclResult_t) = nullptr;
    bool ok = false;
};

NcclApi& nccl() {
    static NcclApi api;
    static std::once_flag once;
    std::call_once(once, [] {
        // Prefer a libnccl already loaded in the process (e.g. by the host framework).
        void* h = dlopen("libnccl.so.2", RTLD_NOW | RTLD_GLOBAL | RTLD_NOLOAD);
        if (!h) h = dlopen("libnccl.so.2", RTLD_NOW | RTLD_GLOBAL);
        if (!h) h = dlopen("libnccl.so", RTLD_NOW | RTLD_GLOBAL);
        if (!h) return;
        api.handle = h;
        api.GetUniqueId = (decltype(api.GetUniqueId))dlsym(h, "ncclGetUniqueId");
        api.CommInitRankConfig = (decltype(api.CommInitRankConfig))dlsym(h, "ncclCommInitRankConfig");
        api.CommGetAsyncError = (decltype(api.CommGetAsyncError))dlsym(h, "ncclCommGetAsyncError");
        api.CommFinalize = (decltype(api.CommFinalize))dlsym(h, "ncclCommFinalize");
        api.CommDestroy = (decltype(api.CommDestroy))dlsym(h, "ncclCommDestroy");
        api.CommAbort = (decltype(api.CommAbort))dlsym(h, "ncclCommAbort");
        api.AllGather = (decltype(api.AllGather))dlsym(h, "ncclAllGather");
        api.GetErrorString = (decltype(api.GetErrorString))dlsym(h, "ncclGetErrorString");
        api.ok = api.GetUniqueId && api.CommInitRankConfig && api.CommGetAsyncError && api.CommFinalize &&
                 api.CommDestroy && api.CommAbort && api.AllGather && api.GetErrorString;
    });
    return api;
}

}  // namespace

struct vdxs_comm {
    vdxs_context* ctx = nullptr;
    ncclComm_t comm = nullptr;
    int nranks = 0;
    int rank = 0;
    int timeout_ms = 0;    // deadline of every host-side wait on the communicator
    bool aborted = false;  // ncclCommAbort was called: the communicator is unusable
};

namespace {

using Clock = std::chrono::steady_clock;

// Aborts the communicator (NCCL stops its kernels and proxy threads); it stays unusable.
void comm_abort(vdxs_comm* c) {
    if (c->comm && !c->aborted) {
        DeviceGuard g(c->ctx->device);
        nccl().CommAbort(c->comm);
    }
    c->aborted = true;
}

// Polls the non-blocking communicator until its pending host-side operation (init,
// enqueue, finalize) is done. Returns VDXS_OK, VDXS_E_NCCL (asynchronous error) or
// VDXS_E_TIMEOUT; the communicator is aborted on both failures.
int32_t comm_settle(vdxs_comm* c, const char* what) {
    NcclApi& n = nccl();
    const auto t0 = Clock::now();
    for (;;) {
        ncclResult_t st = ncclSuccess;
        ncclResult_t r = n.CommGetAsyncError(c->comm, &st);
        if (r != ncclSuccess) st = r;
        if (st == ncclSuccess) return VDXS_OK;
        if (st != ncclInProgress) {
            comm_abort(c);
            return fail(c->ctx, VDXS_E_NCCL, "%s: %s; the communicator was aborted", what, n.GetErrorString(st));
        }
        if (std::chrono::duration_cast<std::chrono::milliseconds>(Clock::now() - t0).count() > c->timeout_ms) {
            comm_abort(c);
            return fail(c->ctx, VDXS_E_TIMEOUT,
                        "%s did not complete within %d ms (a rank did not join or stopped); the communicator "
                        "was aborted",
                        what, c->timeout_ms);
        }
        std::this_thread::sleep_for(std::chrono::microseconds(200));
    }
}

}  // namespace

extern "C" {

VDXS_API int32_t vdxs_comm_unique_id(uint8_t out_id[VDXS_NCCL_UNIQUE_ID_BYTES]) {
    static_assert(sizeof(ncclUniqueId) == VDXS_NCCL_UNIQUE_ID_BYTES, "ncclUniqueId size");
    if (!out_id) return fail(nullptr, VDXS_E_INVALID_ARG, "NULL argument");
    NcclApi& n = nccl();
    if (!n.ok) return fail(nullptr, VDXS_E_NCCL, "libnccl.so.2 could not be loaded");
    ncclUniqueId id;
    ncclResult_t r = n.GetUniqueId(&id);
    if (r != ncclSuccess) return fail(nullptr, VDXS_E_NCCL, "ncclGetUniqueId: %s", n.GetErrorString(r));
    std::memcpy(out_id, &id, sizeof(id));
    return VDXS_OK;
}

VDXS_API int32_t vdxs_comm_create_ex(vdxs_context* ctx, int32_t nranks, int32_t rank,
                                     const uint8_t unique_id[VDXS_NCCL_UNIQUE_ID_BYTES], int32_t timeout_ms,
                                     vdxs_comm** out) {
    if (!ctx || !unique_id || !out) return fail(ctx, VDXS_E_INVALID_ARG, "NULL argument");
    *out = nullptr;
    if (nranks < 1 || rank < 0 || rank >= nranks)
        return fail(ctx, VDXS_E_INVALID_ARG, "rank %d / nranks %d invalid", rank, nranks);
    if (timeout_ms < 1) return fail(ctx, VDXS_E_INVALID_ARG, "timeout_ms must be >= 1 (got %d)", timeout_ms);
    NcclApi& n = nccl();
    if (!n.ok) return fail(ctx, VDXS_E_NCCL, "libnccl.so.2 could not be loaded");
    DeviceGuard g(ctx->device);
    ncclUniqueId id;
    std::memcpy(&id, unique_id, sizeof(id));
    auto* c = new vdxs_comm();
    c->ctx = ctx;
    c->nranks = nranks;
    c->rank = rank;
    c->timeout_ms = timeout_ms;
    // Non-blocking: the init returns at once and is polled against the deadline, so a
    // rank that never joins ends in VDXS_E_TIMEOUT instead of a hang.
    ncclConfig_t cfg = NCCL_CONFIG_INITIALIZER;
    cfg.blocking = 0;
    ncclResult_t r = n.CommInitRankConfig(&c->comm, nranks, id, rank, &cfg);
    if (r != ncclSuccess && r != ncclInProgress) {
        if (c->comm) n.CommAbort(c->comm);
        delete c;
        return fail(ctx, VDXS_E_NCCL, "ncclCommInitRankConfig: %s", n.GetErrorString(r));
    }
    const int32_t rc = comm_settle(c, "communicator initialisation");
    if (rc != VDXS_OK) {
        const std::string msg = ctx->last_error;
        delete c;
        return fail(ctx, rc, "%s", msg.c_str());
    }
    *out = c;
    ok(ctx);
    return VDXS_OK;
}

VDXS_API int32_t vdxs_comm_create(vdxs_context* ctx, int32_t nranks, int32_t rank,
                                  const uint8_t unique_id[VDXS_NCCL_UNIQUE_ID_BYTES], vdxs_comm** out) {
    return vdxs_comm_create_ex(ctx, nranks, rank, unique_id, VDXS_COMM_DEFAULT_TIMEOUT_MS, out);
}

VDXS_API int32_t vdxs_comm_abort(vdxs_comm* c) {
    if (!c) return fail(nullptr, VDXS_E_INVALID_ARG, "communicator is NULL");
    comm_abort(c);
    return VDXS_OK;
}

VDXS_API int32_t vdxs_comm_status(vdxs_comm* c) {
    if (!c) return fail(nullptr, VDXS_E_INVALID_ARG, "communicator is NULL");
    if (c->aborted) return fail(c->ctx, VDXS_E_NCCL, "the communicator was aborted");
    ncclResult_t st = ncclSuccess;
    ncclResult_t r = nccl().CommGetAsyncError(c->comm, &st);
    if (r != ncclSuccess) st = r;
    if (st == ncclSuccess || st == ncclInProgress) return VDXS_OK;
    return fail(c->ctx, VDXS_E_NCCL, "communicator error: %s", nccl().GetErrorString(st));
}

VDXS_API int32_t vdxs_comm_wait(vdxs_comm* c, void* stream, int32_t timeout_ms) {
    if (!c) return fail(nullptr, VDXS_E_INVALID_ARG, "communicator is NULL");
    if (c->aborted) return fail(c->ctx, VDXS_E_NCCL, "the communicator was aborted");
    DeviceGuard g(c->ctx->device);
    const cudaStream_t st = (cudaStream_t)stream;
    const int limit = timeout_ms > 0 ? timeout_ms : c->timeout_ms;
    NcclApi& n = nccl();
    const auto t0 = Clock::now();
    for (;;) {
        const cudaError_t q = cudaStreamQuery(st);
        if (q == cudaSuccess) break;
        if (q != cudaErrorNotReady) return cuda_fail(c->ctx, q, "stream query");
        ncclResult_t as = ncclSuccess;
        ncclResult_t r = n.CommGetAsyncError(c->comm, &as);
        if (r != ncclSuccess) as = r;
        if (as != ncclSuccess && as != ncclInProgress) {
            comm_abort(c);
            return fail(c->ctx, VDXS_E_NCCL, "communicator error while waiting: %s; the communicator was aborted",
                        n.GetErrorString(as));
        }
        if (std::chrono::duration_cast<std::chrono::milliseconds>(Clock::now() - t0).count() > limit) {
            comm_abort(c);
            return fail(c->ctx, VDXS_E_TIMEOUT,
                        "the stream did not complete within %d ms (a peer stopped in a collective?); the "
                        "communicator was aborted",
                        limit);
        }
        std::this_thread::sleep_for(std::chrono::microseconds(100));
    }
    return VDXS_OK;
}

VDXS_API int32_t vdxs_comm_destroy(vdxs_comm* c) {
    if (!c) return VDXS_OK;
    NcclApi& n = nccl();
    if (c->comm && n.ok) {
        DeviceGuard g(c->ctx->device);
        if (!c->aborted) {
            // Flush the pending operations under the deadline, then free.
            ncclResult_t r = n.CommFinalize(c->comm);
            if ((r == ncclSuccess || r == ncclInProgress) && comm_settle(c, "communicator finalisation") == VDXS_OK)
                n.CommDestroy(c->comm);
            else
                comm_abort(c);
        }
    }
    delete c;
    return VDXS_OK;
}

VDXS_API int32_t vdxs_sample_sharded(vdxs_context* ctx, vdxs_comm* comm, const vdxs_config* cfg,
                                     const void* d_logits_shard, int32_t dtype, int32_t batch, int32_t vocab_shard,
                                     int64_t row_stride, int64_t vocab_offset, int64_t vocab_total,
                                     const int32_t* d_history, int64_t history_stride,
                                     const int32_t* d_history_count, const float* d_uniform,
                                     int32_t* d_out_tokens, uint32_t* d_out_flags, void* stream) {
    int32_t rc = validate_common(ctx, cfg, d_logits_shard, dtype, batch, vocab_shard, row_stride, d_history,
                                 history_stride, d_history_count, d_out_tokens);
    if (rc != VDXS_OK) return rc;
    if (!comm) return fail(ctx, VDXS_E_INVALID_ARG, "communicator is NULL");
    if (comm->aborted) return fail(ctx, VDXS_E_NCCL, "the communicator was aborted; create a new one");
    if ((rc = vdxs_comm_status(comm)) != VDXS_OK) {
        comm_abort(comm);
        return fail(ctx, rc, "%s (nothing was launched); the communicator was aborted", vdxs_last_error(ctx));
    }
    if (vocab_offset < 0 || vocab_total < vocab_offset + vocab_shard || vocab_total > INT32_MAX)
        return fail(ctx, VDXS_E_INVALID_ARG, "shard [%lld, %lld) does not fit vocab_total %lld",
                    (long long)vocab_offset, (long long)(vocab_offset + vocab_shard), (long long)vocab_total);
    SampleArgs a;
    if ((rc = resolve_config(ctx, cfg, vocab_total, &a)) != VDXS_OK) return rc;
    if (a.path == kFull)
        return fail(ctx, VDXS_E_UNSUPPORTED, "the vocab-sharded path needs 0 < top_k < vocab_total or temperature 0");
    if (a.path == kTopK && a.K > kMaxTopK)
        return fail(ctx, VDXS_E_UNSUPPORTED, "the vocab-sharded path serves top_k <= %d (got %d)", kMaxTopK, a.K);
    if (a.path != kGreedy && !d_uniform)
        return fail(ctx, VDXS_E_INVALID_ARG, "uniform pointer is NULL but temperature != 0");
    NcclApi& n = nccl();
    if (!n.ok) return fail(ctx, VDXS_E_NCCL, "libnccl.so.2 could not be loaded");
    a.logits = d_logits_shard;
    a.dtype = dtype;
    a.B = batch;
    a.V = vocab_shard;
    a.stride = row_stride;
    a.penalty_on = cfg->repeat_penalty != 1.0f && d_history != nullptr && d_history_count != nullptr;
    a.hist = d_history;
    a.hist_stride = history_stride;
    a.hist_count = d_history_count;
    a.uniform = d_uniform;
    a.tokens = d_out_tokens;
    a.flags = d_out_flags;
    a.tie_mode = VDXS_TIES_CANONICAL;
    a.vocab_offset = vocab_offset;
    a.vocab_total = vocab_total;
    a.local_emit = true;
    a.stream = (cudaStream_t)stream;
    attach_diagnostics(ctx, &a);
    DeviceGuard g(ctx->device);
    LaunchPlan plan;
    std::string msg;
    cudaError_t e = plan_topk(a, ctx->smem_optin, &plan, &msg);
    if (e != cudaSuccess) return fail(ctx, VDXS_E_UNSUPPORTED, "%s", msg.c_str());
    if ((e = ensure_workspace(ctx->ws, a, plan, comm->nranks, a.stream, &msg)) != cudaSuccess)
        return cuda_fail(ctx, e, "workspace");
    if ((e = launch_sample(a, plan, ctx->ws, &msg)) != cudaSuccess) return cuda_fail(ctx, e, "local select launch");
    const size_t words = (size_t)batch * (size_t)(a.K + 1) * 2;
    ncclResult_t r = n.AllGather(ctx->ws.shard_send, ctx->ws.shard_recv, words, ncclUint32, comm->comm, a.stream);
    if (r == ncclInProgress) {
        // Non-blocking communicator: wait (under the deadline) until the enqueue is done.
        if ((rc = comm_settle(comm, "ncclAllGather enqueue")) != VDXS_OK) return rc;
    } else if (r != ncclSuccess) {
        comm_abort(comm);
        return fail(ctx, VDXS_E_NCCL, "ncclAllGather: %s; the communicator was aborted", n.GetErrorString(r));
    }
    if ((e = launch_merge_draw(a, comm->nranks, ctx->ws, &msg)) != cudaSuccess)
        return cuda_fail(ctx, e, "merge launch");
    ok(ctx);
    return VDXS_OK;
}

}  // extern "C"

// ---------------------------------------------------------------------------------
// Unembedding: TVdxModel.UnembedToLogits (Model.pas:1258-1271) with the tied Q4_0
// embedding matvec of shaders/matvec_q4_0.comp (:45-88), in front of the sampler.
// ---------------------------------------------------------------------------------
struct vdxs_q4_0_weights {
    int device = 0;
    int in_dim = 0;
    int out_dim = 0;
    uint32_t* nib = nullptr;
    uint16_t* scales = nullptr;
};

extern "C" {

VDXS_API int32_t vdxs_q4_0_prepare(vdxs_context* ctx, const void* d_q4_0, int32_t in_dim, int32_t out_dim,
                                   void* stream, vdxs_q4_0_weights** out) {
    if (!ctx) return fail(nullptr, VDXS_E_INVALID_ARG, "context is NULL");
    if (!d_q4_0 || !out) return fail(ctx, VDXS_E_INVALID_ARG, "weights or output pointer is NULL");
    *out = nullptr;
    if (in_dim <= 0 || (in_dim % 32) != 0)
        return fail(ctx, VDXS_E_INVALID_ARG, "in_dim %d is not a positive multiple of 32 (Q4_0 blocks)", in_dim);
    if (out_dim <= 0) return fail(ctx, VDXS_E_INVALID_ARG, "out_dim must be >= 1 (got %d)", out_dim);
    if (unembed_chunk_rows(in_dim) < 1)
        return fail(ctx, VDXS_E_UNSUPPORTED, "in_dim %d: one input vector does not fit the matvec's shared memory",
                    in_dim);
    DeviceGuard g(ctx->device);
    auto* w = new vdxs_q4_0_weights();
    w->device = ctx->device;
    w->in_dim = in_dim;
    w->out_dim = out_dim;
    const size_t nw = (size_t)q4_0_words_per_lane(in_dim);
    cudaError_t e = cudaMalloc((void**)&w->nib, (size_t)out_dim * nw * 32 * sizeof(uint32_t));
    if (e == cudaSuccess) e = cudaMalloc((void**)&w->scales, (size_t)out_dim * nw * 8 * sizeof(uint16_t));
    if (e == cudaSuccess) e = q4_0_repack((const uint8_t*)d_q4_0, in_dim, out_dim, w->nib, w->scales, (cudaStream_t)stream);
    if (e == cudaSuccess) e = cudaStreamSynchronize((cudaStream_t)stream);
    if (e != cudaSuccess) {
        cudaFree(w->nib);
        cudaFree(w->scales);
        delete w;
        return e == cudaErrorMemoryAllocation ? fail(ctx, VDXS_E_NO_MEMORY, "Q4_0 weight allocation failed")
                                              : cuda_fail(ctx, e, "Q4_0 repack");
    }
    ctx->launches += 1;
    *out = w;
    ok(ctx);
    return VDXS_OK;
}

VDXS_API int32_t vdxs_q4_0_release(vdxs_q4_0_weights* w) {
    if (!w) return VDXS_OK;
    DeviceGuard g(w->device);
    cudaFree(w->nib);
    cudaFree(w->scales);
    delete w;
    return VDXS_OK;
}

VDXS_API int32_t vdxs_unembed_q4_0(vdxs_context* ctx, const vdxs_q4_0_weights* w, const float* d_hidden,
                                   int32_t batch, float* d_logits, void* stream) {
    if (!ctx) return fail(nullptr, VDXS_E_INVALID_ARG, "context is NULL");
    if (!w || !d_hidden || !d_logits) return fail(ctx, VDXS_E_INVALID_ARG, "weights, hidden or logits pointer is NULL");
    if (batch < 1) return fail(ctx, VDXS_E_INVALID_ARG, "batch must be >= 1 (got %d)", batch);
    if (w->device != ctx->device)
        return fail(ctx, VDXS_E_INVALID_ARG, "weights live on device %d, the context on device %d", w->device,
                    ctx->device);
    DeviceGuard g(ctx->device);
    int launches = 0;
    cudaError_t e = q4_0_matvec(w->nib, w->scales, w->in_dim, w->out_dim, d_hidden, batch, d_logits,
                                (cudaStream_t)stream, &launches);
    ctx->launches += launches;
    if (e != cudaSuccess) return cuda_fail(ctx, e, "unembedding matvec");
    ok(ctx);
    return VDXS_OK;
}

VDXS_API int32_t vdxs_sample_unembed_q4_0(vdxs_context* ctx, const vdxs_config* cfg, const vdxs_q4_0_weights* w,
                                          const float* d_hidden, int32_t batch, const int32_t* d_history,
                                          int64_t history_stride, const int32_t* d_history_count,
                                          const float* d_uniform, int32_t* d_out_tokens, void* stream) {
    if (!ctx) return fail(nullptr, VDXS_E_INVALID_ARG, "context is NULL");
    if (!w) return fail(ctx, VDXS_E_INVALID_ARG, "weights pointer is NULL");
    if (batch < 1) return fail(ctx, VDXS_E_INVALID_ARG, "batch must be >= 1 (got %d)", batch);
    DeviceGuard g(ctx->device);
    // The logits stay in a context buffer; for decode batches they are still in L2 when
    // the sampler streams them.
    cudaError_t e = grow_dev(&ctx->ws.unembed_logits, &ctx->ws.unembed_cap, (size_t)batch * (size_t)w->out_dim,
                             (cudaStream_t)stream);
    if (e != cudaSuccess) return fail(ctx, VDXS_E_NO_MEMORY, "logits buffer allocation failed");
    int32_t rc = vdxs_unembed_q4_0(ctx, w, d_hidden, batch, ctx->ws.unembed_logits, stream);
    if (rc != VDXS_OK) return rc;
    return vdxs_sample_ex(ctx, cfg, ctx->ws.unembed_logits, VDXS_DTYPE_F32, batch, w->out_dim, w->out_dim, d_history,
                          history_stride, d_history_count, d_uniform, d_out_tokens, nullptr, nullptr, nullptr, 0,
                          stream);
}

}  // extern "C"

// vdxs_internal.h - declarations shared by the C-ABI layer (vdxs_api.cpp) and the
// sm_100a kernels (vdxs_kernels.cu). Not part of the public ABI.
#pragma once

#include <cstdint>
#include <string>

#include <cuda_runtime.h>

namespace vdxs {

constexpr int kThreads = 256;        // threads per CTA in every sampling kernel
constexpr int kMaxTopK = 1024;       // largest top_k served by the stream path (larger: the large top-k kernel)
constexpr int kMaxHistory = 8192;    // largest history stride served by the penalty prep
constexpr int kFaithfulSub = 512;    // elements per sub-tile of the min-buffer emulation
constexpr int kFaithfulSlots = 12;  // candidate regions of the min-buffer emulation, in units of kFaithfulSub entries
constexpr int kTauStride = 32;       // words between rows of the stream path's row bounds (one L2 line)

enum Path : int { kGreedy = 0, kTopK = 1, kFull = 2 };

// Unembedding matvec (vdxs_unembed.cu): input rows per launch and their shared memory.
constexpr int kMaxUnembedBatch = 8;
constexpr size_t kUnembedSmemBytes = 200 * 1024;

// Device workspace owned by a context (TVdxSampler.EnsureWorkspace analogue,
// Sampler.pas:250-263). Grown on demand; never shrunk until the context dies.
struct Workspace {
    uint2* cand = nullptr;          // stage-1 (key, index) candidates: [rows * cand_cap] (stream path)
    size_t cand_cap = 0;            // elements
    uint32_t* rhist = nullptr;      // [rows * kRowHistWords] stream path key histograms, self-resetting
    size_t rhist_cap = 0;
    uint32_t* row_cnt = nullptr;    // [rows] stream path list counts, self-resetting
    size_t row_cnt_cap = 0;
    unsigned long long* unit_next = nullptr;  // [2] stream path slot claims and finished warps, self-resetting
    uint32_t* row_counter = nullptr;  // [rows] completion counters, self-resetting
    size_t row_counter_cap = 0;
    uint32_t* row_tau = nullptr;      // [rows * kTauStride] stream path K-th key bounds, self-resetting
    size_t row_tau_cap = 0;
    int32_t* pen_ids = nullptr;     // [rows * pen_stride] sorted unique history ids
    float* pen_vals = nullptr;      // [rows * pen_stride] penalised values
    int32_t* pen_cnt = nullptr;     // [rows]
    uint32_t* pen_bits = nullptr;   // [rows * ceil(vocab / 32)] stream path penalised-id bitmaps, self-resetting
    size_t pen_bits_cap = 0;
    size_t pen_cap = 0;             // rows * pen_stride
    size_t pen_rows_cap = 0;
    uint32_t* fmax = nullptr;       // [rows * nchunks] full path: chunk max keys
    double* fsum = nullptr;         // [rows * nchunks] full path: chunk sums
    size_t full_cap = 0;
    uint2* shard_send = nullptr;    // [rows * K] sharded: local candidates
    uint2* shard_recv = nullptr;    // [ranks * rows * K]
    size_t shard_send_cap = 0, shard_recv_cap = 0;
    uint64_t* lk_buf = nullptr;     // top_k above the stream path's maximum: per-CTA sort buffers and slots
    size_t lk_cap = 0;              // 64-bit words
    float* unembed_logits = nullptr;  // vdxs_sample_unembed_q4_0: [rows * vocab] logits
    size_t unembed_cap = 0;
    int32_t* err = nullptr;         // device error word (0 = ok)
    // host-buffer entry point staging
    void* d_logits = nullptr;
    size_t d_logits_cap = 0;
    int32_t* d_hist = nullptr;
    size_t d_hist_cap = 0;
    int32_t* d_hcnt = nullptr;
    float* d_unif = nullptr;
    int32_t* d_tok = nullptr;
    size_t d_rows_cap = 0;
    int32_t* h_tok_pinned = nullptr;
};

// Everything one sampling call needs, already validated by the API layer.
struct SampleArgs {
    const void* logits = nullptr;
    int dtype = 0;
    int B = 0;
    int V = 0;                       // local vocab (the shard size when sharded)
    int64_t stride = 0;              // elements between rows
    const int32_t* hist = nullptr;
    int64_t hist_stride = 0;
    const int32_t* hist_count = nullptr;
    const float* uniform = nullptr;
    int32_t* tokens = nullptr;
    uint32_t* flags = nullptr;
    int32_t* out_idx = nullptr;
    float* out_prob = nullptr;
    int out_k = 0;
    // resolved configuration
    int path = kGreedy;
    int K = 1;
    float inv_temp = 1.0f;
    float min_p = 0.0f;
    float top_p = 1.0f;
    float penalty = 1.0f;
    bool penalty_on = false;
    int tie_mode = 0;
    // sharding
    int64_t vocab_offset = 0;
    int64_t vocab_total = 0;
    bool local_emit = false;         // emit local top-K candidates instead of drawing
    cudaStream_t stream = nullptr;
    // diagnostics
    cudaEvent_t ev_begin = nullptr;  // recorded just before the dominant pass
    cudaEvent_t ev_end = nullptr;    // recorded just after it
    int64_t* launches = nullptr;     // incremented per kernel launch
};

struct LaunchPlan {
    int chunk = 0;    // full path: elements per CTA; cluster path: elements per CTA of a row
    int nchunks = 0;  // chunks per row (full-softmax path: CTAs per row)
    int span = 1;     // cluster path: bytes of the staged row chunk
    int nspans = 0;   // stream paths: stage-1 pieces per row
    int elems = 32;   // stream path: warp list registers R (0 = wide stream path)
    bool stream = false;  // top-k path: persistent stream kernel + finish kernel
    bool cluster = false; // top-k path, small batches: one thread-block cluster per row
    bool large = false;   // top-k path, top_k above kMaxTopK: one CTA per row, global workspace
    int large_grid = 0;   // large top-k kernel grid (CTAs)
    size_t large_smem = 0;  // large top-k kernel shared memory
    int cluster_ctas = 8; // CTAs per cluster
    int grid = 0;         // stream kernel grid (CTAs)
    int cand_cap = 0;     // top-k path: candidates each stage-1 list may hold (stream path: per row)
    int gather_cap = 0;   // stream path: finish kernel gather capacity
    long long items = 0;  // top-k path: stage-1 candidate lists
    int slots = 0;        // stream path: 4 KB slots per row
    int unit_slots = 0;   // stream path: slots per claimed unit
    size_t smem = 0;
    size_t smem2 = 0;     // finish kernel shared memory
};

// Host-side launchers (vdxs_kernels.cu). Return cudaSuccess or the launch error;
// `err` receives a message for argument/capacity problems (returned as
// cudaErrorInvalidValue).
cudaError_t plan_topk(const SampleArgs& a, int device_smem_optin, LaunchPlan* plan, std::string* err);
cudaError_t plan_full(const SampleArgs& a, LaunchPlan* plan, std::string* err);
cudaError_t ensure_workspace(Workspace& ws, const SampleArgs& a, const LaunchPlan& plan, int ranks,
                             cudaStream_t stream, std::string* err);
cudaError_t launch_sample(const SampleArgs& a, const LaunchPlan& plan, Workspace& ws, std::string* err);
cudaError_t launch_merge_draw(const SampleArgs& a, int ranks, Workspace& ws, std::string* err);
// Unembedding (vdxs_unembed.cu): Q4_0 repack and the matvec in the reference shader's order.
int q4_0_words_per_lane(int in_dim);
size_t q4_0_packed_bytes(int in_dim, int out_dim);
int unembed_chunk_rows(int in_dim);
cudaError_t q4_0_repack(const uint8_t* src, int in_dim, int out_dim, uint32_t* nib, uint16_t* scales,
                        cudaStream_t stream);
cudaError_t q4_0_matvec(const uint32_t* nib, const uint16_t* scales, int in_dim, int out_dim, const float* x,
                        int batch, float* out, cudaStream_t stream, int* launches);
// Device-resident decode state (one thread per row).
cudaError_t launch_device_uniforms(uint64_t* prng, int batch, float* out, cudaStream_t stream);
cudaError_t launch_history_push(int32_t* hist, int32_t* pos, int32_t* count, int window, const int32_t* tokens,
                                int batch, const int32_t* stop_ids, int n_stop, int32_t* stopped,
                                cudaStream_t stream);
void free_workspace(Workspace& ws);
// Clears the device error word and the self-resetting counters (after a failed launch).
cudaError_t reset_device_state(Workspace& ws, cudaStream_t stream);

// Fixed device scratch used by vdxs_sample_noalloc (no allocation on any call).
constexpr size_t kNoAllocScratchBytes = (size_t)32 << 20;
// Byte offset of the device error word inside that array (the first field carved).
constexpr size_t kNoAllocErrOffset = 0;
// Device address of the scratch on the current device (resolved once per device) and
// that device's opt-in shared-memory limit.
cudaError_t noalloc_scratch(void** ptr, int* smem_optin);
// Lays out the workspace of one call inside [base, base + cap) without allocating.
// Returns the bytes the call needs; the pointers are set only when it fits.
size_t carve_workspace(Workspace& ws, unsigned char* base, size_t cap, const SampleArgs& a, const LaunchPlan& plan);

}  // namespace vdxs

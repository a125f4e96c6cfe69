// vdxs_kernels.cu - sm_100a kernels of the token sampler.
//
// Hot path: TVdxSampler.Process (src/VindexLLM.Sampler.pas:265-528) for a batch of
// [B, V] device-resident logits.
//
//   penalty_prep_kernel   Sampler.pas:285-303  history ids -> sorted unique (id, f^n(x))
//   topk_stream_kernel    Sampler.pas:305-383  top_k <= 1024 and greedy: one 16-warp CTA
//                         per SM; warps claim row segments from a global counter, stream
//                         them through per-warp bulk-copy rings, filter against a per-row
//                         bound taken from a shared key histogram, and append candidates
//                         to one list per row.
//   topk_large_kernel     1024 < top_k < V: one CTA per row, radix select over the row in
//                         global memory, a single-CTA radix sort of the K survivors, the
//                         reference's sequential walk; faithful rows re-run the min-buffer
//                         with a tournament tree (vdxs_large_topk.cuh).
//   finish_kernel         Sampler.pas:305-459  one CTA per row (programmatic dependent
//                         launch): gathers the candidates at the row's bound plus the
//                         penalised history entries, selects the exact top-K, then exp /
//                         min-p / sort / top-p / draw. Rows whose token depends on the
//                         reference's min-buffer slot order are re-resolved in the same
//                         CTA by an exact emulation of the scan (faithful mode).
//   row_cluster_kernel    batches of at most 8 rows: one 8-CTA cluster per row, the row
//                         staged in shared memory, candidates sent to the leader CTA
//                         through distributed shared memory; the leader finishes.
//   full_max_kernel,      Sampler.pas:461-527  full-softmax path: max pass, then an
//   full_sum_kernel       exp/sum pass whose last CTA per row locates the draw.
//   merge_draw_kernel     vocab-sharded path: merge the all-gathered candidates, draw.
//
// Ordering: every top-k decision uses the composite order (value desc, index asc) on
// order-preserving 32-bit keys of the fp32 value (-0 folded onto +0), so ties go to
// the lowest index. Probabilities are computed as the reference stores them:
// Single((x - max) * invT evaluated in Double, exp in Double).
#include "vdxs_internal.h"
#include "../../include/vdx_sampler.h"

#include <cuda_runtime.h>
#include <cooperative_groups.h>
#include <algorithm>
#include <climits>
#include <cstdint>
#include <cstdio>
#include <cstdlib>
#include <mutex>
#include <string>

namespace vdxs {

constexpr int NT = kThreads;
constexpr int NWARPS = NT / 32;
constexpr unsigned FULL = 0xFFFFFFFFu;
constexpr int kHistBins = 464;   // log-bins of the distance to the maximum key
constexpr int kHistWords = 512;
constexpr int kShWords = 64;
constexpr size_t kHeadBytes = (kHistWords + kShWords) * 4;  // hist + scalars at smem start

enum ErrCode : int32_t { kErrNone = 0, kErrSelect = 1, kErrFaithful = 2, kErrTimeout = 3 };

// Phase timing for development builds (-DVDXS_TIMING): thread 0 of each CTA adds the
// cycles of each phase to a per-phase total. Compiled out of the library otherwise.
#ifdef VDXS_TIMING
__device__ unsigned long long g_phase_cycles[64];
__device__ unsigned long long g_phase_count[64];
#define VDXS_T0(v) long long v = clock64()
#define VDXS_T1(id, v)                                                          \
    do {                                                                        \
        if (threadIdx.x == 0) {                                                 \
            atomicAdd(&g_phase_cycles[id], (unsigned long long)(clock64() - v)); \
            atomicAdd(&g_phase_count[id], 1ull);                                \
        }                                                                       \
    } while (0)
// Adds v to counter id from the calling thread (call from one lane per warp).
#define VDXS_ADD(id, v) atomicAdd(&g_phase_cycles[id], (unsigned long long)(v))
#else
#define VDXS_ADD(id, v) \
    do {                \
    } while (0)
#define VDXS_T0(v) \
    do {           \
    } while (0)
#define VDXS_T1(id, v) \
    do {               \
    } while (0)
#endif

struct KParams {
    const void* logits;
    int64_t stride;
    int V;
    int B;
    int chunk;    // elements per chunk (top-k path: NT * keys per thread)
    int nchunks;  // full path: CTAs (chunks) per row; stream paths: pieces per row
    int span;     // cluster path: bytes of the staged row chunk
    int K;
    int path;
    // penalty list (sorted unique local ids and their penalised values); null when off
    const int32_t* pen_ids;
    const float* pen_vals;
    const int32_t* pen_cnt;
    int pen_stride;
    uint32_t* pen_bits;  // stream path: [B][pen_words] bitmap of the penalised ids (cleared by finish)
    int pen_words;
    // workspace
    uint2* cand;        // stage-1 (key, index) candidates (stream path: [B][cand_cap], one list per row)
    int cand_cap;       // candidates a list may hold
    int gather_cap;     // finish kernel: fixed gather capacity
    // Stream path: rows of flat_ng 4 KB slots, claimed in units of unit_slots slots.
    int flat_ng;
    int unit_slots;
    uint32_t* rhist;      // [B][kRowHistWords] per-row key histograms (reset by finish)
    uint32_t* row_cnt;    // [B] list counts (reset by finish)
    unsigned long long* unit_next;  // [2] slot claims and finished warps (reset by the last warp)
    uint32_t* row_counter;
    uint32_t* row_tau;  // stream path: per-row lower bound on the K-th key (reset by finish)
    int32_t* err;
    uint32_t* fmax;
    double* fsum;
    uint2* fstat;  // full path: per chunk (nonzero count, min exponent + 1024 | pmax key)
    // results
    const float* uniform;
    int32_t* tokens;
    uint32_t* flags;
    int32_t* out_idx;
    float* out_prob;
    int out_k;
    float inv_temp;
    float min_p;
    float top_p;
    int tie_mode;
    // sharding
    int64_t vocab_offset;
    int local_emit;
    uint2* emit_out;  // [B][K+1]
    // top_k above the stream path's maximum: per-CTA global workspace (lk_cta_words(K) words each)
    uint64_t* lk_buf;
    int lk_list;  // the large top-k kernel selects from stage-1 lists (the stream kernel ran first)
};

// ---------------------------------------------------------------------------------
// Keys and loads
// ---------------------------------------------------------------------------------
__device__ __forceinline__ uint32_t f2key(float f) {
    uint32_t u = __float_as_uint(f);
    if (u == 0x80000000u) u = 0u;  // -0.0 compares equal to +0.0
    return (u & 0x80000000u) ? ~u : (u | 0x80000000u);
}
__device__ __forceinline__ float key2f(uint32_t k) {
    uint32_t u = (k & 0x80000000u) ? (k & 0x7FFFFFFFu) : ~k;
    return __uint_as_float(u);
}
__device__ __forceinline__ float ld_elem(const float* p, int64_t i) { return __ldg(p + i); }
__device__ __forceinline__ float ld_elem(const uint16_t* p, int64_t i) {
    return __uint_as_float(((uint32_t)__ldg(p + i)) << 16);
}
// 128-bit streaming load; the data is read once, so it bypasses L1 allocation.
__device__ __forceinline__ uint4 ld_stream16(const void* p) {
    uint4 r;
    asm("ld.global.nc.L1::no_allocate.v4.u32 {%0,%1,%2,%3}, [%4];"
        : "=r"(r.x), "=r"(r.y), "=r"(r.z), "=r"(r.w)
        : "l"(p));
    return r;
}
template <typename T> struct VecTraits;
template <> struct VecTraits<float> { static constexpr int N = 4; };
template <> struct VecTraits<uint16_t> { static constexpr int N = 8; };

__device__ __forceinline__ void unpack(const uint4& r, float* out, float) {
    out[0] = __uint_as_float(r.x);
    out[1] = __uint_as_float(r.y);
    out[2] = __uint_as_float(r.z);
    out[3] = __uint_as_float(r.w);
}
__device__ __forceinline__ void unpack(const uint4& r, float* out, uint16_t) {
    out[0] = __uint_as_float(r.x << 16);
    out[1] = __uint_as_float(r.x & 0xFFFF0000u);
    out[2] = __uint_as_float(r.y << 16);
    out[3] = __uint_as_float(r.y & 0xFFFF0000u);
    out[4] = __uint_as_float(r.z << 16);
    out[5] = __uint_as_float(r.z & 0xFFFF0000u);
    out[6] = __uint_as_float(r.w << 16);
    out[7] = __uint_as_float(r.w & 0xFFFF0000u);
}

// Log-scale bin of the distance d = kmax - key: exact for d < 16, then 4 mantissa
// bits per power of two. Monotone in d, 464 bins.
__device__ __forceinline__ int logbin(uint32_t d) {
    if (d < 16u) return (int)d;
    int e = 31 - __clz(d);
    return 16 + ((e - 4) << 4) + (int)((d >> (e - 4)) & 15u);
}
__device__ __forceinline__ void logbin_range(int b, uint32_t* lo, int* bits) {
    if (b < 16) {
        *lo = (uint32_t)b;
        *bits = 0;
        return;
    }
    int e = ((b - 16) >> 4) + 4;
    int m = (b - 16) & 15;
    *lo = (uint32_t)(16 + m) << (e - 4);
    *bits = e - 4;
}

__device__ __forceinline__ unsigned lanemask_lt() {
    unsigned m;
    asm("mov.u32 %0, %%lanemask_lt;" : "=r"(m));
    return m;
}

// ---- 1-D TMA bulk copies (global -> shared) completed on an mbarrier ---------------
__device__ __forceinline__ uint32_t smem_u32(const void* p) { return (uint32_t)__cvta_generic_to_shared(p); }
__device__ __forceinline__ void mbar_init(uint64_t* bar, uint32_t count) {
    asm volatile("mbarrier.init.shared::cta.b64 [%0], %1;" ::"r"(smem_u32(bar)), "r"(count) : "memory");
}
__device__ __forceinline__ void fence_mbar_init() { asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory"); }
__device__ __forceinline__ void mbar_arrive_expect_tx(uint64_t* bar, uint32_t bytes) {
    asm volatile("mbarrier.arrive.expect_tx.shared::cta.b64 _, [%0], %1;" ::"r"(smem_u32(bar)), "r"(bytes)
                 : "memory");
}
// Bulk copy of `bytes` (a multiple of 16; both addresses 16-byte aligned) into this
// CTA's shared memory; completion is counted on `bar`.
// Orders this thread's earlier generic-proxy shared-memory accesses (made visible to it
// by a warp barrier for the other lanes) before its later async-proxy (bulk copy) ones.
__device__ __forceinline__ void fence_proxy_async_smem() {
    asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
}
__device__ __forceinline__ void tma_load_1d(void* dst, const void* src, uint32_t bytes, uint64_t* bar) {
    asm volatile("cp.async.bulk.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1], %2, [%3];" ::"r"(
                     smem_u32(dst)),
                 "l"(src), "r"(bytes), "r"(smem_u32(bar))
                 : "memory");
}
__device__ __forceinline__ void mbar_arrive(uint64_t* bar) {
    asm volatile("mbarrier.arrive.shared::cta.b64 _, [%0];" ::"r"(smem_u32(bar)) : "memory");
}
__device__ __forceinline__ void mbar_inval(uint64_t* bar) {
    asm volatile("mbarrier.inval.shared::cta.b64 [%0];" ::"r"(smem_u32(bar)) : "memory");
}
__device__ __forceinline__ bool mbar_try_wait(uint64_t* bar, uint32_t parity) {
    uint32_t ok;
    asm volatile(
        "{\n .reg .pred p;\n mbarrier.try_wait.parity.shared::cta.b64 p, [%1], %2;\n selp.u32 %0, 1, 0, p;\n}"
        : "=r"(ok)
        : "r"(smem_u32(bar)), "r"(parity)
        : "memory");
    return ok != 0u;
}
__device__ __forceinline__ uint32_t ld_relaxed_u32(const uint32_t* p) {
    uint32_t v;
    asm volatile("ld.relaxed.gpu.global.u32 %0, [%1];" : "=r"(v) : "l"(p) : "memory");
    return v;
}
__device__ __forceinline__ uint64_t ld_relaxed_u64(const unsigned long long* p) {
    uint64_t v;
    asm volatile("ld.relaxed.gpu.global.u64 %0, [%1];" : "=l"(v) : "l"(p) : "memory");
    return v;
}
__device__ __forceinline__ uint64_t global_ns() {
    uint64_t t;
    asm volatile("mov.u64 %0, %%globaltimer;" : "=l"(t));
    return t;
}
// Waits for phase `parity` of `bar`, giving up after about 2 s (returns false).
__device__ __forceinline__ bool mbar_wait_bounded(uint64_t* bar, uint32_t parity) {
    if (mbar_try_wait(bar, parity)) return true;
    const uint64_t t0 = global_ns();
    for (;;) {
        for (int i = 0; i < 64; ++i)
            if (mbar_try_wait(bar, parity)) return true;
        if (global_ns() - t0 > 2000000000ull) return false;
    }
}

// ---------------------------------------------------------------------------------
// Block primitives (NT threads)
// ---------------------------------------------------------------------------------
__device__ __forceinline__ uint32_t block_max_u32(uint32_t v, uint32_t* sh) {
    v = __reduce_max_sync(FULL, v);
    __syncthreads();
    if ((threadIdx.x & 31) == 0) sh[threadIdx.x >> 5] = v;
    __syncthreads();
    uint32_t r = (threadIdx.x & 31) < NWARPS ? sh[threadIdx.x & 31] : 0u;
    return __reduce_max_sync(FULL, r);
}
__device__ __forceinline__ uint32_t block_min_u32(uint32_t v, uint32_t* sh) {
    v = __reduce_min_sync(FULL, v);
    __syncthreads();
    if ((threadIdx.x & 31) == 0) sh[threadIdx.x >> 5] = v;
    __syncthreads();
    uint32_t r = (threadIdx.x & 31) < NWARPS ? sh[threadIdx.x & 31] : 0xFFFFFFFFu;
    return __reduce_min_sync(FULL, r);
}
__device__ __forceinline__ uint32_t block_sum_u32(uint32_t v, uint32_t* sh) {
    v = __reduce_add_sync(FULL, v);
    __syncthreads();
    if ((threadIdx.x & 31) == 0) sh[threadIdx.x >> 5] = v;
    __syncthreads();
    uint32_t r = (threadIdx.x & 31) < NWARPS ? sh[threadIdx.x & 31] : 0u;
    return __reduce_add_sync(FULL, r);
}
// Exclusive scan of one int per thread; *total receives the block sum.
__device__ __forceinline__ int block_excl_scan(int v, int* sh, int* total) {
    const int l = threadIdx.x & 31, w = threadIdx.x >> 5;
    int x = v;
#pragma unroll
    for (int o = 1; o < 32; o <<= 1) {
        int y = __shfl_up_sync(FULL, x, o);
        if (l >= o) x += y;
    }
    __syncthreads();
    if (l == 31) sh[w] = x;
    __syncthreads();
    if (w == 0) {
        int s = l < NWARPS ? sh[l] : 0;
#pragma unroll
        for (int o = 1; o < 32; o <<= 1) {
            int y = __shfl_up_sync(FULL, s, o);
            if (l >= o) s += y;
        }
        if (l < NWARPS) sh[l] = s;
    }
    __syncthreads();
    *total = sh[NWARPS - 1];
    return (w > 0 ? sh[w - 1] : 0) + x - v;
}
// Exclusive scan of one double per thread (sums of non-negative terms).
__device__ __forceinline__ double block_excl_scan_d(double v, double* sh, double* total) {
    const int l = threadIdx.x & 31, w = threadIdx.x >> 5;
    double x = v;
#pragma unroll
    for (int o = 1; o < 32; o <<= 1) {
        double y = __shfl_up_sync(FULL, x, o);
        if (l >= o) x += y;
    }
    __syncthreads();
    if (l == 31) sh[w] = x;
    __syncthreads();
    if (w == 0) {
        double s = l < NWARPS ? sh[l] : 0.0;
#pragma unroll
        for (int o = 1; o < 32; o <<= 1) {
            double y = __shfl_up_sync(FULL, s, o);
            if (l >= o) s += y;
        }
        if (l < NWARPS) sh[l] = s;
    }
    __syncthreads();
    *total = sh[NWARPS - 1];
    double r = (w > 0 ? sh[w - 1] : 0.0) + (x - v);
    return r;
}

// Descending bitonic sort of n (power of two) 64-bit keys in shared memory.
__device__ void bitonic_sort_desc(uint64_t* a, int n) {
    for (int k = 2; k <= n; k <<= 1) {
        for (int j = k >> 1; j > 0; j >>= 1) {
            for (int i = threadIdx.x; i < n; i += NT) {
                int ixj = i ^ j;
                if (ixj > i) {
                    uint64_t x = a[i], y = a[ixj];
                    bool desc = (i & k) == 0;
                    if (desc ? (x < y) : (x > y)) {
                        a[i] = y;
                        a[ixj] = x;
                    }
                }
            }
            __syncthreads();
        }
    }
}

__device__ __forceinline__ uint64_t shfl64_xor(uint64_t v, int m) {
    const uint32_t lo = __shfl_xor_sync(FULL, (uint32_t)v, m), hi = __shfl_xor_sync(FULL, (uint32_t)(v >> 32), m);
    return ((uint64_t)hi << 32) | lo;
}

// Bitonic sort (descending) of a[0, EPT*NT) with EPT consecutive elements per thread in
// registers: exchanges between elements of one thread stay in registers, partners in
// the same warp are reached by shuffles, and only the widest stages (partner distance
// of a warp's span or more) go through shared memory.
template <int EPT>
__device__ void block_bitonic_desc_regs(uint64_t* a) {
    constexpr int N = EPT * NT;
    const int tid = threadIdx.x;
    uint64_t v[EPT];
#pragma unroll
    for (int u = 0; u < EPT; ++u) v[u] = a[EPT * tid + u];
    for (int k = 2; k <= N; k <<= 1) {
        for (int j = k >> 1; j > 0; j >>= 1) {
            if (j >= 32 * EPT) {
                __syncthreads();
#pragma unroll
                for (int u = 0; u < EPT; ++u) a[EPT * tid + u] = v[u];
                __syncthreads();
#pragma unroll
                for (int u = 0; u < EPT; ++u) {
                    const int i = EPT * tid + u;
                    const uint64_t y = a[i ^ j];
                    const bool hi = ((i & k) == 0) == (i < (i ^ j));  // keep the larger
                    v[u] = hi ? max(v[u], y) : min(v[u], y);
                }
            } else if (j >= EPT) {
#pragma unroll
                for (int u = 0; u < EPT; ++u) {
                    const int i = EPT * tid + u;
                    const uint64_t y = shfl64_xor(v[u], j / EPT);
                    const bool hi = ((i & k) == 0) == (i < (i ^ j));
                    v[u] = hi ? max(v[u], y) : min(v[u], y);
                }
            } else {
                // Partner in this thread; jj is a compile-time copy of j, so v stays in
                // registers.
#pragma unroll
                for (int jj = 1; jj < EPT; jj <<= 1) {
                    if (jj == j) {
#pragma unroll
                        for (int u = 0; u < EPT; ++u) {
                            if ((u & jj) == 0) {
                                const int i = EPT * tid + u;
                                const uint64_t x = v[u], y = v[u ^ jj];
                                const bool desc = (i & k) == 0;
                                v[u] = desc ? max(x, y) : min(x, y);
                                v[u ^ jj] = desc ? min(x, y) : max(x, y);
                            }
                        }
                    }
                }
            }
        }
    }
    __syncthreads();
#pragma unroll
    for (int u = 0; u < EPT; ++u) a[EPT * tid + u] = v[u];
    __syncthreads();
}

// Descending sort of a[0, n) (n <= P2, a power of two) where a[0, nvalid) are distinct
// non-zero keys and a[nvalid, P2) are zero. Up to NT keys: each thread's rank among the
// valid keys is its position (two barriers); 512 and 1024 keys: the register bitonic
// network; above that, the shared-memory one.
__device__ void block_sort_desc_distinct(uint64_t* a, int nvalid, int P2) {
    if (P2 == 2 * NT) {
        block_bitonic_desc_regs<2>(a);
        return;
    }
    if (P2 == 4 * NT) {
        block_bitonic_desc_regs<4>(a);
        return;
    }
    if (P2 > NT) {
        bitonic_sort_desc(a, P2);
        return;
    }
    const int tid = threadIdx.x;
    const uint64_t mine = tid < nvalid ? a[tid] : 0ull;
    int rank = 0;
    if (tid < nvalid)
        for (int j = 0; j < nvalid; ++j) rank += a[j] > mine ? 1 : 0;
    __syncthreads();
    if (tid < nvalid) a[rank] = mine;
    __syncthreads();
}

// Warp 0 only: first bin g of hist[0..nb) whose inclusive prefix reaches `need`.
// Writes sh[0] = g (or -1), sh[1] = count before g, sh[2] = total.
__device__ void warp_find(const uint32_t* hist, int nb, uint32_t need, uint32_t* sh) {
    const int l = threadIdx.x & 31;
    const int seg = (nb + 31) >> 5;
    const int b0 = min(l * seg, nb), b1 = min(b0 + seg, nb);
    uint32_t s = 0;
    for (int b = b0; b < b1; ++b) s += hist[b];
    uint32_t incl = s;
#pragma unroll
    for (int o = 1; o < 32; o <<= 1) {
        uint32_t y = __shfl_up_sync(FULL, incl, o);
        if (l >= o) incl += y;
    }
    const uint32_t total = __shfl_sync(FULL, incl, 31);
    const unsigned m = __ballot_sync(FULL, incl >= need);
    if (m == 0u) {
        if (l == 0) {
            sh[0] = 0xFFFFFFFFu;
            sh[1] = total;
        }
    } else {
        const int L = __ffs(m) - 1;
        if (l == L) {
            uint32_t c = incl - s;
            int g = b0;
            for (; g < b1; ++g) {
                if (c + hist[g] >= need) break;
                c += hist[g];
            }
            sh[0] = (uint32_t)g;
            sh[1] = c;
        }
    }
    if (l == 0) sh[2] = total;
}

// ---------------------------------------------------------------------------------
// Block top-K select on (key desc, tb asc). Keys equal to 0 are invalid and ignored.
// Finds the K-th best element; the caller emits every element that is not worse.
// ---------------------------------------------------------------------------------
struct SelectOut {
    uint32_t kth_key;  // 0 = every valid element is selected
    uint32_t kth_tb;
    uint32_t n_valid;
    int tie_cut;       // elements equal to kth_key were left out
};

struct SmemKeySrc {  // stage 1: keys in shared memory, tie-break = position
    const uint32_t* k;
    __device__ __forceinline__ uint32_t key(int i) const { return k[i]; }
    __device__ __forceinline__ uint32_t tb(int i) const { return (uint32_t)i; }
};
struct SmemPairSrc {  // stage 2: (key, index) pairs in shared memory, tie-break = index
    const uint32_t* k;
    const uint32_t* t;
    __device__ __forceinline__ uint32_t key(int i) const { return k[i]; }
    __device__ __forceinline__ uint32_t tb(int i) const { return t[i]; }
};

template <class Src>
__device__ SelectOut block_select(const Src& src, int n, int K, uint32_t kmax, int tb_bits,
                                  uint32_t* hist, uint32_t* sh) {
    const int tid = threadIdx.x;
    SelectOut r;
    r.tie_cut = 0;
    for (int i = tid; i < kHistBins; i += NT) hist[i] = 0u;
    __syncthreads();
    // Every pass loads four elements per thread before it counts them, so that reads
    // from global memory (a row source) overlap.
    for (int i0 = tid; i0 < n; i0 += 4 * NT) {
        uint32_t k[4];
#pragma unroll
        for (int u = 0; u < 4; ++u) k[u] = i0 + u * NT < n ? src.key(i0 + u * NT) : 0u;
#pragma unroll
        for (int u = 0; u < 4; ++u)
            if (k[u]) atomicAdd(&hist[logbin(kmax - k[u])], 1u);
    }
    __syncthreads();
    if (tid < 32) warp_find(hist, kHistBins, (uint32_t)K, sh);
    __syncthreads();
    const uint32_t total = sh[2];
    r.n_valid = total;
    if (total <= (uint32_t)K) {
        r.kth_key = 0u;
        r.kth_tb = 0xFFFFFFFFu;
        __syncthreads();
        return r;
    }
    const int g0 = (int)sh[0];
    uint32_t need = (uint32_t)K - sh[1];
    uint32_t dlo;
    int bits;
    logbin_range(g0, &dlo, &bits);
    uint32_t n_eq = hist[g0];
    __syncthreads();
    while (bits > 0) {
        const int w = bits < 8 ? bits : 8;
        const int shift = bits - w;
        const uint32_t width = 1u << bits;
        for (int i = tid; i < 256; i += NT) hist[i] = 0u;
        __syncthreads();
        for (int i0 = tid; i0 < n; i0 += 4 * NT) {
            uint32_t k[4];
#pragma unroll
            for (int u = 0; u < 4; ++u) k[u] = i0 + u * NT < n ? src.key(i0 + u * NT) : 0u;
#pragma unroll
            for (int u = 0; u < 4; ++u) {
                const uint32_t dd = (kmax - k[u]) - dlo;
                if (k[u] && dd < width) atomicAdd(&hist[dd >> shift], 1u);
            }
        }
        __syncthreads();
        if (tid < 32) warp_find(hist, 1 << w, need, sh);
        __syncthreads();
        const int g = (int)sh[0];
        const uint32_t before = sh[1];
        n_eq = hist[g];
        __syncthreads();
        dlo += (uint32_t)g << shift;
        need -= before;
        bits = shift;
    }
    r.kth_key = kmax - dlo;
    if (need == n_eq) {
        r.kth_tb = 0xFFFFFFFFu;
        return r;
    }
    r.tie_cut = 1;
    // The `need` lowest tie-breaks among elements whose key equals kth_key.
    uint32_t tlo = 0u;
    int tbits = tb_bits;
    while (tbits > 0) {
        const int w = tbits < 8 ? tbits : 8;
        const int shift = tbits - w;
        const uint32_t hi_mask = tbits >= 32 ? 0u : (0xFFFFFFFFu << tbits);
        for (int i = tid; i < 256; i += NT) hist[i] = 0u;
        __syncthreads();
        for (int i0 = tid; i0 < n; i0 += 4 * NT) {
            bool eq[4];
#pragma unroll
            for (int u = 0; u < 4; ++u) eq[u] = i0 + u * NT < n && src.key(i0 + u * NT) == r.kth_key;
#pragma unroll
            for (int u = 0; u < 4; ++u) {
                if (eq[u]) {
                    const uint32_t t = src.tb(i0 + u * NT);
                    if (((t ^ tlo) & hi_mask) == 0u) atomicAdd(&hist[(t >> shift) & ((1u << w) - 1u)], 1u);
                }
            }
        }
        __syncthreads();
        if (tid < 32) warp_find(hist, 1 << w, need, sh);
        __syncthreads();
        const int g = (int)sh[0];
        const uint32_t before = sh[1];
        __syncthreads();
        tlo |= (uint32_t)g << shift;
        need -= before;
        tbits = shift;
    }
    r.kth_tb = tlo;
    return r;
}

__device__ __forceinline__ bool selected(uint32_t k, uint32_t t, const SelectOut& s) {
    return k != 0u && (k > s.kth_key || (k == s.kth_key && t <= s.kth_tb));
}

__device__ __forceinline__ int bits_for(uint32_t maxval) { return maxval == 0u ? 1 : 32 - __clz(maxval); }

// Binary search in a sorted id list: index of the first element >= v.
__device__ __forceinline__ int lower_bound_i32(const int32_t* a, int n, int64_t v) {
    int lo = 0, hi = n;
    while (lo < hi) {
        int mid = (lo + hi) >> 1;
        if ((int64_t)a[mid] < v) lo = mid + 1;
        else hi = mid;
    }
    return lo;
}

// ---------------------------------------------------------------------------------
// Penalty prep (Sampler.pas:285-303): per row, the history ids that fall in
// [vocab_offset, vocab_offset + V) are sorted, deduplicated, and each distinct id gets
// f^n(x) where n is its multiplicity and f(x) = x>0 ? x/p : (x<0 ? x*p : x) in fp32.
// ---------------------------------------------------------------------------------
template <typename T>
__global__ void __launch_bounds__(NT) penalty_prep_kernel(const T* logits, int64_t stride, int V,
                                                          int64_t lo, const int32_t* hist,
                                                          int64_t hist_stride,
                                                          const int32_t* hist_count, float penalty,
                                                          int32_t* pen_ids, float* pen_vals,
                                                          int32_t* pen_cnt, int pen_stride, uint32_t* pen_bits,
                                                          int pen_words) {
    extern __shared__ __align__(16) unsigned char smem_raw[];
    int32_t* a = (int32_t*)smem_raw;  // [P2]
    __shared__ int sh[NWARPS + 1];
    const int b = blockIdx.x, tid = threadIdx.x;
    int cnt = hist_count[b];
    cnt = cnt < 0 ? 0 : cnt;
    if (cnt > pen_stride) cnt = pen_stride;
    int P2 = 1;
    while (P2 < cnt) P2 <<= 1;
    const int32_t* h = hist + (int64_t)b * hist_stride;
    for (int i = tid; i < P2; i += NT) {
        int32_t v = INT_MAX;
        if (i < cnt) {
            int64_t local = (int64_t)h[i] - lo;
            if (local >= 0 && local < V) v = (int32_t)local;
        }
        a[i] = v;
    }
    __syncthreads();
    for (int k = 2; k <= P2; k <<= 1)
        for (int j = k >> 1; j > 0; j >>= 1) {
            for (int i = tid; i < P2; i += NT) {
                int ixj = i ^ j;
                if (ixj > i) {
                    int32_t x = a[i], y = a[ixj];
                    bool asc = (i & k) == 0;
                    if (asc ? (x > y) : (x < y)) {
                        a[i] = y;
                        a[ixj] = x;
                    }
                }
            }
            __syncthreads();
        }
    // Each thread owns a contiguous segment so the output keeps ascending id order.
    const int seg = (P2 + NT - 1) / NT;
    const int s0 = min(tid * seg, P2), s1 = min(s0 + seg, P2);
    int firsts = 0;
    for (int i = s0; i < s1; ++i)
        if (a[i] != INT_MAX && (i == 0 || a[i - 1] != a[i])) ++firsts;
    int total;
    int off = block_excl_scan(firsts, sh, &total);
    const T* row = logits + (int64_t)b * stride;
    const float p = penalty;
    for (int i = s0; i < s1; ++i) {
        int32_t id = a[i];
        if (id == INT_MAX || (i > 0 && a[i - 1] == id)) continue;
        int n = 1;
        while (i + n < P2 && a[i + n] == id) ++n;
        float v = ld_elem(row, id);
        for (int r = 0; r < n; ++r) {
            if (v > 0.0f) v = __fdiv_rn(v, p);
            else if (v < 0.0f) v = __fmul_rn(v, p);
        }
        pen_ids[(int64_t)b * pen_stride + off] = id;
        pen_vals[(int64_t)b * pen_stride + off] = v;
        if (pen_bits) atomicOr(&pen_bits[(int64_t)b * pen_words + (id >> 5)], 1u << (id & 31));
        ++off;
    }
    if (tid == 0) pen_cnt[b] = total;
    // Stage 1 may be launched as a programmatic dependent of this kernel (it waits for
    // the whole grid before it reads the lists). The trigger comes after this CTA's
    // work, so no CTA of this grid is left waiting for an SM held by stage 1.
    asm volatile("griddepcontrol.launch_dependents;" ::: "memory");
}

// ---------------------------------------------------------------------------------
// Stage 2, canonical: survivors sk/si (nsel of them, nsel <= K <= 1024) -> exp,
// min-p, sort by (prob desc, index asc), top-p, draw. Returns true when the row has to
// be re-resolved by the faithful emulation (token not written in that case).
// `work` must hold 24 * 1024 + 8 bytes.
// ---------------------------------------------------------------------------------
__device__ bool stage2_canonical(const KParams& p, int b, const uint32_t* sk, const uint32_t* si,
                                 int nsel, uint32_t kmax, uint32_t kth_key, uint32_t flags_in,
                                 unsigned char* work, uint32_t* shu, uint32_t* flags_out) {
    __shared__ double s_dsh[NWARPS];
    __shared__ double s_d[4];
    __shared__ int s_i[4];
    const int tid = threadIdx.x;
    int P2 = 32;
    while (P2 < nsel) P2 <<= 1;
    uint64_t* sortb = (uint64_t*)work;
    float* q = (float*)(sortb + P2);
    int32_t* qid = (int32_t*)(q + P2);
    double* pre = (double*)(qid + P2);  // [P2 + 1]

    VDXS_T0(t_e);
    const float M = key2f(kmax);
    const double Md = (double)M, it = (double)p.inv_temp;
    for (int s = tid; s < P2; s += NT) q[s] = s < nsel ? (float)exp(((double)key2f(sk[s]) - Md) * it) : 0.0f;
    __syncthreads();
    // Probability of the boundary value (the k-th largest); when more elements share it
    // than fit, the reference's survivor among them depends on its slot history.
    float qb = kth_key ? (float)exp(((double)key2f(kth_key) - Md) * it) : -1.0f;
    if (p.min_p > 0.0f) {
        uint32_t mk = 0u;
        for (int s = tid; s < nsel; s += NT) mk = max(mk, f2key(q[s]));
        mk = block_max_u32(mk, shu);
        const float thr = __fmul_rn(key2f(mk), p.min_p);
        for (int s = tid; s < nsel; s += NT)
            if (q[s] < thr) q[s] = 0.0f;
        if (qb >= 0.0f && qb < thr) qb = 0.0f;
        __syncthreads();
    }
    for (int s = tid; s < P2; s += NT)
        sortb[s] = s < nsel ? (((uint64_t)__float_as_uint(q[s]) << 32) | (uint64_t)(~si[s])) : 0ull;
    __syncthreads();
    VDXS_T1(1, t_e);
    VDXS_T0(t_so);
    block_sort_desc_distinct(sortb, nsel, P2);  // indices are distinct, ~index is non-zero
    VDXS_T1(2, t_so);
    VDXS_T0(t_wk);
    uint32_t cnt = 0u, emin = 0xFFFFFFFFu;
    for (int s = tid; s < P2; s += NT) {
        float v = s < nsel ? __uint_as_float((uint32_t)(sortb[s] >> 32)) : 0.0f;
        q[s] = v;
        qid[s] = s < nsel ? (int32_t)(~(uint32_t)sortb[s]) : -1;
        if (v > 0.0f) {
            ++cnt;
            int e = ilogbf(v);
            e = e < -126 ? -126 : e;
            emin = min(emin, (uint32_t)(e + 1024));
        }
    }
    cnt = block_sum_u32(cnt, shu);
    emin = block_min_u32(emin, shu);
    bool exact = true;
    if (cnt > 0u) {
        int E = ilogb((double)cnt * (double)q[0]);
        exact = (int)emin - 1024 >= E - 29;
    }
    const float u = p.uniform ? p.uniform[b] : 0.0f;
    // Each thread owns EPT consecutive walk positions (P2 <= 1024 = EPT * NT).
    constexpr int EPT = 1024 / NT;
    const int i0 = EPT * tid;
    if (exact && P2 <= 64) {
        // Up to 64 survivors: warp 0 alone, two walk positions per lane, a shuffled scan
        // and ballots (the sums are exact, so their order does not matter).
        if (tid < 32) {
            const int lane = tid, w0 = 2 * tid;
            const double a0 = w0 < nsel ? (double)q[w0] : 0.0;
            const double a1 = w0 + 1 < nsel ? (double)q[w0 + 1] : 0.0;
            double incl = a0 + a1;
#pragma unroll
            for (int d = 1; d < 32; d <<= 1) {
                const double y = __shfl_up_sync(FULL, incl, d);
                if (lane >= d) incl += y;
            }
            const double tot = __shfl_sync(FULL, incl, 31);
            double pre0 = __shfl_up_sync(FULL, incl, 1);
            if (lane == 0) pre0 = 0.0;
            const double pre1 = pre0 + a0;
            // Prefix sum before walk position i (uniform i): tot when i is past the lanes.
            auto pre_at = [&](int i) -> double {
                const double v = __shfl_sync(FULL, (i & 1) ? pre1 : pre0, (i >> 1) & 31);
                return i >= 64 ? tot : v;
            };
            auto first = [&](bool f0, bool f1) -> int {
                const unsigned b0 = __ballot_sync(FULL, f0), b1 = __ballot_sync(FULL, f1);
                const int p0 = b0 ? 2 * (__ffs(b0) - 1) : INT_MAX;
                const int p1 = b1 ? 2 * (__ffs(b1) - 1) + 1 : INT_MAX;
                return min(p0, p1);
            };
            double lsum = tot;
            int m = nsel;
            if (p.top_p < 1.0f) {
                const double target = (double)p.top_p * tot;
                const int f = first(w0 < nsel && !(pre0 < target && a0 > 0.0),
                                    w0 + 1 < nsel && !(pre1 < target && a1 > 0.0));
                m = min(f, nsel);
                lsum = pre_at(m);
            }
            const double t = (double)u * lsum;
            const int jj = first(w0 < m && pre0 + a0 > t, w0 + 1 < m && pre1 + a1 > t);
            const double before = pre_at(jj == INT_MAX ? 0 : jj);
            if (lane == 0) {
                s_i[0] = jj == INT_MAX ? -1 : jj;
                s_d[0] = t;
                s_d[1] = lsum;
                s_d[2] = jj == INT_MAX ? 0.0 : before;
            }
        }
    } else if (exact) {
        double a[EPT];
        double part = 0.0;
#pragma unroll
        for (int e = 0; e < EPT; ++e) {
            a[e] = i0 + e < P2 ? (double)q[i0 + e] : 0.0;
            part += a[e];
        }
        double tot;
        double off = block_excl_scan_d(part, s_dsh, &tot);
#pragma unroll
        for (int e = 0; e < EPT; ++e) {
            if (i0 + e < P2) pre[i0 + e] = off;
            off += a[e];
        }
        if (tid == 0) pre[P2] = tot;
        __syncthreads();
        double lsum = tot;
        int m = nsel;
        if (p.top_p < 1.0f) {
            const double target = (double)p.top_p * tot;
            uint32_t mm = (uint32_t)nsel;
            for (int i = i0; i < i0 + EPT && i < nsel; ++i)
                if (!(pre[i] < target && q[i] > 0.0f)) mm = min(mm, (uint32_t)i);
            m = (int)block_min_u32(mm, shu);
            lsum = pre[m];
        }
        const double t = (double)u * lsum;
        uint32_t jj = 0xFFFFFFFFu;
        for (int i = i0; i < i0 + EPT && i < m; ++i)
            if (pre[i] + (double)q[i] > t) jj = min(jj, (uint32_t)i);
        jj = block_min_u32(jj, shu);
        if (tid == 0) {
            s_i[0] = (int)jj;
            s_d[0] = t;
            s_d[1] = lsum;
            s_d[2] = jj != 0xFFFFFFFFu ? pre[jj] : 0.0;
        }
    } else if (tid == 0) {
        // Sequential walk, exactly the reference's arithmetic on the canonical order.
        double lsum = 0.0;
        for (int i = 0; i < nsel; ++i) lsum += q[i];
        int m = nsel;
        if (p.top_p < 1.0f) {
            const double target = (double)p.top_p * lsum;
            double cum = 0.0;
            lsum = 0.0;
            m = 0;
            for (int i = 0; i < nsel; ++i) {
                if (cum < target && q[i] > 0.0f) {
                    cum += q[i];
                    lsum += q[i];
                    m = i + 1;
                } else break;
            }
        }
        const double t = (double)u * lsum;
        double cum = 0.0, before = 0.0;
        int j = -1;
        for (int i = 0; i < m; ++i) {
            before = cum;
            cum += q[i];
            if (cum > t) {
                j = i;
                break;
            }
        }
        s_i[0] = j;
        s_d[0] = t;
        s_d[1] = lsum;
        s_d[2] = before;
    }
    __syncthreads();
    VDXS_T1(3, t_wk);
    int j = s_i[0];
    const bool fallback = j < 0 || j >= nsel;
    if (fallback) j = nsel - 1;
    uint32_t f = flags_in | VDXS_FLAG_TOPK;
    if (!exact) f |= VDXS_FLAG_INEXACT_SUM;
    if (!(p.top_p < 1.0f) && p.K > 1) f |= VDXS_FLAG_SLOT_ORDER;
    if (fallback) f |= VDXS_FLAG_FALLBACK;
    if (nsel > 1 && ((j > 0 && q[j - 1] == q[j]) || (j + 1 < nsel && q[j + 1] == q[j])))
        f |= VDXS_FLAG_DRAW_TIE_RUN;
    {
        const double t = s_d[0], lsum = s_d[1], before = s_d[2];
        const double after = before + (double)q[j];
        const double eps = 1e-6 * lsum;
        if (fallback || (t - before) <= eps || (after - t) <= eps) f |= VDXS_FLAG_NEAR_BOUNDARY;
    }
    *flags_out = f;
    const bool boundary_draw = (f & VDXS_FLAG_BOUNDARY_TIE) && q[j] == qb;
    const bool need_faithful = p.tie_mode == VDXS_TIES_FAITHFUL && p.K > 1 &&
                               (boundary_draw ||
                                (f & (VDXS_FLAG_DRAW_TIE_RUN | VDXS_FLAG_INEXACT_SUM | VDXS_FLAG_SLOT_ORDER)));
    if (!need_faithful) {
        if (tid == 0) {
            p.tokens[b] = qid[j];
            if (p.flags) p.flags[b] = f;
        }
        if (p.out_k > 0) {
            for (int s = tid; s < p.out_k; s += NT) {
                if (p.out_idx) p.out_idx[(int64_t)b * p.out_k + s] = s < nsel ? qid[s] : -1;
                if (p.out_prob) p.out_prob[(int64_t)b * p.out_k + s] = s < nsel ? q[s] : 0.0f;
            }
        }
    }
    __syncthreads();
    return need_faithful;
}

// ---------------------------------------------------------------------------------
// Faithful emulation of the reference min-buffer (Sampler.pas:341-383) over one row,
// followed by the reference's sequential double arithmetic (Sampler.pas:385-459).
// `work` must hold faithful_bytes(K) bytes (8*K for the buffer, the candidate regions,
// then the stage-2 tail).
// ---------------------------------------------------------------------------------
template <typename T>
__device__ void faithful_row(const KParams& p, int b, uint32_t flags_in, unsigned char* work,
                             uint32_t* shu) {
    // The first K elements fill the buffer in slot order (Sampler.pas:352-356): one
    // parallel pass. The rest of the row is taken in pieces of geometrically growing
    // length, in lockstep:
    // - every warp filters a contiguous share of the piece (penalised values overlaid)
    //   against the buffer minimum at the piece's start and compacts, in index order,
    //   the elements above it into its own region. The minimum only grows, so nothing
    //   the reference inserts is dropped;
    // - warp 0 replays the regions in warp order: an element strictly above the current
    //   minimum replaces the minimum's slot, and the lowest slot holding the minimum
    //   value becomes the next one. Lane l keeps the minimum of the slots s = l (mod 32).
    //   For top_k <= 64 (at most two slots per lane) the slot keys stay in registers and
    //   an insertion costs one warp reduction and two ballots; otherwise the warp rescans
    //   the owning lane's slots and two pairs of warp reductions give the new minimum.
    // A piece whose share overflows a region is filtered again at the shortest length,
    // where a share (kFaithfulSub elements) always fits.
    constexpr int CW = kFaithfulSlots * kFaithfulSub / NWARPS;  // region entries per warp
    constexpr int RS = kFaithfulSub / 32;                        // elements per lane per step
    static_assert(CW >= kFaithfulSub, "a shortest-piece share must fit a region");
    __shared__ float s_mv;
    __shared__ int s_cnt[NWARPS];
    const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
    const int K = p.K, V = p.V;
    const T* row = (const T*)p.logits + (int64_t)b * p.stride;
    float* sval = (float*)work;
    int32_t* sidx = (int32_t*)(sval + K);
    float* rval = (float*)(sidx + K);                 // [NWARPS][CW]
    int32_t* ridx = (int32_t*)(rval + NWARPS * CW);  // [NWARPS][CW]
    unsigned char* tail = (unsigned char*)(ridx + NWARPS * CW);
    tail = (unsigned char*)(((uintptr_t)tail + 15) & ~(uintptr_t)15);
    const int npen = p.pen_cnt ? p.pen_cnt[b] : 0;
    const int32_t* pid = p.pen_ids ? p.pen_ids + (int64_t)b * p.pen_stride : nullptr;
    const float* pvl = p.pen_vals ? p.pen_vals + (int64_t)b * p.pen_stride : nullptr;
    const int RL = (K + 31) / 32;  // slots per lane (lane l owns slots l, l + 32, ...)
    // Minimum of the slots this lane owns; the first slot wins ties (strict '<'). Eight
    // slots are loaded at a time so that their latencies overlap.
    auto lane_min = [&](int& bs) -> uint32_t {
        float bv = 0.0f;
        bs = INT_MAX;
        for (int s0 = lane; s0 < K; s0 += 32 * 8) {
            float x[8];
#pragma unroll
            for (int u = 0; u < 8; ++u) x[u] = s0 + 32 * u < K ? sval[s0 + 32 * u] : 0.0f;
#pragma unroll
            for (int u = 0; u < 8; ++u) {
                const int s2 = s0 + 32 * u;
                if (s2 < K && (bs == INT_MAX || x[u] < bv)) {
                    bv = x[u];
                    bs = s2;
                }
            }
        }
        return bs == INT_MAX ? 0xFFFFFFFFu : f2key(bv);
    };

    for (int s = tid; s < K; s += NT) {
        sval[s] = ld_elem(row, s);
        sidx[s] = s;
    }
    __syncthreads();
    for (int j = tid; j < npen; j += NT) {  // penalised ids ascend
        const int id = pid[j];
        if (id >= K) break;
        sval[id] = pvl[j];
    }
    __syncthreads();
    // Scanner state (warp 0): per lane the key and slot of its minimum; warp-uniform the
    // buffer minimum mv and its slot ms.
    uint32_t kv = 0xFFFFFFFFu;
    int bs = INT_MAX, ms = 0;
    float mv = -INFINITY;
    // top_k <= 64: the keys of slots lane and lane + 32 (0xFFFFFFFF: no slot).
    const bool regs = RL <= 2;
    uint32_t k0 = 0xFFFFFFFFu, k1 = 0xFFFFFFFFu;
    if (warp == 0) {
        kv = lane_min(bs);
        const uint32_t mk = __reduce_min_sync(FULL, kv);
        ms = (int)__reduce_min_sync(FULL, kv == mk ? (uint32_t)bs : 0xFFFFFFFFu);
        mv = key2f(mk);
        if (lane == 0) s_mv = mv;
        if (regs) {
            if (lane < K) k0 = f2key(sval[lane]);
            if (lane + 32 < K) k1 = f2key(sval[lane + 32]);
        }
    }
    __syncthreads();
    VDXS_T0(t_floop);
    // Two step kinds: vector steps of SPAN elements (16-byte loads, VL per lane; they
    // need a 16-byte aligned start and a whole step inside the share) and scalar steps
    // of kFaithfulSub elements (any alignment; row tails). A "safe" piece uses scalar
    // steps only and is at most kMinPiece long, so no share outgrows its region.
    constexpr int E = 16 / (int)sizeof(T);  // elements per 16-byte load
    constexpr int VL = 8;                   // 16-byte loads per lane per vector step
    constexpr int SPAN = 32 * VL * E;       // elements per vector step
    constexpr int kMinPiece = NWARPS * kFaithfulSub;
    const uintptr_t rowaddr = (uintptr_t)row;
    auto aligned_at = [&](int64_t i) { return ((rowaddr + (uintptr_t)i * sizeof(T)) & 15u) == 0u; };
    int64_t pos = K;
    bool safe = true;
    // The first piece is safe and ends at a 16-byte aligned element, so that vector
    // pieces (whose lengths are multiples of SPAN) start aligned.
    int64_t first_end = min((int64_t)V, pos + kMinPiece);
    while (first_end > pos + 1 && first_end < V && !aligned_at(first_end)) --first_end;
    int L = (int)(first_end - pos);
    while (pos < V) {
        VDXS_T0(t_pf);
        const int len = (int)min((int64_t)L, (int64_t)V - pos);
        const int gran = safe ? kFaithfulSub : SPAN;
        // Warp shares are whole steps.
        const int per = ((len + NWARPS - 1) / NWARPS + gran - 1) / gran * gran;
        const int64_t s0 = pos + (int64_t)warp * per;
        const int64_t s1 = min(s0 + per, pos + len);
        const float tau = s_mv;
        float* cv = rval + warp * CW;
        int32_t* ci = ridx + warp * CW;
        int cnt = 0;
        int jc = npen ? lower_bound_i32(pid, npen, s0) : 0;  // first penalised id of the share
        // Overlays the penalised values of ids in [lo, lo + n) onto f (f[e] holds element
        // lo + lane * EL + e).
        auto overlay = [&](float* f, int EL, int64_t lo, int n) {
            while (jc < npen) {
                const int j = jc + lane;
                const int id = j < npen ? pid[j] : INT_MAX;
                const bool in = id >= lo && id < lo + n;
                const unsigned mb = __ballot_sync(FULL, id < lo), mi = __ballot_sync(FULL, in);
                const float pv = in ? pvl[j] : 0.0f;
                for (unsigned m = mi; m; m &= m - 1) {
                    const int l = __ffs(m) - 1;
                    const int off = (int)(__shfl_sync(FULL, id, l) - lo);
                    const float val = __shfl_sync(FULL, pv, l);
                    // Select form (no store indexed by a run-time value, so f stays in
                    // registers).
                    const int tl = off / EL, te = off - (off / EL) * EL;
#pragma unroll
                    for (int e = 0; e < 8; ++e)
                        if (e < EL) f[e] = (lane == tl && e == te) ? val : f[e];
                }
                const int adv = __popc(mb | mi);
                jc += adv;
                if (adv < 32) break;
            }
        };
        int64_t a = s0;
        while (a < s1) {
            if (!safe && a + SPAN <= s1 && aligned_at(a)) {
                uint4 r4[VL];
#pragma unroll
                for (int r = 0; r < VL; ++r) r4[r] = ld_stream16(row + a + (int64_t)(r * 32 + lane) * E);
#pragma unroll
                for (int r = 0; r < VL; ++r) {
                    const int64_t br = a + (int64_t)r * 32 * E;
                    float f[8];
                    unpack(r4[r], f, T());
                    if (npen) overlay(f, E, br, 32 * E);
                    uint32_t cm = 0u;
#pragma unroll
                    for (int e = 0; e < E; ++e)
                        if (f[e] > tau) cm |= 1u << e;
                    if (!__any_sync(FULL, cm != 0u)) continue;
                    const int c = __popc(cm);
                    int ex = c;
#pragma unroll
                    for (int d = 1; d < 32; d <<= 1) {
                        const int o = __shfl_up_sync(FULL, ex, d);
                        if (lane >= d) ex += o;
                    }
                    const int tot = __shfl_sync(FULL, ex, 31);
                    ex -= c;
                    if (cm) {
                        int k = cnt + ex;
#pragma unroll
                        for (int e = 0; e < E; ++e)
                            if ((cm >> e) & 1u) {
                                if (k < CW) {
                                    cv[k] = f[e];
                                    ci[k] = (int32_t)(br + lane * E + e);
                                }
                                ++k;
                            }
                    }
                    cnt += tot;
                }
                a += SPAN;
            } else {
                float v[RS];
#pragma unroll
                for (int r = 0; r < RS; ++r) {
                    const int64_t i = a + r * 32 + lane;
                    v[r] = i < s1 ? ld_elem(row, i) : 0.0f;
                }
                if (npen) {
                    // Element a + r * 32 + lane: overlay one 32-element row at a time.
#pragma unroll
                    for (int r = 0; r < RS; ++r) {
                        float f1[8];
                        f1[0] = v[r];
                        overlay(f1, 1, a + r * 32, 32);
                        v[r] = f1[0];
                    }
                }
#pragma unroll
                for (int r = 0; r < RS; ++r) {
                    const int64_t i = a + r * 32 + lane;
                    const bool c = i < s1 && v[r] > tau;
                    const unsigned m = __ballot_sync(FULL, c);
                    if (c) {
                        const int q = cnt + __popc(m & lanemask_lt());
                        if (q < CW) {
                            cv[q] = v[r];
                            ci[q] = (int32_t)i;
                        }
                    }
                    cnt += __popc(m);
                }
                a += kFaithfulSub;
            }
        }
        VDXS_T1(25, t_pf);
        VDXS_T0(t_pw);
        if (lane == 0) s_cnt[warp] = cnt;
        __syncthreads();
        VDXS_T1(26, t_pw);
        int total = 0;
        bool over = false;
#pragma unroll
        for (int w = 0; w < NWARPS; ++w) {
            total += s_cnt[w];
            over |= s_cnt[w] > CW;
        }
        if (over) {
            // Again as a safe piece: every share is one scalar step, which always fits.
            L = kMinPiece;
            safe = true;
            __syncthreads();
            continue;
        }
        VDXS_T0(t_pr);
        if (warp == 0) {
            for (int w = 0; w < NWARPS; ++w) {
                const int nw = s_cnt[w];
                for (int c0 = 0; c0 < nw; c0 += 32) {
                    const int c = c0 + lane;
                    const bool valid = c < nw;
                    const float v = valid ? rval[w * CW + c] : 0.0f;
                    const int32_t gi = valid ? ridx[w * CW + c] : 0;
                    unsigned pend = __ballot_sync(FULL, valid && v > mv);
                    while (pend) {
                        VDXS_T0(t_in);
                        const int l = __ffs(pend) - 1;
                        const float nv = __shfl_sync(FULL, v, l);
                        const int32_t ngi = __shfl_sync(FULL, gi, l);
#ifdef VDXS_TIMING
                        if (lane == 0) atomicAdd(&g_phase_count[24], 1ull);
#endif
                        if (regs) {
                            // The owner updates its key in registers; the lowest slot holding
                            // the minimum key is in the lowest lane holding it as its first
                            // slot, else in the lowest lane holding it as its second.
                            if (lane == (ms & 31)) {
                                sval[ms] = nv;
                                sidx[ms] = ngi;
                                const uint32_t nk = f2key(nv);
                                if (ms >= 32) k1 = nk;
                                else k0 = nk;
                                kv = min(k0, k1);
                            }
                            const uint32_t mk = __reduce_min_sync(FULL, kv);
                            const unsigned first = __ballot_sync(FULL, k0 == mk);
                            ms = first ? __ffs(first) - 1 : __ffs(__ballot_sync(FULL, k1 == mk)) + 31;
                            mv = key2f(mk);
                        } else {
                            if (lane == (ms & 31)) {
                                sval[ms] = nv;
                                sidx[ms] = ngi;
                            }
                            __syncwarp();
                            // The owner's slots are rescanned by the whole warp (lane u reads
                            // slot owner + 32*u), then the buffer minimum over the lanes' minima.
                            const int owner = ms & 31, s2 = owner + 32 * lane;
                            const uint32_t ok = lane < RL && s2 < K ? f2key(sval[s2]) : 0xFFFFFFFFu;
                            const uint32_t omk = __reduce_min_sync(FULL, ok);
                            const uint32_t obs = __reduce_min_sync(FULL, ok == omk ? (uint32_t)s2 : 0xFFFFFFFFu);
                            if (lane == owner) {
                                kv = omk;
                                bs = (int)obs;
                            }
                            const uint32_t mk = __reduce_min_sync(FULL, kv);
                            ms = (int)__reduce_min_sync(FULL, kv == mk ? (uint32_t)bs : 0xFFFFFFFFu);
                            mv = key2f(mk);
                        }
                        pend &= ~(1u << l);
                        pend &= __ballot_sync(FULL, valid && v > mv);
                        VDXS_T1(28, t_in);
                    }
                }
            }
            if (lane == 0) s_mv = mv;
        }
        VDXS_T1(27, t_pr);
#ifdef VDXS_TIMING
        if (tid == 0) atomicAdd(&g_phase_count[23], (unsigned long long)total);
#endif
        __syncthreads();
        pos += len;
        if (safe) {
            // Back to vector pieces (lengths in whole vector steps per warp).
            safe = false;
            L = NWARPS * SPAN;
        } else if (total < 4 * CW) {
            // Candidates per piece stay near K when the length tracks the position.
            L = (int)min((int64_t)L * 2, (int64_t)1 << 24);
        }
    }
    VDXS_T1(22, t_floop);

    // Sequential stage 2 in slot order (Sampler.pas:385-459).
    int P2 = 32;
    while (P2 < K) P2 <<= 1;
    uint64_t* sortb = (uint64_t*)tail;
    float* prob = (float*)(sortb + P2);
    int32_t* wid = (int32_t*)(prob + P2);
    uint32_t mk = 0u;
    for (int s = tid; s < K; s += NT) mk = max(mk, f2key(sval[s]));
    mk = block_max_u32(mk, shu);
    const double Md = (double)key2f(mk), it = (double)p.inv_temp;
    for (int s = tid; s < K; s += NT) prob[s] = (float)exp(((double)sval[s] - Md) * it);
    __syncthreads();
    __shared__ double s_lsum;
    if (tid == 0) {
        double lsum = 0.0;
        for (int s = 0; s < K; ++s) lsum += prob[s];
        if (p.min_p > 0.0f) {
            float best = prob[0];
            for (int s = 1; s < K; ++s)
                if (prob[s] > best) best = prob[s];
            const float thr = __fmul_rn(best, p.min_p);
            lsum = 0.0;
            for (int s = 0; s < K; ++s)
                if (prob[s] < thr) prob[s] = 0.0f;
                else lsum += prob[s];
        }
        s_lsum = lsum;
    }
    __syncthreads();
    const bool sorted = p.top_p < 1.0f;
    if (sorted) {
        // Stable descending insertion sort == sort by (prob desc, slot asc).
        for (int s = tid; s < P2; s += NT)
            sortb[s] = s < K ? (((uint64_t)__float_as_uint(prob[s]) << 32) | (uint64_t)(0xFFFFFFFFu - (uint32_t)s)) : 0ull;
        __syncthreads();
        block_sort_desc_distinct(sortb, K, P2);  // slots are distinct, 0xFFFFFFFF - slot is non-zero
        for (int s = tid; s < K; s += NT) {
            const uint32_t slot = 0xFFFFFFFFu - (uint32_t)sortb[s];
            wid[s] = sidx[slot];
        }
        __syncthreads();
        for (int s = tid; s < K; s += NT) prob[s] = __uint_as_float((uint32_t)(sortb[s] >> 32));
    } else {
        for (int s = tid; s < K; s += NT) wid[s] = sidx[s];
    }
    __syncthreads();
    if (p.out_k > 0) {
        for (int s = tid; s < p.out_k; s += NT) {
            if (p.out_idx) p.out_idx[(int64_t)b * p.out_k + s] = s < K ? wid[s] : -1;
            if (p.out_prob) p.out_prob[(int64_t)b * p.out_k + s] = s < K ? prob[s] : 0.0f;
        }
    }
    __syncthreads();
    if (tid == 0) {
        double lsum = s_lsum;
        int m = K;
        if (sorted) {
            const double target = (double)p.top_p * lsum;
            double cum = 0.0;
            lsum = 0.0;
            m = 0;
            for (int i = 0; i < K; ++i) {
                if (cum < target && prob[i] > 0.0f) {
                    cum += prob[i];
                    lsum += prob[i];
                    m = i + 1;
                } else break;
            }
        }
        const float u = p.uniform ? p.uniform[b] : 0.0f;
        const double t = (double)u * lsum;
        double cum = 0.0, before = 0.0;
        int j = -1;
        for (int i = 0; i < m; ++i) {
            before = cum;
            cum += prob[i];
            if (cum > t) {
                j = i;
                break;
            }
        }
        const bool fallback = j < 0;
        if (fallback) j = K - 1;
        uint32_t f = (flags_in & (VDXS_FLAG_BOUNDARY_TIE | VDXS_FLAG_INEXACT_SUM)) | VDXS_FLAG_TOPK |
                     VDXS_FLAG_FAITHFUL_PASS;
        if (!sorted && K > 1) f |= VDXS_FLAG_SLOT_ORDER;
        if (fallback) f |= VDXS_FLAG_FALLBACK;
        if (sorted && K > 1 && ((j > 0 && prob[j - 1] == prob[j]) || (j + 1 < K && prob[j + 1] == prob[j])))
            f |= VDXS_FLAG_DRAW_TIE_RUN;
        const double after = before + (fallback ? 0.0 : (double)prob[j]);
        const double eps = 1e-6 * lsum;
        if (fallback || (t - before) <= eps || (after - t) <= eps) f |= VDXS_FLAG_NEAR_BOUNDARY;
        p.tokens[b] = wid[j];
        if (p.flags) p.flags[b] = f;
    }
    __syncthreads();
}

// Element loads as float (bf16 widened exactly).
__device__ __forceinline__ float to_f(float v) { return v; }
__device__ __forceinline__ float to_f(uint16_t v) { return __uint_as_float((uint32_t)v << 16); }

// Writes every selected element of src to (ok, oi), returns the count (uniform).
template <class Src, class IdxF>
__device__ int block_emit(const Src& src, int n, const SelectOut& s, uint32_t* ok, uint32_t* oi, int cap,
                          uint32_t* counter, IdxF idx_of) {
    const int tid = threadIdx.x;
    if (tid == 0) *counter = 0u;
    __syncthreads();
    for (int i0 = tid; i0 - tid < n; i0 += 4 * NT) {
        uint32_t k[4];
        bool sel[4];
#pragma unroll
        for (int u = 0; u < 4; ++u) k[u] = i0 + u * NT < n ? src.key(i0 + u * NT) : 0u;
#pragma unroll
        for (int u = 0; u < 4; ++u) sel[u] = i0 + u * NT < n && selected(k[u], src.tb(i0 + u * NT), s);
#pragma unroll
        for (int u = 0; u < 4; ++u) {
            const unsigned m = __ballot_sync(FULL, sel[u]);
            if (m) {
                uint32_t base = 0u;
                if ((tid & 31) == 0) base = atomicAdd(counter, (uint32_t)__popc(m));
                base = __shfl_sync(FULL, base, 0);
                if (sel[u]) {
                    const uint32_t slot = base + __popc(m & lanemask_lt());
                    if (slot < (uint32_t)cap) {
                        ok[slot] = k[u];
                        oi[slot] = idx_of(i0 + u * NT);
                    }
                }
            }
        }
    }
    __syncthreads();
    const uint32_t c = *counter;
    __syncthreads();
    return (int)min(c, (uint32_t)cap);
}

struct IdentIdx {
    const uint32_t* t;
    __device__ __forceinline__ uint32_t operator()(int i) const { return t[i]; }
};
struct OffsetIdx {
    uint32_t base;
    __device__ __forceinline__ uint32_t operator()(int i) const { return base + (uint32_t)i; }
};

// Stage 2 of one row from gathered candidates (ckey, cidx)[0, n2) in shared memory:
// exact top-K (block_select), boundary-tie evidence (selection cuts, and cut_of(i) for
// the ncut stage-1 items), then greedy / draw / publication for the all-gather, and
// the faithful re-resolution when the row needs it. sk/si are placed at `region`.
template <typename T, class CutOf>
__device__ void finish_select(const KParams& p, int b, uint32_t* ckey, uint32_t* cidx, int n2, uint32_t gmax,
                              int ncut, CutOf cut_of, unsigned char* region, uint32_t* hist, uint32_t* sh) {
    const int tid = threadIdx.x;
    const int K = p.K;
    uint32_t* sk = (uint32_t*)region;
    uint32_t* si = sk + K;
    const int tbb = bits_for((uint32_t)(p.vocab_offset + p.V - 1));
    VDXS_T0(t_sel);
    SelectOut s2;
    int nsel;
    if (n2 <= NT) {
        // Few candidates: rank select. (key, ~index) composites are distinct, so the
        // rank of each valid entry is its position in (key desc, index asc) order; key 0
        // ranks below every valid entry and is never selected.
        const int tid2 = threadIdx.x;
        const uint64_t mine = tid2 < n2 ? ((uint64_t)ckey[tid2] << 32) | (uint32_t)~cidx[tid2] : 0ull;
        const bool valid = tid2 < n2 && ckey[tid2] != 0u;
        int rank = 0;
        if (valid)
            for (int j = 0; j < n2; ++j) rank += (((uint64_t)ckey[j] << 32) | (uint32_t)~cidx[j]) > mine ? 1 : 0;
        const uint32_t nv = block_sum_u32(valid ? 1u : 0u, sh + 32);
        if (valid && rank == K - 1) sh[8] = (uint32_t)(mine >> 32);
        __syncthreads();
        const uint32_t kth = nv > (uint32_t)K ? sh[8] : 0u;
        const bool cut = valid && rank >= K && (uint32_t)(mine >> 32) == kth;
        s2.tie_cut = __syncthreads_or(cut) ? 1 : 0;
        s2.kth_key = kth;
        s2.kth_tb = 0xFFFFFFFFu;
        s2.n_valid = nv;
        if (valid && rank < K) {
            sk[rank] = (uint32_t)(mine >> 32);
            si[rank] = ~(uint32_t)mine;
        }
        nsel = (int)min(nv, (uint32_t)K);
        __syncthreads();
    } else {
        s2 = block_select(SmemPairSrc{ckey, cidx}, n2, K, gmax, tbb, hist, sh);
        nsel = block_emit(SmemPairSrc{ckey, cidx}, n2, s2, sk, si, K, &sh[8], IdentIdx{cidx});
    }
    VDXS_T1(4, t_sel);
    // The boundary value is the smallest selected key. A boundary tie exists when the
    // merge cut elements of that value, or a stage-1 item cut elements of that value.
    uint32_t kb = 0xFFFFFFFFu;
    for (int s = tid; s < nsel; s += NT) kb = min(kb, sk[s]);
    kb = block_min_u32(kb, sh + 32);
    uint32_t ck_tie = 0u;
    for (int i = tid; i < ncut; i += NT) {
        const uint32_t c = cut_of(i);
        if (c != 0u && c == kb) ck_tie = 1u;
    }
    ck_tie = block_max_u32(ck_tie, sh + 32);
    const uint32_t btie = (s2.tie_cut || ck_tie) ? VDXS_FLAG_BOUNDARY_TIE : 0u;
    if (tid == 0) p.row_counter[b] = 0u;  // ready for the next launch

    if (p.local_emit) {
        // Vocab-sharded: publish the local top-K and tie evidence for the all-gather.
        uint2* eo = p.emit_out + (int64_t)b * (K + 1);
        for (int s = tid; s < K; s += NT) eo[s] = s < nsel ? make_uint2(sk[s], si[s]) : make_uint2(0u, 0xFFFFFFFFu);
        if (tid == 0) eo[K] = make_uint2(kb, btie ? 1u : 0u);
        return;
    }
    if (p.path == kGreedy) {
        // Greedy (Sampler.pas:305-322): the canonical top-1 is the first maximum.
        if (tid == 0) {
            p.tokens[b] = (int32_t)si[0];
            if (p.flags) p.flags[b] = VDXS_FLAG_GREEDY;
        }
        for (int s = tid; s < p.out_k; s += NT) {
            if (p.out_idx) p.out_idx[(int64_t)b * p.out_k + s] = s == 0 ? (int32_t)si[0] : -1;
            if (p.out_prob) p.out_prob[(int64_t)b * p.out_k + s] = 0.0f;
        }
        return;
    }
    unsigned char* work = (unsigned char*)(ckey);
    work = (unsigned char*)(((uintptr_t)work + 15) & ~(uintptr_t)15);
    uint32_t f2;
    VDXS_T0(t_s2);
    const bool faithful = stage2_canonical(p, b, sk, si, nsel, gmax, kb, btie, work, sh + 32, &f2);
    VDXS_T1(6, t_s2);
    if (faithful) {
        VDXS_T0(t_ff);
        faithful_row<T>(p, b, f2, region, sh + 32);
        VDXS_T1(7, t_ff);
    }
}

template <typename T>
struct RowKeySrc {  // a row in global memory (NaN: no element), tie-break = position
    const T* row;
    __device__ __forceinline__ uint32_t key(int i) const {
        const float v = ld_elem(row, i);
        return v == v ? f2key(v) : 0u;
    }
    __device__ __forceinline__ uint32_t tb(int i) const { return (uint32_t)i; }
};

// A row's stage-1 list (every element at or above the row's bound, plus candidates taken
// while the bounds were rising) followed by the row's penalised entries: entries below
// the bound read as absent, and the tie-break and emitted index is the element's index.
struct ListSrc {
    const uint2* cand;
    int n;
    uint32_t bound;
    const int32_t* pid;
    const float* pvl;
    int64_t offset;
    __device__ __forceinline__ uint2 entry(int i) const {
        if (i < n) return __ldcg(cand + i);
        const float v = pvl[i - n];
        return make_uint2(v == v ? f2key(v) : 0u, (uint32_t)(pid[i - n] + offset));
    }
    __device__ __forceinline__ uint32_t key(int i) const {
        const uint32_t k = entry(i).x;
        return k >= bound ? k : 0u;
    }
    __device__ __forceinline__ uint32_t tb(int i) const { return entry(i).y; }
};
struct ListIdx {
    const ListSrc* src;
    __device__ __forceinline__ uint32_t operator()(int i) const { return src->tb(i); }
};

// Exact fallback of the finish for a row whose stage-1 lists are incomplete or do not
// fit the gather: the top (K + npen) of the raw row (penalties not applied) contain the
// top K of its non-penalised elements, so that select, with the penalised ids among it
// replaced by their penalised entries, gives finish_select the same candidates as a
// complete gather. Elements equal to the select's boundary key that it left out are
// reported as a cut. ckey/cidx hold gcap >= K + npen entries each (cidx = ckey + gcap).
template <typename T>
__device__ __noinline__ void finish_row_exact(const KParams& p, int b, uint32_t* ckey, int gcap, unsigned char* region,
                                 uint32_t* hist, uint32_t* sh) {
    const int tid = threadIdx.x;
    const int npen = p.pen_cnt ? p.pen_cnt[b] : 0;
    const int32_t* pid = p.pen_ids ? p.pen_ids + (int64_t)b * p.pen_stride : nullptr;
    const float* pvl = p.pen_vals ? p.pen_vals + (int64_t)b * p.pen_stride : nullptr;
    uint32_t* cidx = ckey + gcap;
    const RowKeySrc<T> src{(const T*)p.logits + (int64_t)b * p.stride};
    uint32_t km = 0u;
    for (int i0 = tid; i0 < p.V; i0 += 4 * NT) {
        uint32_t k[4];
#pragma unroll
        for (int u = 0; u < 4; ++u) k[u] = i0 + u * NT < p.V ? src.key(i0 + u * NT) : 0u;
        km = max(max(km, max(k[0], k[1])), max(k[2], k[3]));
    }
    km = block_max_u32(km, sh + 32);
    const int kx = min(p.K + npen, gcap - npen);  // the plan makes gcap - npen >= K + npen
    const SelectOut so = block_select(src, p.V, kx, km, bits_for((uint32_t)(p.V - 1)), hist, sh);
    const int m = block_emit(src, p.V, so, ckey, cidx, gcap - npen, &sh[8], OffsetIdx{(uint32_t)p.vocab_offset});
    for (int i = tid; i < m; i += NT) {
        const int64_t local = (int64_t)cidx[i] - p.vocab_offset;
        const int j = lower_bound_i32(pid, npen, local);
        if (j < npen && pid[j] == local) ckey[i] = 0u;  // re-enters with its penalised value
    }
    for (int j = tid; j < npen; j += NT) {
        ckey[m + j] = f2key(pvl[j]);
        cidx[m + j] = (uint32_t)(pid[j] + p.vocab_offset);
    }
    __syncthreads();
    uint32_t gm = 0u;
    for (int i = tid; i < m + npen; i += NT) gm = max(gm, ckey[i]);
    gm = block_max_u32(gm, sh + 32);
    const uint32_t cut = so.tie_cut ? so.kth_key : 0u;
    finish_select<T>(p, b, ckey, cidx, m + npen, gm, 1, [&](int) -> uint32_t { return cut; }, region, hist, sh);
}

// Exact select of the finish for a row whose stage-1 list is complete but whose entries
// at or above the row bound tb do not fit the gather: the top K of the list's entries at
// or above tb and the row's penalised entries (the list holds no penalised id) are the
// top K of the row's candidates, and the select reads the list, not the row. Elements
// equal to the select's boundary key that it left out are reported as a cut, as in
// finish_row_exact.
template <typename T>
__device__ __noinline__ void finish_list_exact(const KParams& p, int b, uint32_t tb, int count, uint32_t* ckey,
                                               int gcap, unsigned char* region, uint32_t* hist, uint32_t* sh) {
    const int tid = threadIdx.x;
    const int npen = p.pen_cnt ? p.pen_cnt[b] : 0;
    uint32_t* cidx = ckey + gcap;
    const ListSrc src{p.cand + (size_t)b * p.cand_cap, count, tb,
                      p.pen_ids ? p.pen_ids + (int64_t)b * p.pen_stride : nullptr,
                      p.pen_vals ? p.pen_vals + (int64_t)b * p.pen_stride : nullptr, p.vocab_offset};
    const int n = count + npen;
    uint32_t km = 0u;
    for (int i0 = tid; i0 < n; i0 += 4 * NT) {
        uint32_t k[4];
#pragma unroll
        for (int u = 0; u < 4; ++u) k[u] = i0 + u * NT < n ? src.key(i0 + u * NT) : 0u;
        km = max(max(km, max(k[0], k[1])), max(k[2], k[3]));
    }
    km = block_max_u32(km, sh + 32);
    const SelectOut so = block_select(src, n, p.K, km, bits_for((uint32_t)(p.vocab_offset + p.V - 1)),
                                               hist, sh);
    const int m = block_emit(src, n, so, ckey, cidx, gcap, &sh[8], ListIdx{&src});
    const uint32_t cut = so.tie_cut ? so.kth_key : 0u;
    finish_select<T>(p, b, ckey, cidx, m, km, 1, [&](int) -> uint32_t { return cut; }, region, hist, sh);
}

template <typename T>
__device__ void finish_row(const KParams& p, int b, unsigned char* region, uint32_t* hist, uint32_t* sh) {
    const int tid = threadIdx.x;
    const int K = p.K;
    const int npen = p.pen_cnt ? p.pen_cnt[b] : 0;
    const int32_t* pid = p.pen_ids ? p.pen_ids + (int64_t)b * p.pen_stride : nullptr;
    uint32_t* sk = (uint32_t*)region;
    uint32_t* si = sk + K;
    uint32_t* ckey = si + K;
    const uint32_t cc = (uint32_t)p.cand_cap;
    // The row's bound: the largest bound any stage-1 warp published, a lower bound on the
    // row's K-th key; the row's list holds every element at or above it. Candidates and
    // penalised entries below it can be neither selected nor tied at the boundary, and
    // are not gathered.
    const uint32_t tb = __ldcg(&p.row_tau[(size_t)b * kTauStride]);
    const uint32_t craw = __ldcg(&p.row_cnt[b]);
    // A list that outgrew its capacity (count > cand_cap) is incomplete, and a gather that
    // does not fit the shared arrays: both send the row to the exact fallback below.
    const bool incomplete = craw > cc;
    const int gcap = p.gather_cap + npen;
    uint32_t* cidx = ckey + gcap;
    uint32_t lm = 0u;
    VDXS_T0(t_gather);
    {
        const int lane = tid & 31;
        if (tid == 0) sh[40] = 0u;
        __syncthreads();
        // Appends the kept entries of a warp-uniform step at slots from a shared counter.
        auto put = [&](bool keep, uint32_t k, uint32_t ix) {
            const unsigned m = __ballot_sync(FULL, keep);
            uint32_t base = 0u;
            if (lane == 0 && m) base = atomicAdd(&sh[40], (uint32_t)__popc(m));
            base = __shfl_sync(FULL, base, 0);
            if (keep) {
                const uint32_t pos = base + __popc(m & lanemask_lt());
                if (pos < (uint32_t)gcap) {
                    ckey[pos] = k;
                    cidx[pos] = ix;
                }
                lm = max(lm, k);
            }
        };
        if (!incomplete) {
            // The whole CTA walks the list, eight loads in flight per thread; a warp reserves
            // the slots of its eight entries at once (one shared atomic per step).
            constexpr int GU = 8;
            const int c = (int)craw;
            const uint2* src = p.cand + (size_t)b * cc;
            for (int j0 = 0; j0 < c; j0 += GU * NT) {
                uint2 e[GU];
#pragma unroll
                for (int u = 0; u < GU; ++u) {
                    const int j = j0 + u * NT + tid;
                    e[u] = j < c ? __ldcg(src + j) : make_uint2(0u, 0u);
                }
                unsigned m[GU];
                uint32_t tot = 0u;
#pragma unroll
                for (int u = 0; u < GU; ++u) {
                    m[u] = __ballot_sync(FULL, j0 + u * NT + tid < c && e[u].x >= tb);
                    tot += (uint32_t)__popc(m[u]);
                }
                if (tot == 0u) continue;
                uint32_t base = 0u;
                if (lane == 0) base = atomicAdd(&sh[40], tot);
                base = __shfl_sync(FULL, base, 0);
#pragma unroll
                for (int u = 0; u < GU; ++u) {
                    if ((m[u] >> lane) & 1u) {
                        const uint32_t pos = base + __popc(m[u] & lanemask_lt());
                        if (pos < (uint32_t)gcap) {
                            ckey[pos] = e[u].x;
                            cidx[pos] = e[u].y;
                        }
                        lm = max(lm, e[u].x);
                    }
                    base += (uint32_t)__popc(m[u]);
                }
            }
        }
        for (int j0 = 0; j0 < npen; j0 += NT) {
            const int j = j0 + tid;
            uint32_t k = 0u;
            if (j < npen) k = f2key(p.pen_vals[(int64_t)b * p.pen_stride + j]);
            put(j < npen && k >= tb, k, j < npen ? (uint32_t)(pid[j] + p.vocab_offset) : 0u);
        }
        __syncthreads();
    }
    VDXS_T1(29, t_gather);
    const int n2 = (int)sh[40];
    if (incomplete) {
#ifdef VDXS_TIMING
        if (tid == 0) atomicAdd(&g_phase_count[30], 1ull);
#endif
        finish_row_exact<T>(p, b, ckey, gcap, region, hist, sh);
        return;
    }
    if (n2 > gcap) {
#ifdef VDXS_TIMING
        if (tid == 0) atomicAdd(&g_phase_count[31], 1ull);
#endif
        finish_list_exact<T>(p, b, tb, (int)craw, ckey, gcap, region, hist, sh);
        return;
    }
    const uint32_t gmax = block_max_u32(lm, sh + 32);
    finish_select<T>(p, b, ckey, cidx, n2, gmax, 0, [&](int) -> uint32_t { return 0u; }, region, hist, sh);
}

// ---------------------------------------------------------------------------------
// Warp-level select (one warp, warp-private histogram; __syncwarp only). Same result
// as block_select: the K-th best element of src[0..n) in (key desc, tb asc) order.
// ---------------------------------------------------------------------------------
struct WarpFind {
    int g;
    uint32_t before, total, cnt_g;
};
// First bin g of hist[0..NB) whose inclusive prefix reaches `need` (one warp).
template <int NB>
__device__ __forceinline__ WarpFind warp_find_reg(const uint32_t* hist, uint32_t need) {
    constexpr int SEG = (NB + 31) / 32;
    const int l = threadIdx.x & 31;
    uint32_t v[SEG];
    uint32_t s = 0;
#pragma unroll
    for (int j = 0; j < SEG; ++j) {
        const int bI = l * SEG + j;
        v[j] = bI < NB ? hist[bI] : 0u;
        s += v[j];
    }
    uint32_t incl = s;
#pragma unroll
    for (int o = 1; o < 32; o <<= 1) {
        const uint32_t y = __shfl_up_sync(FULL, incl, o);
        if (l >= o) incl += y;
    }
    WarpFind f;
    f.total = __shfl_sync(FULL, incl, 31);
    const unsigned m = __ballot_sync(FULL, incl >= need);
    if (m == 0u) {
        f.g = -1;
        f.before = f.total;
        f.cnt_g = 0;
        return f;
    }
    const int L = __ffs(m) - 1;
    // Resolve inside lane L's segment from registers.
    uint32_t c = incl - s;
    int gj = SEG - 1;
    uint32_t cg = 0;
    bool found = false;
#pragma unroll
    for (int j = 0; j < SEG; ++j) {
        if (!found && c + v[j] >= need) {
            gj = j;
            cg = v[j];
            found = true;
        } else if (!found) {
            c += v[j];
        }
    }
    f.g = __shfl_sync(FULL, l * SEG + gj, L);
    f.before = __shfl_sync(FULL, c, L);
    f.cnt_g = __shfl_sync(FULL, cg, L);
    return f;
}

template <class Src>
__device__ SelectOut warp_select(const Src& src, int n, int K, uint32_t kmax, int tb_bits, uint32_t* wh) {
    const int lane = threadIdx.x & 31;
    SelectOut r;
    r.tie_cut = 0;
    for (int i = lane; i < kHistBins; i += 32) wh[i] = 0u;
    __syncwarp();
    for (int i = lane; i < n; i += 32) {
        const uint32_t k = src.key(i);
        if (k) atomicAdd(&wh[logbin(kmax - k)], 1u);
    }
    __syncwarp();
    WarpFind f = warp_find_reg<kHistBins>(wh, (uint32_t)K);
    r.n_valid = f.total;
    if (f.total <= (uint32_t)K) {
        r.kth_key = 0u;
        r.kth_tb = 0xFFFFFFFFu;
        __syncwarp();
        return r;
    }
    uint32_t need = (uint32_t)K - f.before;
    uint32_t dlo;
    int bits;
    logbin_range(f.g, &dlo, &bits);
    const uint32_t width = 1u << bits;
    __syncwarp();
    if (f.cnt_g <= 32u) {
        // Few elements in the boundary bin: gather them one per lane and rank them
        // exactly in the composite order (key desc, tb asc).
        uint32_t mk = 0u, mt = 0xFFFFFFFFu;
        int got = 0;
        for (int base = 0; base < n; base += 32) {
            const int i = base + lane;
            uint32_t k = 0u, t = 0u;
            bool in = false;
            if (i < n) {
                k = src.key(i);
                in = k != 0u && ((kmax - k) - dlo) < width;
                if (in) t = src.tb(i);
            }
            const unsigned m = __ballot_sync(FULL, in);
            const int pos = got + __popc(m & lanemask_lt());
            // Lane `pos` receives this element.
            for (unsigned mm = m; mm; mm &= mm - 1) {
                const int src_l = __ffs(mm) - 1;
                const int dst = got + __popc(m & ((1u << src_l) - 1u));
                const uint32_t kk = __shfl_sync(FULL, k, src_l);
                const uint32_t tt = __shfl_sync(FULL, t, src_l);
                if (lane == dst) {
                    mk = kk;
                    mt = tt;
                }
            }
            (void)pos;
            got += __popc(m);
        }
        // rank = number of gathered elements that beat mine
        int rank = 0;
        for (int j = 0; j < got; ++j) {
            const uint32_t kj = __shfl_sync(FULL, mk, j);
            const uint32_t tj = __shfl_sync(FULL, mt, j);
            rank += (kj > mk || (kj == mk && tj < mt)) ? 1 : 0;
        }
        const unsigned hit = __ballot_sync(FULL, lane < got && rank == (int)need - 1);
        const int hl = __ffs(hit) - 1;
        r.kth_key = __shfl_sync(FULL, mk, hl);
        r.kth_tb = __shfl_sync(FULL, mt, hl);
        // Tie cut: some gathered element with the same key ranks below the K-th.
        const bool cut = lane < got && mk == r.kth_key && rank > (int)need - 1;
        r.tie_cut = __any_sync(FULL, cut) ? 1 : 0;
        if (!r.tie_cut) r.kth_tb = 0xFFFFFFFFu;  // every element equal to kth_key is taken
        return r;
    }
    uint32_t n_eq = f.cnt_g;
    while (bits > 0) {
        const int w = bits < 8 ? bits : 8;
        const int shift = bits - w;
        const uint32_t wd = 1u << bits;
        for (int i = lane; i < 256; i += 32) wh[i] = 0u;
        __syncwarp();
        for (int i = lane; i < n; i += 32) {
            const uint32_t k = src.key(i);
            if (k) {
                const uint32_t dd = (kmax - k) - dlo;
                if (dd < wd) atomicAdd(&wh[dd >> shift], 1u);
            }
        }
        __syncwarp();
        f = warp_find_reg<256>(wh, need);
        __syncwarp();
        n_eq = f.cnt_g;
        dlo += (uint32_t)f.g << shift;
        need -= f.before;
        bits = shift;
    }
    r.kth_key = kmax - dlo;
    if (need == n_eq) {
        r.kth_tb = 0xFFFFFFFFu;
        return r;
    }
    r.tie_cut = 1;
    uint32_t tlo = 0u;
    int tbits = tb_bits;
    while (tbits > 0) {
        const int w = tbits < 8 ? tbits : 8;
        const int shift = tbits - w;
        const uint32_t hi_mask = tbits >= 32 ? 0u : (0xFFFFFFFFu << tbits);
        for (int i = lane; i < 256; i += 32) wh[i] = 0u;
        __syncwarp();
        for (int i = lane; i < n; i += 32) {
            if (src.key(i) == r.kth_key) {
                const uint32_t t = src.tb(i);
                if (((t ^ tlo) & hi_mask) == 0u) atomicAdd(&wh[(t >> shift) & ((1u << w) - 1u)], 1u);
            }
        }
        __syncwarp();
        f = warp_find_reg<256>(wh, need);
        __syncwarp();
        tlo |= (uint32_t)f.g << shift;
        need -= f.before;
        tbits = shift;
    }
    r.kth_tb = tlo;
    return r;
}

// ---------------------------------------------------------------------------------
// Warp sorting networks on 64-bit composites (key << 32 | ~index): larger = better,
// so ties go to the lower index; 0 = empty. A warp array of N = 32*R elements keeps
// element i = r*32 + lane in register r of lane `lane`.
// ---------------------------------------------------------------------------------
__device__ __forceinline__ uint64_t shfl_xor64(uint64_t v, int m) {
    const uint32_t lo = __shfl_xor_sync(FULL, (uint32_t)v, m);
    const uint32_t hi = __shfl_xor_sync(FULL, (uint32_t)(v >> 32), m);
    return ((uint64_t)hi << 32) | lo;
}
__device__ __forceinline__ uint64_t shfl64(uint64_t v, int src) {
    const uint32_t lo = __shfl_sync(FULL, (uint32_t)v, src);
    const uint32_t hi = __shfl_sync(FULL, (uint32_t)(v >> 32), src);
    return ((uint64_t)hi << 32) | lo;
}
__device__ __forceinline__ uint64_t comp_key(uint32_t key, uint32_t idx) {
    return ((uint64_t)key << 32) | (uint64_t)(~idx);
}

// One compare-exchange stage (distance J) of a descending bitonic network whose
// sub-sequences of length KB alternate direction (KB = 0: every block descending).
// KB and J are compile-time so that every register index is static.
template <int R, int KB, int J>
__device__ __forceinline__ void bitonic_stage(uint64_t (&a)[R]) {
    const int lane = threadIdx.x & 31;
    if constexpr (J >= 32) {
        constexpr int RJ = J >> 5;
#pragma unroll
        for (int r = 0; r < R; ++r) {
            if ((r ^ RJ) > r) {
                const int i = r * 32 + lane;
                const bool desc = KB == 0 || (i & KB) == 0;
                const uint64_t x = a[r], y = a[r ^ RJ];
                const bool sw = desc ? (x < y) : (x > y);
                a[r] = sw ? y : x;
                a[r ^ RJ] = sw ? x : y;
            }
        }
    } else {
#pragma unroll
        for (int r = 0; r < R; ++r) {
            const int i = r * 32 + lane;
            const uint64_t y = shfl_xor64(a[r], J);
            const bool desc = KB == 0 || (i & KB) == 0;
            const bool lower = (lane & J) == 0;
            a[r] = (lower == desc) ? max(a[r], y) : min(a[r], y);
        }
    }
}
template <int R, int KB, int J>
__device__ __forceinline__ void bitonic_stages(uint64_t (&a)[R]) {
    if constexpr (J > 0) {
        bitonic_stage<R, KB, J>(a);
        bitonic_stages<R, KB, J / 2>(a);
    }
}
template <int R, int KK>
__device__ __forceinline__ void bitonic_levels(uint64_t (&a)[R]) {
    if constexpr (KK <= 32 * R) {
        bitonic_stages<R, (KK == 32 * R ? 0 : KK), KK / 2>(a);
        bitonic_levels<R, KK * 2>(a);
    }
}

// Sorts the warp array descending.
template <int R>
__device__ __forceinline__ void warp_sort_desc(uint64_t (&a)[R]) {
    bitonic_levels<R, 2>(a);
}

// a, b sorted descending -> a = the 32*R largest of a and b, sorted descending.
// Returns the largest element dropped (key part only), for tie bookkeeping.
template <int R>
__device__ __forceinline__ uint64_t warp_merge_desc(uint64_t (&a)[R], const uint64_t (&b)[R]) {
    const int lane = threadIdx.x & 31;
    uint64_t dropped = 0;
#pragma unroll
    for (int r = 0; r < R; ++r) {
        const uint64_t br = shfl64(b[R - 1 - r], 31 - lane);
        dropped = max(dropped, min(a[r], br));
        a[r] = max(a[r], br);
    }
    bitonic_stages<R, 0, 16 * R>(a);
    uint32_t hi = __reduce_max_sync(FULL, (uint32_t)(dropped >> 32));
    return (uint64_t)hi << 32;
}

// Element i of a warp array (broadcast to all lanes).
template <int R>
__device__ __forceinline__ uint64_t warp_elem(const uint64_t (&a)[R], int i) {
    uint64_t v = 0;
#pragma unroll
    for (int r = 0; r < R; ++r)
        if (r == (i >> 5)) v = a[r];
    return shfl64(v, i & 31);
}

#ifdef VDXS_TIMING
// Development self-test of the sorting networks: sorts/merges n_tests arrays.
template <int R>
__global__ void warp_network_selftest(const uint64_t* in, uint64_t* out_sorted, uint64_t* out_merged, int n_tests) {
    const int lane = threadIdx.x & 31;
    const int t = blockIdx.x * (blockDim.x / 32) + (threadIdx.x >> 5);
    if (t >= n_tests) return;
    uint64_t a[R], b[R];
#pragma unroll
    for (int r = 0; r < R; ++r) {
        a[r] = in[(size_t)t * 64 * R + r * 32 + lane];
        b[r] = in[(size_t)t * 64 * R + 32 * R + r * 32 + lane];
    }
    warp_sort_desc<R>(a);
    warp_sort_desc<R>(b);
#pragma unroll
    for (int r = 0; r < R; ++r) out_sorted[(size_t)t * 32 * R + r * 32 + lane] = a[r];
    warp_merge_desc<R>(a, b);
#pragma unroll
    for (int r = 0; r < R; ++r) out_merged[(size_t)t * 32 * R + r * 32 + lane] = a[r];
}
#endif

// Moves the selected entries of (k, t)[0..n) to the front, in order; returns the count.
__device__ __forceinline__ int warp_compact_selected(uint32_t* k, uint32_t* t, int n, const SelectOut& s) {
    const int lane = threadIdx.x & 31;
    int out = 0;
    for (int base = 0; base < n; base += 32) {
        const int i = base + lane;
        uint32_t kk = 0u, tt = 0u;
        bool sel = false;
        if (i < n) {
            kk = k[i];
            tt = t[i];
            sel = selected(kk, tt, s);
        }
        const unsigned m = __ballot_sync(FULL, sel);
        __syncwarp();
        if (sel) {
            const int pos = out + __popc(m & lanemask_lt());
            k[pos] = kk;
            t[pos] = tt;
        }
        out += __popc(m);
        __syncwarp();
    }
    return out;
}

// ---------------------------------------------------------------------------------
// Threshold histogram of the stream kernel. Bins are the top 12 bits of the key (sign,
// exponent and 3 mantissa bits); groups are the top 6 bits (64 bins each). Every count
// is of distinct elements of one row, so any bin edge with at least K counted elements
// at or above it is a lower bound on that row's K-th key.
// ---------------------------------------------------------------------------------
constexpr int kTBins = 4096;
constexpr int kTGroups = 64;

__device__ __forceinline__ void lds_v2_volatile(const uint32_t* a, uint32_t& x, uint32_t& y) {
    asm volatile("ld.volatile.shared.v2.u32 {%0, %1}, [%2];" : "=r"(x), "=r"(y) : "r"(smem_u32(a)));
}

// Inclusive suffix sum over lanes: lane l receives the sum of lanes l..31.
__device__ __forceinline__ uint32_t warp_suffix_sum(uint32_t v) {
    const int lane = threadIdx.x & 31;
#pragma unroll
    for (int d = 1; d < 32; d <<= 1) {
        const uint32_t o = __shfl_down_sync(FULL, v, d);
        if (lane + d < 32) v += o;
    }
    return v;
}

// Largest bin lower edge (a key) with at least K counted elements at or above it, or 0.
// Counts only grow, so reads that race with increments can only make the edge lower.
__device__ __forceinline__ uint32_t hist_threshold(const uint32_t* H, const uint32_t* G, int K) {
    const int lane = threadIdx.x & 31;
    uint32_t g0, g1;
    lds_v2_volatile(G + 2 * lane, g0, g1);
    const uint32_t s = warp_suffix_sum(g0 + g1);  // count in groups >= 2*lane
    const unsigned m0 = __ballot_sync(FULL, s >= (uint32_t)K);
    if (m0 == 0u) return 0u;
    const unsigned m1 = __ballot_sync(FULL, s - g0 >= (uint32_t)K);  // groups >= 2*lane+1
    const int l0 = 31 - __clz((int)m0);
    const int hi = (int)((m1 >> l0) & 1u);
    const int grp = 2 * l0 + hi;
    const uint32_t s_l0 = __shfl_sync(FULL, s, l0);
    const uint32_t g0_l0 = __shfl_sync(FULL, g0, l0);
    const uint32_t s_next = __shfl_sync(FULL, s, (l0 + 1) & 31);
    const uint32_t above = hi ? (l0 < 31 ? s_next : 0u) : s_l0 - g0_l0;  // count in groups > grp
    uint32_t h0, h1;
    lds_v2_volatile(H + grp * 64 + 2 * lane, h0, h1);
    const uint32_t t = warp_suffix_sum(h0 + h1) + above;
    const unsigned n0 = __ballot_sync(FULL, t >= (uint32_t)K);
    if (n0 == 0u) return (uint32_t)grp << 26;  // the group count qualified, its bins not yet
    const unsigned n1 = __ballot_sync(FULL, t - h0 >= (uint32_t)K);
    const int j0 = 31 - __clz((int)n0);
    return (uint32_t)(grp * 64 + 2 * j0 + (int)((n1 >> j0) & 1u)) << 20;
}

// Float threshold for "key >= k". Bin edges below the key of -inf (0x007FFFFF) are
// NaN bit patterns as floats; every non-NaN value is at or above them.
__device__ __forceinline__ float key_threshold(uint32_t k) { return k > 0x007FFFFFu ? key2f(k) : -INFINITY; }

__device__ __forceinline__ float fmax3f(float a, float b, float c) {
    float d;
    asm("max.f32 %0, %1, %2, %3;" : "=f"(d) : "f"(a), "f"(b), "f"(c));
    return d;
}

// Maximum of the 16 register values of a lane (NaN marks an empty slot and is ignored).
__device__ __forceinline__ float max16(const float (&x)[16]) {
    const float a = fmax3f(x[0], x[1], x[2]), b = fmax3f(x[3], x[4], x[5]), c = fmax3f(x[6], x[7], x[8]);
    const float d = fmax3f(x[9], x[10], x[11]), e = fmax3f(x[12], x[13], x[14]);
    return fmaxf(fmax3f(a, b, c), fmax3f(d, e, x[15]));
}

// ---------------------------------------------------------------------------------
// Small batches: one thread-block cluster of CL CTAs per row. Each CTA copies its 1/CL
// of the row into its own shared memory (plain bulk copies of this CTA's part), masks
// the penalised ids, and sends each thread's maximum to the leader CTA through
// distributed shared memory. The leader takes the K-th largest of those maxima, a lower
// bound on the row's K-th key (they are distinct elements of the row); every CTA then
// sends the leader its elements at or above it, or, if more than its slot holds, its
// exact top-K with tie evidence. The leader runs stage 2 on what it gathered.
// ---------------------------------------------------------------------------------
constexpr int kClusterCTAs = 8;     // CTAs per row's cluster (portable size)
constexpr int kClusterMaxRows = 8;  // batches up to this size take the cluster path
constexpr int kClusterMaxWords = 8 * NT;  // thread-maxima area (then the warps' send batches)

template <typename T>
__device__ __forceinline__ T nan_bits();
template <>
__device__ __forceinline__ float nan_bits<float>() { return __uint_as_float(0x7FC00000u); }
template <>
__device__ __forceinline__ uint16_t nan_bits<uint16_t>() { return (uint16_t)0x7FC0u; }

// ---------------------------------------------------------------------------------
// Stream stage 1 (topk_stream_kernel): every top_k of the top-k path, and greedy.
//
// Work: each row is cut into 4 KB slots (1024 fp32 or 2048 bf16 elements) and its slots
// into units of p.unit_slots consecutive slots. Warps claim units one at a time from a
// global counter, in column-major order (unit u is row u % B, segment u / B): every
// row's first segments are streamed first, so later segments start from a bound that
// earlier segments of the same row have already raised, and no SM waits on a static
// share of the work. There is no CTA-wide synchronisation: every warp runs on its own.
//
// Loading: each warp streams its slots through its own two-slot ring of bulk copies.
// Lane l owns the slot's l-th 128-byte group and reads it as eight 16-byte chunks in a
// rotated order (conflict-free); it keeps the maxima of its chunks, so one compare of the
// lane maximum decides the whole group. Few hot lanes: the warp tests each hot group
// together from shared memory. Many: each lane extracts its own candidates from its
// registers, testing only chunks whose maximum reaches the bound.
//
// Bound: one key histogram per row in global memory (top 12 key bits, and 64 group
// counts), counted with fire-and-forget atomics by every warp working on the row. Every
// count is of a distinct element of the row, so the highest bin edge with at least K
// counts at or above it is a lower bound on the row's K-th key. Candidates are counted
// as they are taken (not those in the bound's own bin, which cannot raise it), and the
// first slot of each unit is filtered against the K-th largest of its chunk maxima as
// well (top_k <= 256). A warp raises the row bound (row_tau, atomicMax) from the
// histogram asynchronously: the group counts are read at the end of a slot, the bin
// counts at the start of the next, and the raise completes at that slot's end.
//
// Output: one list per row. Candidates wait in a per-warp shared region and are written
// out when it fills and at the end of each unit if they still reach the bound then. The
// final row bound is the largest bound any warp published, and every element at or
// above it is in the list (an element at or above it was at or above every bound it was
// tested or flushed against). row_cnt counts the list; a count above cand_cap marks it
// incomplete and sends the row to the finish kernel's exact fallback. The finish kernel
// resets the row's histogram, count and bound, and the claim counter, for the next call.
// ---------------------------------------------------------------------------------
constexpr int kS1Threads = 512;
constexpr int kS1Warps = kS1Threads / 32;
constexpr int kS1SlotBytes = 4096;                    // one bulk copy; a 128-byte group per lane
constexpr int kS1Ring = 2;                            // ring slots per warp
constexpr int kS1WCap = 128;                          // region entries per warp
constexpr int kS1CoopLanes = 8;                       // up to this many hot lanes: warp-cooperative test
constexpr int kS1RaiseEvery = 1;                      // counted candidates between bound raises
constexpr int kRowHistWords = kTBins + kTGroups;      // per-row histogram in global memory
constexpr int kS1WarpBytes = kS1Ring * kS1SlotBytes + 64 + 8 * kS1WCap + 4 * 256;
static_assert(kS1WarpBytes % 16 == 0, "16-byte aligned warp areas");

#include "vdxs_large_topk.cuh"

__host__ __device__ constexpr size_t s1_smem_bytes() { return (size_t)kS1Warps * kS1WarpBytes; }
template <typename T>
__host__ __device__ constexpr int s1_slot_elems() { return kS1SlotBytes / (int)sizeof(T); }

__device__ __forceinline__ uint32_t bmax2(uint32_t a, uint32_t b) {  // packed bf16 max (NaN ignored)
    uint32_t d;
    asm("max.bf16x2 %0, %1, %2;" : "=r"(d) : "r"(a), "r"(b));
    return d;
}
__device__ __forceinline__ float bf_lo(uint32_t w) { return __uint_as_float(w << 16); }
__device__ __forceinline__ float bf_hi(uint32_t w) { return __uint_as_float(w & 0xFFFF0000u); }
__device__ __forceinline__ void red_add_u32(uint32_t* a, uint32_t v) {
    asm volatile("red.relaxed.gpu.global.add.u32 [%0], %1;" ::"l"(a), "r"(v) : "memory");
}
__device__ __forceinline__ uint2 ld_relaxed_v2(const uint32_t* p) {
    uint2 v;
    asm volatile("ld.relaxed.gpu.global.v2.u32 {%0, %1}, [%2];" : "=r"(v.x), "=r"(v.y) : "l"(p) : "memory");
    return v;
}

// Element e of a 16-byte chunk (4 fp32 or 8 bf16 values; e is a compile-time constant).
template <typename T>
__device__ __forceinline__ float chunk_elem(const uint4& v, int e) {
    if constexpr (sizeof(T) == 4) {
        return __uint_as_float(e == 0 ? v.x : e == 1 ? v.y : e == 2 ? v.z : v.w);
    } else {
        const uint32_t w = (e >> 1) == 0 ? v.x : (e >> 1) == 1 ? v.y : (e >> 1) == 2 ? v.z : v.w;
        return (e & 1) ? bf_hi(w) : bf_lo(w);
    }
}
template <typename T>
__device__ __forceinline__ float chunk_max(const uint4& v) {
    if constexpr (sizeof(T) == 4) {
        return fmaxf(fmax3f(__uint_as_float(v.x), __uint_as_float(v.y), __uint_as_float(v.z)), __uint_as_float(v.w));
    } else {
        const uint32_t m = bmax2(bmax2(v.x, v.y), bmax2(v.z, v.w));
        return fmaxf(bf_lo(m), bf_hi(m));
    }
}

// One warp: a lower bound on the K-th largest of 8 keys per lane (key 0 = no element),
// with the low 16 bits cleared: two radix passes of 8 bits over a 256-word warp-private
// histogram. Returns 0 when fewer than K keys are valid.
__device__ uint32_t warp_kth_of_keys8(const uint32_t (&k)[8], int K, uint32_t* wh) {
    const int lane = threadIdx.x & 31;
    uint32_t prefix = 0u, need = (uint32_t)K;
#pragma unroll
    for (int pass = 0; pass < 2; ++pass) {
        const int shift = 24 - 8 * pass;
        reinterpret_cast<uint4*>(wh)[2 * lane] = make_uint4(0u, 0u, 0u, 0u);
        reinterpret_cast<uint4*>(wh)[2 * lane + 1] = make_uint4(0u, 0u, 0u, 0u);
        __syncwarp();
#pragma unroll
        for (int j = 0; j < 8; ++j)
            if (k[j] != 0u && (pass == 0 || (k[j] >> 24) == (prefix >> 24))) atomicAdd(&wh[(k[j] >> shift) & 255u], 1u);
        __syncwarp();
        const uint4 a = reinterpret_cast<const uint4*>(wh)[2 * lane];
        const uint4 c = reinterpret_cast<const uint4*>(wh)[2 * lane + 1];
        const uint32_t cnt[8] = {a.x, a.y, a.z, a.w, c.x, c.y, c.z, c.w};
        const uint32_t mine = a.x + a.y + a.z + a.w + c.x + c.y + c.z + c.w;
        const uint32_t suf = warp_suffix_sum(mine);  // counts in bins >= 8 * lane
        const unsigned m = __ballot_sync(FULL, suf >= need);
        __syncwarp();
        if (m == 0u) return pass == 0 ? 0u : prefix;
        const int l0 = 31 - __clz((int)m);  // lane holding the bin that reaches `need`
        uint32_t above = __shfl_sync(FULL, suf - mine, l0);  // counts in bins >= 8 * (l0 + 1)
        int bin = 8 * l0;
        if (lane == l0) {
            uint32_t s = above;
            int j = 7;
            for (; j > 0; --j) {
                if (s + cnt[j] >= need) break;
                s += cnt[j];
            }
            bin += j;
            above = s;
        }
        bin = __shfl_sync(FULL, bin, l0);
        above = __shfl_sync(FULL, above, l0);
        prefix |= (uint32_t)bin << shift;
        need -= above;
    }
    return prefix;
}

// Development counters of topk_stream_kernel (-DVDXS_TIMING builds only): each warp sums
// its phase cycles and event counts in registers and adds them once at the end
// (g_phase_cycles[40 + i]), so the counting barely perturbs the kernel.
#ifdef VDXS_TIMING
#define S1_DBG_DECL unsigned long long s1dbg[16] = {0}
#define S1_ADD(i, v) (s1dbg[i] += (unsigned long long)(v))
#define S1_T0(v) long long v = clock64()
#define S1_T1(i, v) (s1dbg[i] += (unsigned long long)(clock64() - v))
#define S1_FLUSH()                                                               \
    do {                                                                         \
        if ((threadIdx.x & 31) == 0)                                             \
            for (int i_ = 0; i_ < 16; ++i_) atomicAdd(&g_phase_cycles[40 + i_], s1dbg[i_]); \
    } while (0)
#else
#define S1_DBG_DECL \
    do {            \
    } while (0)
#define S1_ADD(i, v) \
    do {             \
    } while (0)
#define S1_T0(v) \
    do {         \
    } while (0)
#define S1_T1(i, v) \
    do {            \
    } while (0)
#define S1_FLUSH() \
    do {           \
    } while (0)
#endif

template <typename T, bool TMA>
__global__ void __launch_bounds__(kS1Threads, 1) topk_stream_kernel(KParams p) {
    extern __shared__ __align__(16) unsigned char smem_raw[];
    S1_DBG_DECL;
    S1_T0(t_all);
    constexpr int SE = s1_slot_elems<T>();  // elements per slot
    constexpr int GE = SE / 32;             // elements per lane group
    constexpr int CE = GE / 8;              // elements per 16-byte chunk
    const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
    const int sw = lane & 7;
    const int K = p.K;
    unsigned char* wa = smem_raw + (size_t)warp * kS1WarpBytes;
    unsigned char* ring = wa;
    uint64_t* full = (uint64_t*)(wa + kS1Ring * kS1SlotBytes);
    int32_t* wq = (int32_t*)(full + kS1Ring);  // [kS1Ring][2]: (row, slot) staged in each ring slot
    uint32_t* rkey = (uint32_t*)(wa + kS1Ring * kS1SlotBytes + 64);
    uint32_t* ridx = rkey + kS1WCap;
    uint32_t* wh = ridx + kS1WCap;  // 256-word warp histogram (first-slot bound)
    const int ng = p.flat_ng;       // slots per row
    const int U = p.unit_slots;     // slots per row segment
    const int nseg = (ng + U - 1) / U;
    // Slot enumeration, column-major over row segments: position g is segment
    // g / (B * U), row (g / U) % B, slot (g / (B * U)) * U + g % U of that row (positions past
    // the row's last slot are skipped).
    const uint32_t ne = (uint32_t)p.B * (uint32_t)nseg * (uint32_t)U;  // below 2^31 (host check)
    const uint32_t nwarps = gridDim.x * (uint32_t)kS1Warps;

    // Producer (lane 0): claims runs of positions and issues the ring's bulk copies in order.
    // Runs are U positions long until the remaining work nears two runs per warp, then
    // shrink to one slot, so that warps run out of work together.
    uint32_t cg = 0u, ce = 0u;   // the producer's claimed run [cg, ce)
    uint32_t ng0 = 0u, nc = 0u;  // the next run, claimed one run ahead: start (atomic result) and length
    bool have_next = false;
    uint32_t pn = 0;             // copies issued
    bool pr_done = false;
    // Every warp's first run is assigned statically (warp w takes [w * c0, (w + 1) * c0)),
    // so the launch does not start with every warp claiming from one counter; claims from
    // the counter start after those runs.
    const uint32_t c0 = max(1u, min((uint32_t)U, ne / (2u * nwarps)));
    const uint32_t base = c0 * nwarps;
    const uint32_t guide_full = (uint32_t)U * 2u * nwarps;  // below this, runs shrink
    auto claim_next = [&](uint32_t left_est) {
        nc = left_est >= guide_full ? (uint32_t)U : max(1u, left_est / (2u * nwarps));
        ng0 = base + (uint32_t)atomicAdd((unsigned long long*)p.unit_next, (unsigned long long)nc);
        have_next = true;
    };
    {
        ng0 = (blockIdx.x * (uint32_t)kS1Warps + (threadIdx.x >> 5)) * c0;
        nc = c0;
        have_next = true;
    }
    // Position of cg within the enumeration: segment, row and slot offset, advanced
    // incrementally (one division per run).
    int cseg = 0, crow = 0, ct = 0;
    auto issue = [&]() {
        int pr_row = -1, pr_q = 0;
        while (!pr_done) {
            if (cg >= ce) {
                if (!have_next) claim_next(ne);
                // Move to the run claimed ahead (its atomic result is first needed here),
                // and claim the one after it.
                cg = ng0;
                ce = min(ng0 + nc, ne);
                have_next = false;
                if (cg >= ne) {
                    pr_done = true;
                    break;
                }
                claim_next(ne - ce);
                const uint32_t su = cg / (uint32_t)U;
                ct = (int)(cg - su * (uint32_t)U);
                cseg = (int)(su / (uint32_t)p.B);
                crow = (int)(su - (uint32_t)cseg * (uint32_t)p.B);
            }
            const int q = cseg * U + ct;
            const int r = crow;
            ++cg;
            if (++ct == U) {
                ct = 0;
                if (++crow == p.B) {
                    crow = 0;
                    ++cseg;
                }
            }
            if (q < ng) {
                pr_row = r;
                pr_q = q;
                break;
            }
        }
        const int s = (int)(pn % kS1Ring);
        if (pr_done) {
            wq[2 * s] = -1;  // no more work
            mbar_arrive(&full[s]);
        } else {
            const int64_t e0 = (int64_t)pr_q * SE;
            const int n = (int)min((int64_t)SE, (int64_t)p.V - e0);
            const uint32_t bytes = ((uint32_t)n * (uint32_t)sizeof(T)) & ~15u;
            wq[2 * s] = pr_row;
            wq[2 * s + 1] = pr_q;
            if (TMA && bytes) {
                mbar_arrive_expect_tx(&full[s], bytes);
                tma_load_1d(ring + s * kS1SlotBytes, (const T*)p.logits + (int64_t)pr_row * p.stride + e0, bytes,
                            &full[s]);
            } else {
                mbar_arrive(&full[s]);
            }
        }
        ++pn;
    };
    if (lane == 0) {
        for (int s = 0; s < kS1Ring; ++s) mbar_init(&full[s], 1);
        fence_mbar_init();
    }
    __syncwarp();
    // With a history, this kernel is a programmatic dependent of the penalty prep; the
    // penalty lists are read only after this wait (a no-op for an ordinary launch). The
    // claim counter is reset by the previous call's finish kernel, so claims come after.
    asm volatile("griddepcontrol.wait;" ::: "memory");
    if (lane == 0)
        for (int s = 0; s < kS1Ring; ++s) issue();
    __syncwarp();

    uint32_t cn = 0;  // slots consumed (ring position and phase)
    bool timed_out = false;
    // Current row of the consumer (-1: none yet).
    int row = -1;
    const T* rowp = nullptr;
    uint32_t* rtp = nullptr;
    uint32_t* rh = nullptr;  // the row's histogram
    uint2* out = nullptr;
    uint32_t* rcnt = nullptr;
    const uint32_t cap = (uint32_t)p.cand_cap;
    uint32_t rtau = 0u, rtau_next = 0u, lbound = 0u, wcnt = 0u, since = 0u;
    // Asynchronous bound raise: 0 idle, 1 group counts in flight, 2 bin counts in flight.
    // The raise keeps its row's pointers, so it completes after the warp moves on.
    int rs_state = 0;
    uint2 rs_g = make_uint2(0u, 0u), rs_h = make_uint2(0u, 0u);
    int rs_grp = 0;
    uint32_t rs_above = 0u;
    const uint32_t* rs_rh = nullptr;
    uint32_t* rs_rtp = nullptr;

    // Writes the region entries at or above tmin to the row's list; empties the region.
    auto flush_region = [&](uint32_t tmin) {
        S1_ADD(10, 1);
        for (uint32_t i0 = 0; i0 < wcnt; i0 += 32) {
            const uint32_t i = i0 + lane;
            uint32_t k = 0u, ix = 0u;
            bool keep = false;
            if (i < wcnt) {
                k = rkey[i];
                ix = ridx[i];
                keep = k >= tmin;
            }
            const unsigned m = __ballot_sync(FULL, keep);
            if (m) {
                uint32_t base = 0u;
                if (lane == 0) base = atomicAdd(rcnt, (uint32_t)__popc(m));
                base = __shfl_sync(FULL, base, 0);
                const uint32_t pos = base + __popc(m & lanemask_lt());
                if (keep && pos < cap) out[pos] = make_uint2(k, ix);
            }
        }
        __syncwarp();
        wcnt = 0u;
    };
    auto cur_bound = [&]() -> uint32_t { return max(rtau, lbound); };
    // Advances the asynchronous raise by one step (called once per slot).
    auto raise_step = [&]() {
        if (rs_state == 1) {
            const uint32_t s = warp_suffix_sum(rs_g.x + rs_g.y);  // counts in groups >= 2 * lane
            const unsigned m0 = __ballot_sync(FULL, s >= (uint32_t)K);
            if (m0 == 0u) {
                rs_state = 0;
                return;
            }
            const unsigned m1 = __ballot_sync(FULL, s - rs_g.x >= (uint32_t)K);
            const int l0 = 31 - __clz((int)m0);
            const int hi = (int)((m1 >> l0) & 1u);
            rs_grp = 2 * l0 + hi;
            const uint32_t s_l0 = __shfl_sync(FULL, s, l0);
            const uint32_t g0_l0 = __shfl_sync(FULL, rs_g.x, l0);
            const uint32_t s_next = __shfl_sync(FULL, s, (l0 + 1) & 31);
            rs_above = hi ? (l0 < 31 ? s_next : 0u) : s_l0 - g0_l0;  // counts in groups > grp
            rs_h = ld_relaxed_v2(rs_rh + rs_grp * 64 + 2 * lane);
            rs_state = 2;
        } else if (rs_state == 2) {
            const uint32_t t = warp_suffix_sum(rs_h.x + rs_h.y) + rs_above;
            const unsigned n0 = __ballot_sync(FULL, t >= (uint32_t)K);
            uint32_t edge = (uint32_t)rs_grp << 26;  // the group qualified, its bins not yet
            if (n0 != 0u) {
                const unsigned n1 = __ballot_sync(FULL, t - rs_h.x >= (uint32_t)K);
                const int j0 = 31 - __clz((int)n0);
                edge = (uint32_t)(rs_grp * 64 + 2 * j0 + (int)((n1 >> j0) & 1u)) << 20;
            }
            if (rs_rtp == rtp) {
                if (edge > rtau) {
                    rtau = edge;
                    if (lane == 0) atomicMax(rtp, edge);
                }
            } else if (lane == 0) {
                atomicMax(rs_rtp, edge);
            }
            rs_state = 0;
        }
    };
    auto raise_start = [&]() {
        if (rs_state == 0) {
            S1_ADD(9, 1);
            rs_rh = rh;
            rs_rtp = rtp;
            rs_g = ld_relaxed_v2(rh + kTBins + 2 * lane);
            rs_state = 1;
        }
    };
    // Leaves the current row: the region entries at or above the warp's bound are written
    // to the list and the bound is published.
    auto leave_row = [&]() {
        if (row < 0) return;
        const uint32_t tb = cur_bound();
        flush_region(tb);
        if (lane == 0 && tb > rtau) atomicMax(rtp, tb);
        row = -1;
    };
    // The bound of the row that the next staged slot belongs to, read one slot early.
    int pref_row = -1;
    uint32_t pref_tau = 0u;
    auto enter_row = [&](int b) {
        row = b;
        rowp = (const T*)p.logits + (int64_t)b * p.stride;
        rtp = p.row_tau + (size_t)b * kTauStride;
        rh = p.rhist + (size_t)b * kRowHistWords;
        out = p.cand + (size_t)b * cap;
        rcnt = p.row_cnt + b;
        rtau = b == pref_row ? pref_tau : ld_relaxed_u32(rtp);
        rtau_next = rtau;
        lbound = 0u;
        since = 0u;
    };

    int last_q = -2;
    for (;;) {
        // ---- stage the next slot of this warp's claimed sequence ----
        S1_T0(t_st);
        const int s = (int)(cn % kS1Ring);
        unsigned char* slotp = ring + s * kS1SlotBytes;
        T* sl = (T*)slotp;
        // The slot's (row, slot) entry was written by lane 0 before it issued the copy, in an
        // earlier iteration whose warp barriers order it before these reads: read it, and
        // the penalised-id bitmap words of this lane's group, before waiting for the copy.
        const int b = wq[2 * s], q = wq[2 * s + 1];
        uint32_t pbits[GE / 32];
#pragma unroll
        for (int w = 0; w < GE / 32; ++w) {
            const int wi = (int)(((int64_t)q * SE + lane * GE) >> 5) + w;
            pbits[w] = (p.pen_bits && b >= 0 && wi < p.pen_words) ? __ldcg(p.pen_bits + (size_t)b * p.pen_words + wi)
                                                                   : 0u;
        }
        if (!mbar_wait_bounded(&full[s], (cn / kS1Ring) & 1u)) {
            timed_out = true;
            break;
        }
        if (b < 0) break;  // no more units
        const bool first = b != row || q != last_q + 1;  // first slot of a claimed unit
        if (b != row) {
            S1_T0(t_sw);
            leave_row();
            enter_row(b);
            S1_T1(15, t_sw);
        }
        last_q = q;
        const int64_t start = (int64_t)q * SE;
        const int n = (int)min((int64_t)SE, (int64_t)p.V - start);
        {
            const int n_tma = TMA ? (int)((((uint32_t)n * (uint32_t)sizeof(T)) & ~15u) / sizeof(T)) : 0;
            // Elements the bulk copy did not bring (row tail, or every element without bulk
            // copies) are read directly; positions past the row hold NaN (no element).
            for (int i = n_tma + lane; i < SE; i += 32) sl[i] = i < n ? rowp[start + i] : nan_bits<T>();
        }
        // Penalised ids leave stage 1 (they re-enter with their penalised values in the
        // finish kernel): NaN in the staged slot.
#pragma unroll
        for (int w = 0; w < GE / 32; ++w) {
            uint32_t bits = pbits[w];
            while (bits) {
                const int i = __ffs((int)bits) - 1;
                bits &= bits - 1u;
                sl[lane * GE + w * 32 + i] = nan_bits<T>();
            }
        }
        __syncwarp();
        uint4 v[8];
        {
            const unsigned char* g = slotp + lane * 128;
#pragma unroll
            for (int c = 0; c < 8; ++c) v[c] = *reinterpret_cast<const uint4*>(g + ((c ^ sw) << 4));
        }
        {
            const int nb = wq[2 * (int)((cn + 1) % kS1Ring)];  // written before the last release
            if (nb >= 0 && nb != b && nb != pref_row) {
                pref_row = nb;
                pref_tau = ld_relaxed_u32(p.row_tau + (size_t)nb * kTauStride);
            }
        }
        S1_T1(0, t_st);
        S1_T0(t_rs);
        rtau = max(rtau, rtau_next);  // the row bound is fetched one slot ahead
        rtau_next = ld_relaxed_u32(rtp);
        raise_step();
        S1_T1(14, t_rs);
        float xq[8];
#pragma unroll
        for (int c = 0; c < 8; ++c) xq[c] = chunk_max<T>(v[c]);
        const float lmax = fmaxf(fmax3f(fmax3f(xq[0], xq[1], xq[2]), fmax3f(xq[3], xq[4], xq[5]), xq[6]), xq[7]);
        if (first && K <= 256 && __popc(__ballot_sync(FULL, lmax >= key_threshold(cur_bound()))) > kS1CoopLanes) {
            // The row's bound would let many lanes through: add the K-th largest chunk
            // maximum of this slot (distinct elements of the row) as a bound.
            S1_T0(t_cnt);
            uint32_t kk[8];
#pragma unroll
            for (int c = 0; c < 8; ++c) kk[c] = xq[c] == xq[c] ? f2key(xq[c]) : 0u;
            lbound = max(lbound, warp_kth_of_keys8(kk, K, wh));  // stays a bound of this row
            S1_T1(3, t_cnt);
        }

        // ---- filter the slot against the bound ----
        S1_ADD(5, 1);
        const uint32_t tg = cur_bound();
        const float thr = key_threshold(tg);
        const bool hot = lmax >= thr;
        unsigned hb = __ballot_sync(FULL, hot);
        if (hb != 0u) {
            S1_T0(t_hot);
            S1_ADD(6, 1);
            S1_ADD(7, __popc(hb));
            const uint32_t tbin = tg >> 20;
            const uint32_t gslot = (uint32_t)p.vocab_offset + (uint32_t)start;
            uint32_t counted = 0u;
            // Appends a candidate at region position pos and counts it in the row
            // histogram unless it lies in the bound's own bin.
            auto take = [&](uint32_t pos, uint32_t k, uint32_t ix) {
                rkey[pos] = k;
                ridx[pos] = ix;
                if ((k >> 20) > tbin) {
                    red_add_u32(rh + (k >> 20), 1u);
                    red_add_u32(rh + kTBins + (k >> 26), 1u);
                    ++counted;
                }
            };
            // The same count for one element per lane.
            auto count_step = [&](bool valid, uint32_t k) {
                if (valid && (k >> 20) > tbin) {
                    red_add_u32(rh + (k >> 20), 1u);
                    red_add_u32(rh + kTBins + (k >> 26), 1u);
                    ++counted;
                }
            };
            auto put = [&](uint32_t pos, uint32_t k, uint32_t ix) {
                rkey[pos] = k;
                ridx[pos] = ix;
            };
            if (__popc(hb) <= kS1CoopLanes) {
                while (hb) {
                    const int h = __ffs((int)hb) - 1;
                    hb &= hb - 1u;
                    if (wcnt + 2u * 32u > (uint32_t)kS1WCap) flush_region(tg);
                    if constexpr (sizeof(T) == 4) {
                        const float xv = reinterpret_cast<const float*>(slotp)[h * 32 + lane];
                        const bool pass = xv >= thr;
                        const unsigned m = __ballot_sync(FULL, pass);
                        const uint32_t k = f2key(xv);
                        if (pass) put(wcnt + __popc(m & lanemask_lt()), k, gslot + (uint32_t)(h * 32 + lane));
                        count_step(pass, k);
                        wcnt += (uint32_t)__popc(m);
                        S1_ADD(8, __popc(m));
                    } else {
                        const uint32_t w = reinterpret_cast<const uint32_t*>(slotp)[h * 32 + lane];
                        const float a = bf_lo(w), bb = bf_hi(w);
                        const bool pa = a >= thr, pb = bb >= thr;
                        const unsigned ma = __ballot_sync(FULL, pa), mb = __ballot_sync(FULL, pb);
                        const uint32_t pos = wcnt + __popc(ma & lanemask_lt()) + __popc(mb & lanemask_lt());
                        const uint32_t ix = gslot + (uint32_t)(h * 64 + 2 * lane);
                        const uint32_t ka = f2key(a), kb = f2key(bb);
                        if (pa) put(pos, ka, ix);
                        if (pb) put(pos + (pa ? 1u : 0u), kb, ix + 1u);
                        count_step(pa, ka);
                        count_step(pb, kb);
                        wcnt += (uint32_t)(__popc(ma) + __popc(mb));
                        S1_ADD(8, __popc(ma) + __popc(mb));
                    }
                }
            } else {
                // Bit i of pm: element i of this lane's group reaches the bound (only chunks
                // whose maximum reaches it are tested).
                uint64_t pm = 0ull;
                if (hot) {
#pragma unroll
                    for (int c = 0; c < 8; ++c) {
                        if (xq[c] >= thr) {
                            uint32_t cm = 0u;
#pragma unroll
                            for (int e = 0; e < CE; ++e) cm |= (chunk_elem<T>(v[c], e) >= thr ? 1u : 0u) << e;
                            pm |= (uint64_t)cm << ((c ^ sw) * CE);
                        }
                    }
                }
                const uint32_t cnt = (uint32_t)__popcll(pm);
                uint32_t incl = cnt;
#pragma unroll
                for (int d = 1; d < 32; d <<= 1) {
                    const uint32_t o = __shfl_up_sync(FULL, incl, d);
                    if (lane >= d) incl += o;
                }
                const uint32_t total = __shfl_sync(FULL, incl, 31);
                if (wcnt + total > (uint32_t)kS1WCap && wcnt > 0u) flush_region(tg);
                const bool direct = total > (uint32_t)kS1WCap;  // more than a region: straight to the list
                if (direct) S1_ADD(12, 1);
                uint32_t pos;
                if (direct) {
                    uint32_t base = 0u;
                    if (lane == 0) base = atomicAdd(rcnt, total);
                    pos = __shfl_sync(FULL, base, 0) + incl - cnt;
                } else {
                    pos = wcnt + incl - cnt;
                }
                // Each lane writes its own candidates, re-read from the staged slot.
                const T* grp = reinterpret_cast<const T*>(slotp) + lane * GE;
                const uint32_t gb = gslot + (uint32_t)lane * GE;
                while (pm) {
                    const int i = __ffsll((long long)pm) - 1;
                    pm &= pm - 1ull;
                    const uint32_t k = f2key(to_f(grp[i]));
                    const uint32_t ix = gb + (uint32_t)i;
                    if (direct) {
                        if (pos < cap) out[pos] = make_uint2(k, ix);
                        if ((k >> 20) > tbin) {
                            red_add_u32(rh + (k >> 20), 1u);
                            red_add_u32(rh + kTBins + (k >> 26), 1u);
                            ++counted;
                        }
                    } else {
                        take(pos, k, ix);
                    }
                    ++pos;
                }
                if (!direct) wcnt += total;
                S1_ADD(8, total);
            }
            since += __reduce_add_sync(FULL, counted);
            S1_T1(1, t_hot);
        }
        // A raise whose bin counts were requested at this slot's start completes here (the
        // filter hid the read), and the next one can start at once: one raise per slot.
        if (rs_state == 2) raise_step();
        if (since >= (uint32_t)kS1RaiseEvery && rs_state == 0) {
            since = 0u;
            raise_start();
        }

        // ---- release the slot: its next bulk copy goes behind the warp's reads ----
        S1_T0(t_rel);
        __syncwarp();
        if (lane == 0) {
            fence_proxy_async_smem();
            issue();
        }
        ++cn;
        S1_T1(13, t_rel);
    }
    leave_row();
    const bool any_timeout = __any_sync(FULL, timed_out);
    if (any_timeout && lane == 0) atomicExch(p.err, kErrTimeout);
    __syncwarp();
    // Every copy this warp issued has been consumed (the positions after the end-of-work
    // marker hold markers too, which complete on arrival), so the barriers are idle.
    if (!any_timeout && lane == 0)
        for (int s2 = 0; s2 < kS1Ring; ++s2) mbar_inval(&full[s2]);
    // The last warp of the grid to finish resets the claim counter for the next call:
    // all claims of this call precede every warp's fence and finish count.
    if (lane == 0) {
        __threadfence();
        if (atomicAdd(&p.unit_next[1], 1ull) == (unsigned long long)gridDim.x * kS1Warps - 1ull) {
            atomicExch(&p.unit_next[0], 0ull);
            atomicExch(&p.unit_next[1], 0ull);
        }
    }
    S1_T1(4, t_all);
    S1_FLUSH();
    // This CTA is done: the finish kernel may start launching (it waits for the grid).
    asm volatile("griddepcontrol.launch_dependents;" ::: "memory");
}

// Warp 0 only: the highest bin g of h[0..256) with at least `need` counts in bins >= g.
// Writes sh[0] = g (0xFFFFFFFF if the total is below need), sh[1] = count in bins > g.
__device__ void warp_suffix_find256(const uint32_t* h, uint32_t need, uint32_t* sh) {
    const int l = threadIdx.x & 31;
    uint32_t c[8], s = 0u;
#pragma unroll
    for (int u = 0; u < 8; ++u) {
        c[u] = h[8 * l + u];
        s += c[u];
    }
    const uint32_t suf = warp_suffix_sum(s);  // counts in bins >= 8l
    const unsigned m = __ballot_sync(FULL, suf >= need);
    if (m == 0u) {
        if (l == 0) sh[0] = 0xFFFFFFFFu;
        return;
    }
    if (l == 31 - __clz((int)m)) {
        uint32_t above = suf - s;  // counts in bins >= 8(l+1)
        int g = 8 * l;
        bool found = false;
#pragma unroll
        for (int u = 7; u >= 0; --u) {
            if (!found) {
                if (above + c[u] >= need) {
                    g = 8 * l + u;
                    found = true;
                } else {
                    above += c[u];
                }
            }
        }
        sh[0] = (uint32_t)g;
        sh[1] = above;
    }
}

template <typename T>
struct ChunkKeySrc {  // keys of a row chunk in shared memory (NaN: no element), tie-break = position
    const T* xs;
    int n;
    __device__ __forceinline__ uint32_t key(int i) const {
        if (i >= n) return 0u;
        const float v = to_f(xs[i]);
        return v == v ? f2key(v) : 0u;
    }
    __device__ __forceinline__ uint32_t tb(int i) const { return (uint32_t)i; }
};

template <typename T, bool TMA, int CL>
__global__ void __launch_bounds__(NT, 1) row_cluster_kernel(KParams p) {
    namespace cg = cooperative_groups;
    cg::cluster_group cl = cg::this_cluster();
    extern __shared__ __align__(16) unsigned char smem_raw[];
    __shared__ uint64_t s_bar;
    uint32_t* hist = (uint32_t*)smem_raw;
    uint32_t* sh = hist + kHistWords;
    unsigned char* region = smem_raw + kHeadBytes;
    const int tid = threadIdx.x, lane = tid & 31;
    const int r = (int)cl.block_rank();
    const int b = blockIdx.y;
    const int K = p.K;
    const int L = p.chunk;      // elements per CTA (a multiple of 16)
    const int cap = p.cand_cap; // candidate slots per CTA at the leader (>= K)
    const int64_t lo = (int64_t)r * L;
    const int n = (int)max((int64_t)0, min((int64_t)L, (int64_t)p.V - lo));
    T* xs = (T*)region;
    uint32_t* maxk = (uint32_t*)(region + p.span);  // p.span: bytes of the chunk area
    const int ncap = CL * cap + p.pen_stride;
    uint32_t* ckey = maxk + kClusterMaxWords;
    uint32_t* cidx = ckey + ncap;
    uint32_t* cuts = cidx + ncap;  // [CL]
    const T* row = (const T*)p.logits + (int64_t)b * p.stride;

    // 1. The chunk into shared memory.
    VDXS_T0(t_c1);
    bool timed_out = false;
    if constexpr (TMA) {
        const uint32_t bytes = (uint32_t)((size_t)n * sizeof(T)) & ~15u;
        if (tid == 0) {
            mbar_init(&s_bar, 1);
            fence_mbar_init();
            if (bytes) {
                mbar_arrive_expect_tx(&s_bar, bytes);
                for (uint32_t off = 0; off < bytes; off += 32768u)
                    tma_load_1d((unsigned char*)xs + off, (const unsigned char*)(row + lo) + off, min(32768u, bytes - off),
                                &s_bar);
            } else {
                mbar_arrive(&s_bar);
            }
        }
        __syncthreads();
        for (int i = (int)(bytes / sizeof(T)) + tid; i < n; i += NT) xs[i] = row[lo + i];  // ragged tail
        if (!mbar_wait_bounded(&s_bar, 0u)) timed_out = true;
        __syncthreads();
        if (tid == 0) mbar_inval(&s_bar);
    } else {
        for (int i = tid; i < n; i += NT) xs[i] = row[lo + i];
    }
    __syncthreads();
    if (timed_out && tid == 0) atomicExch(p.err, kErrTimeout);
    VDXS_T1(20, t_c1);
    VDXS_T0(t_c2);
    // 2. Penalised ids are excluded here (they re-enter in stage 2 with their values).
    const int npen = p.pen_cnt ? p.pen_cnt[b] : 0;
    const int32_t* pid = p.pen_ids ? p.pen_ids + (int64_t)b * p.pen_stride : nullptr;
    if (npen > 0) {
        for (int j = tid; j < npen; j += NT) {
            const int64_t id = pid[j];
            if (id >= lo && id < lo + n) xs[id - lo] = nan_bits<T>();
        }
        __syncthreads();
    }
    // 3. Bound: every thread maximum (CL * NT distinct elements of the row) goes to the
    // leader, which takes the K-th largest of them to a 16-bit key prefix: a lower bound
    // on the row's K-th key.
    if (r == 0 && tid == 0) {
        sh[19] = 0u;  // bound
        sh[41] = 0u;  // candidates reserved
        sh[42] = 0u;  // overflow
    }
    // Each thread's maximum over its 16-byte groups of the chunk (any partition of the
    // chunk gives maxima of distinct elements), then the ragged tail.
    constexpr int GV = (int)(16 / sizeof(T));
    float m0 = __uint_as_float(0x7FC00000u), m1 = m0;
    {
        const int ng4 = n / GV;
        for (int g = tid; g < ng4; g += NT) {
            float v[GV];
            unpack(*reinterpret_cast<const uint4*>(xs + (size_t)g * GV), v, T());
#pragma unroll
            for (int e = 0; e < GV; e += 2) {
                m0 = fmaxf(m0, v[e]);
                m1 = fmaxf(m1, v[e + 1]);
            }
        }
        for (int i = ng4 * GV + tid; i < n; i += NT) m0 = fmaxf(m0, to_f(xs[i]));
    }
    const float mx = fmaxf(m0, m1);
    cl.map_shared_rank(maxk, 0)[r * NT + tid] = mx == mx ? f2key(mx) : 0u;
    cl.sync();  // also publishes the leader's zeroed scalars
    if (r == 0 && K <= CL * NT) {
        // Two 256-bin passes over the top 16 key bits.
        uint32_t b1 = 0u, need = (uint32_t)K;
        for (int pass = 0; pass < 2; ++pass) {
            const int shift = pass == 0 ? 24 : 16;
            for (int j = tid; j < 256; j += NT) hist[j] = 0u;
            __syncthreads();
            for (int j = tid; j < CL * NT; j += NT) {
                const uint32_t k = maxk[j];
                if (k != 0u && (pass == 0 || (k >> 24) == b1)) atomicAdd(&hist[(k >> shift) & 255u], 1u);
            }
            __syncthreads();
            if (tid < 32) warp_suffix_find256(hist, need, sh + 16);
            __syncthreads();
            const uint32_t g = sh[16];
            __syncthreads();
            if (g == 0xFFFFFFFFu) break;  // fewer than K maxima: no bound
            if (pass == 0) {
                b1 = g;
                need -= sh[17];
            } else if (tid == 0) {
                sh[19] = (b1 << 24) | (g << 16);
            }
        }
    }
    cl.sync();
    VDXS_T1(21, t_c2);
    VDXS_T0(t_c3);
    const uint32_t t0 = *cl.map_shared_rank(&sh[19], 0);
    // 4. Elements at or above the bound go to the leader, packed by warp reservations.
    uint32_t* lkey = cl.map_shared_rank(ckey, 0);
    uint32_t* lidx = cl.map_shared_rank(cidx, 0);
    uint32_t* lcnt = cl.map_shared_rank(&sh[41], 0);
    uint32_t* lovf = cl.map_shared_rank(&sh[42], 0);
    const uint32_t gbase = (uint32_t)(p.vocab_offset + lo);
    const uint32_t total_cap = (uint32_t)(CL * cap);
    // Each warp gathers its candidates locally (its 1 KB of the maxima area, free now)
    // and reserves the leader's slots once per batch of up to kWarpBatch.
    constexpr int kWarpBatch = (kClusterMaxWords * 4) / (NWARPS * 8);  // 128 (key, index) pairs
    uint32_t* wk = maxk + (size_t)(tid >> 5) * (2 * kWarpBatch);
    uint32_t* wi = wk + kWarpBatch;
    int wn = 0;
    auto flush = [&]() {
        uint32_t base = 0u;
        if (lane == 0) base = atomicAdd(lcnt, (uint32_t)wn);
        base = __shfl_sync(FULL, base, 0);
        if (base + (uint32_t)wn > total_cap) {
            if (lane == 0) atomicOr(lovf, 1u);
        } else {
            for (int j = lane; j < wn; j += 32) {
                lkey[base + j] = wk[j];
                lidx[base + j] = wi[j];
            }
        }
        wn = 0;
        __syncwarp();
    };
    __syncthreads();  // every thread is done with the maxima area
    const float thr = key_threshold(t0);
    auto append = [&](bool sel, float v, int ii) {
        const unsigned mm = __ballot_sync(FULL, sel);
        if (mm == 0u) return;
        if (wn + __popc(mm) > kWarpBatch) flush();
        if (sel) {
            const int s2 = wn + __popc(mm & lanemask_lt());
            wk[s2] = f2key(v);
            wi[s2] = gbase + (uint32_t)ii;
        }
        wn += __popc(mm);
        __syncwarp();
    };
    // 16-byte groups: one lane-maximum test per group, per-element appends only when
    // some lane of the warp has a candidate.
    constexpr int VN = (int)(16 / sizeof(T));
    const int ngrp = n / VN;
    for (int g0 = (tid >> 5) * 32; g0 < ngrp; g0 += NT) {
        const int g = g0 + lane;
        float x[VN];
        if (g < ngrp) {
            unpack(*reinterpret_cast<const uint4*>(xs + (size_t)g * VN), x, T());
        } else {
#pragma unroll
            for (int e = 0; e < VN; ++e) x[e] = __uint_as_float(0x7FC00000u);
        }
        float gm = x[0];
#pragma unroll
        for (int e = 1; e < VN; ++e) gm = fmaxf(gm, x[e]);
        if (!__any_sync(FULL, gm >= thr)) continue;
#pragma unroll
        for (int e = 0; e < VN; ++e) append(x[e] >= thr, x[e], g * VN + e);
    }
    for (int i0 = ngrp * VN + (tid >> 5) * 32; i0 < n; i0 += NT) {  // the last < VN elements
        const int ii = i0 + lane;
        const float v = ii < n ? to_f(xs[ii]) : __uint_as_float(0x7FC00000u);
        append(v >= thr, v, ii);
    }
    if (wn > 0) flush();
    cl.sync();
    const bool overflow = *lovf != 0u;
    if (overflow) {
        // Many keys at the bound (e.g. equal logits): every CTA sends its exact top-K
        // with tie evidence to its own slot instead.
        uint32_t km = 0u;
        for (int j = tid; j < n; j += NT) km = max(km, ChunkKeySrc<T>{xs, n}.key(j));
        km = block_max_u32(km, sh + 32);
        const SelectOut so = block_select(ChunkKeySrc<T>{xs, n}, n, K, km, bits_for((uint32_t)max(n - 1, 1)), hist, sh);
        const int sent = block_emit(ChunkKeySrc<T>{xs, n}, n, so, lkey + r * cap, lidx + r * cap, cap, &sh[8],
                                    OffsetIdx{gbase});
        if (tid == 0) {
            cl.map_shared_rank(sh + 48, 0)[r] = (uint32_t)sent;
            cl.map_shared_rank(cuts, 0)[r] = so.tie_cut ? so.kth_key : 0u;
        }
        cl.sync();
    }
    VDXS_T1(22, t_c3);
    if (r != 0) return;
    VDXS_T0(t_c4);
    // 5. Leader: stage 2 on the gathered candidates and penalised entries.
    int nc;
    if (overflow) {
        for (int j = tid; j < CL * cap; j += NT)
            if ((uint32_t)(j % cap) >= sh[48 + j / cap]) ckey[j] = 0u;  // unused slots: no element
        nc = CL * cap;
    } else {
        nc = (int)sh[41];
        for (int j = tid; j < CL; j += NT) cuts[j] = 0u;
    }
    for (int j = tid; j < npen; j += NT) {
        ckey[nc + j] = f2key(p.pen_vals[(int64_t)b * p.pen_stride + j]);
        cidx[nc + j] = (uint32_t)(pid[j] + p.vocab_offset);
    }
    __syncthreads();
    const int n2 = nc + npen;
    uint32_t gm = 0u;
    for (int j = tid; j < n2; j += NT) gm = max(gm, ckey[j]);
    gm = block_max_u32(gm, sh + 32);
    finish_select<T>(p, b, ckey, cidx, n2, gm, CL, [&](int i) -> uint32_t { return cuts[i]; }, region, hist,
                     sh);
    VDXS_T1(23, t_c4);
}

// Per-row finish (one CTA per row), launched as a programmatic dependent of the stream
// kernel. MINB = 4 caps it at 64 registers, so that four finish CTAs fit an SM and a
// batch of 512 rows finishes in one wave on 148 SMs (c4: 139 -> 133 us per step); it
// spills in the faithful emulation, so batches that fit three CTAs per SM keep the
// uncapped build (MINB = 1).
template <typename T, int MINB>
__global__ void __launch_bounds__(NT, MINB) finish_kernel(KParams p) {
    extern __shared__ __align__(16) unsigned char smem_raw[];
    uint32_t* hist = (uint32_t*)smem_raw;
    uint32_t* sh = hist + kHistWords;
    unsigned char* region = smem_raw + kHeadBytes;
    // Launched as a programmatic dependent of stage 1: wait until that grid has completed
    // and its writes are visible (a no-op for an ordinary launch).
    asm volatile("griddepcontrol.wait;" ::: "memory");
    VDXS_T0(t_fin);
    const int b = blockIdx.x;
    finish_row<T>(p, b, region, hist, sh);
    // The row's stage-1 state is ready for the next call: bound, list count, histogram,
    // penalised-id bitmap words.
    if (threadIdx.x == 0) {
        p.row_tau[(size_t)b * kTauStride] = 0u;
        p.row_cnt[b] = 0u;
    }
    if (p.pen_bits) {
        const int npen = p.pen_cnt[b];
        const int32_t* pid = p.pen_ids + (int64_t)b * p.pen_stride;
        for (int j = threadIdx.x; j < npen; j += NT) p.pen_bits[(size_t)b * p.pen_words + (pid[j] >> 5)] = 0u;
    }
    uint4* rh4 = reinterpret_cast<uint4*>(p.rhist + (size_t)b * kRowHistWords);
    for (int i = threadIdx.x; i < kRowHistWords / 4; i += NT) rh4[i] = make_uint4(0u, 0u, 0u, 0u);
    VDXS_T1(5, t_fin);
}

// ---------------------------------------------------------------------------------
// Vocab-sharded merge and draw: candidates [ranks][B][K+1] from the all-gather.
// ---------------------------------------------------------------------------------
__global__ void __launch_bounds__(NT) merge_draw_kernel(KParams p, const uint2* recv, int ranks) {
    extern __shared__ __align__(16) unsigned char smem_raw[];
    uint32_t* hist = (uint32_t*)smem_raw;
    uint32_t* sh = hist + kHistWords;
    unsigned char* region = smem_raw + kHeadBytes;
    const int tid = threadIdx.x, b = blockIdx.x, K = p.K;
    uint32_t* sk = (uint32_t*)region;
    uint32_t* si = sk + K;
    uint32_t* ckey = si + K;
    const int n2 = ranks * K;
    uint32_t* cidx = ckey + n2;
    uint32_t lm = 0u, mi = 0u;
    for (int i = tid; i < n2; i += NT) {
        const int r = i / K, s = i - r * K;
        const uint2 e = recv[((int64_t)r * p.B + b) * (K + 1) + s];
        ckey[i] = e.x;
        cidx[i] = e.y;
        lm = max(lm, e.x);
        if (e.x) mi = max(mi, e.y);
    }
    const uint32_t gmax = block_max_u32(lm, sh + 32);
    const uint32_t imax = block_max_u32(mi, sh + 32);
    SelectOut s2 = block_select(SmemPairSrc{ckey, cidx}, n2, K, gmax, bits_for(imax), hist, sh);
    if (tid == 0) sh[8] = 0u;
    __syncthreads();
    const int rounds = (n2 + NT - 1) / NT;
    for (int j = 0; j < rounds; ++j) {
        const int i = j * NT + tid;
        uint32_t k = 0u, t = 0u;
        bool s = false;
        if (i < n2) {
            k = ckey[i];
            t = cidx[i];
            s = selected(k, t, s2);
        }
        const unsigned m = __ballot_sync(FULL, s);
        if (m) {
            uint32_t base = 0u;
            if ((tid & 31) == 0) base = atomicAdd(&sh[8], (uint32_t)__popc(m));
            base = __shfl_sync(FULL, base, 0);
            if (s) {
                const uint32_t slot = base + __popc(m & lanemask_lt());
                if (slot < (uint32_t)K) {
                    sk[slot] = k;
                    si[slot] = t;
                }
            }
        }
    }
    __syncthreads();
    const int nsel = (int)min(sh[8], (uint32_t)K);
    if (p.path == kGreedy) {
        if (tid == 0) {
            p.tokens[b] = (int32_t)si[0];
            if (p.flags) p.flags[b] = VDXS_FLAG_GREEDY;
        }
        return;
    }
    uint32_t kb = 0xFFFFFFFFu;
    for (int s = tid; s < nsel; s += NT) kb = min(kb, sk[s]);
    kb = block_min_u32(kb, sh + 32);
    uint32_t rt = 0u;
    for (int r = tid; r < ranks; r += NT) {
        const uint2 info = recv[((int64_t)r * p.B + b) * (K + 1) + K];
        if (info.y && info.x == kb) rt = 1u;
    }
    rt = block_max_u32(rt, sh + 32);
    const uint32_t btie = (s2.tie_cut || rt) ? VDXS_FLAG_BOUNDARY_TIE : 0u;
    unsigned char* work = (unsigned char*)(ckey);
    work = (unsigned char*)(((uintptr_t)work + 15) & ~(uintptr_t)15);
    uint32_t f2;
    stage2_canonical(p, b, sk, si, nsel, gmax, kb, btie, work, sh + 32, &f2);
}

// ---------------------------------------------------------------------------------
// Full-softmax path (Sampler.pas:461-527).
// ---------------------------------------------------------------------------------
struct PenLookup {
    const uint32_t* bitmap;
    const int32_t* ids;
    const float* vals;
    int n;
    __device__ __forceinline__ float apply(int i, int64_t gi, float x) const {
        if (n > 0 && ((bitmap[i >> 5] >> (i & 31)) & 1u)) {
            const int j = lower_bound_i32(ids, n, gi);
            return vals[j];
        }
        return x;
    }
};

__device__ void build_chunk_bitmap(uint32_t* bitmap, int chunk, const int32_t* pid, int npen,
                                   int64_t start, int n) {
    for (int i = threadIdx.x; i < (chunk >> 5); i += NT) bitmap[i] = 0u;
    __syncthreads();
    const int j0 = lower_bound_i32(pid, npen, start);
    for (int j = j0 + threadIdx.x; j < npen && pid[j] < start + n; j += NT) {
        const int e = pid[j] - (int)start;
        atomicOr(&bitmap[e >> 5], 1u << (e & 31));
    }
    __syncthreads();
}

template <typename T>
__global__ void __launch_bounds__(NT) full_max_kernel(KParams p) {
    extern __shared__ __align__(16) unsigned char smem_raw[];
    uint32_t* sh = (uint32_t*)smem_raw;
    uint32_t* bitmap = sh + kShWords;
    const int c = blockIdx.x, b = blockIdx.y, tid = threadIdx.x;
    const int64_t start = (int64_t)c * p.chunk;
    const int n = (int)min((int64_t)p.chunk, (int64_t)p.V - start);
    const T* row = (const T*)p.logits + (int64_t)b * p.stride;
    const int npen = p.pen_cnt ? p.pen_cnt[b] : 0;
    PenLookup pl{bitmap, p.pen_ids ? p.pen_ids + (int64_t)b * p.pen_stride : nullptr,
                 p.pen_vals ? p.pen_vals + (int64_t)b * p.pen_stride : nullptr, npen};
    if (npen > 0) build_chunk_bitmap(bitmap, p.chunk, pl.ids, npen, start, n);
    uint32_t lm = 0u;
    for (int i = tid; i < n; i += NT) {
        const float x = pl.apply(i, start + i, ld_elem(row, start + i));
        lm = max(lm, f2key(__fmul_rn(x, p.inv_temp)));
    }
    lm = block_max_u32(lm, sh);
    if (tid == 0) p.fmax[(int64_t)b * p.nchunks + c] = lm;
}

template <typename T>
__global__ void __launch_bounds__(NT) full_sum_kernel(KParams p) {
    extern __shared__ __align__(16) unsigned char smem_raw[];
    uint32_t* sh = (uint32_t*)smem_raw;
    uint32_t* bitmap = sh + kShWords;
    __shared__ double s_dsh[NWARPS];
    __shared__ double s_d[8];
    __shared__ int s_i[8];
    const int c = blockIdx.x, b = blockIdx.y, tid = threadIdx.x;
    const int64_t start = (int64_t)c * p.chunk;
    const int n = (int)min((int64_t)p.chunk, (int64_t)p.V - start);
    const T* row = (const T*)p.logits + (int64_t)b * p.stride;
    const int npen = p.pen_cnt ? p.pen_cnt[b] : 0;
    PenLookup pl{bitmap, p.pen_ids ? p.pen_ids + (int64_t)b * p.pen_stride : nullptr,
                 p.pen_vals ? p.pen_vals + (int64_t)b * p.pen_stride : nullptr, npen};
    if (npen > 0) build_chunk_bitmap(bitmap, p.chunk, pl.ids, npen, start, n);
    uint32_t gm = 0u;
    for (int i = tid; i < p.nchunks; i += NT) gm = max(gm, p.fmax[(int64_t)b * p.nchunks + i]);
    gm = block_max_u32(gm, sh);
    const float M = key2f(gm);
    const double Md = (double)M;
    const float best = (float)exp(Md - Md);  // the maximum element's probability
    const bool use_min = p.min_p > 0.0f;
    const float thr = __fmul_rn(best, p.min_p);
    double s = 0.0;
    uint32_t nz = 0u, emin = 0xFFFFFFFFu, pmax = 0u;
    for (int i = tid; i < n; i += NT) {
        const float x = pl.apply(i, start + i, ld_elem(row, start + i));
        float e = (float)exp((double)__fmul_rn(x, p.inv_temp) - Md);
        if (use_min && e < thr) e = 0.0f;
        s += (double)e;
        if (e > 0.0f) {
            ++nz;
            int ex = ilogbf(e);
            ex = ex < -126 ? -126 : ex;
            emin = min(emin, (uint32_t)(ex + 1024));
            pmax = max(pmax, f2key(e));
        }
    }
    double tot;
    block_excl_scan_d(s, s_dsh, &tot);
    nz = block_sum_u32(nz, sh);
    emin = block_min_u32(emin, sh);
    pmax = block_max_u32(pmax, sh);
    if (tid == 0) {
        p.fsum[(int64_t)b * p.nchunks + c] = tot;
        p.fstat[(int64_t)b * p.nchunks + c] = make_uint2(nz, emin);
        p.fmax[(int64_t)p.B * p.nchunks + (int64_t)b * p.nchunks + c] = pmax;
    }
    __threadfence();
    __syncthreads();
    if (tid == 0) {
        const uint32_t prev = atomicAdd(&p.row_counter[b], 1u);
        sh[9] = prev == (uint32_t)(p.nchunks - 1) ? 1u : 0u;
    }
    __syncthreads();
    if (sh[9] == 0u) return;
    __threadfence();
    // Last CTA of the row: locate the chunk holding the draw, then the element.
    if (tid == 0) {
        double S = 0.0;
        uint32_t nzt = 0u, em = 0xFFFFFFFFu, pm = 0u;
        for (int i = 0; i < p.nchunks; ++i) {
            S += __ldcg(p.fsum + (int64_t)b * p.nchunks + i);
            const uint2 st = __ldcg(p.fstat + (int64_t)b * p.nchunks + i);
            nzt += st.x;
            em = min(em, st.y);
            pm = max(pm, __ldcg(p.fmax + (int64_t)p.B * p.nchunks + (int64_t)b * p.nchunks + i));
        }
        const float u = p.uniform ? p.uniform[b] : 0.0f;
        const double t = (double)u * S;
        double acc = 0.0;
        int cs = -1;
        for (int i = 0; i < p.nchunks; ++i) {
            const double cs_sum = __ldcg(p.fsum + (int64_t)b * p.nchunks + i);
            if (acc + cs_sum > t) {
                cs = i;
                break;
            }
            acc += cs_sum;
        }
        bool exact = true;
        if (nzt > 0u) {
            const int E = ilogb((double)nzt * (double)key2f(pm));
            exact = (int)em - 1024 >= E - 29;
        }
        s_i[0] = cs;
        s_i[1] = exact ? 1 : 0;
        s_d[0] = t;
        s_d[1] = S;
        s_d[2] = acc;
    }
    __syncthreads();
    const int cs = s_i[0];
    const double t = s_d[0], S = s_d[1];
    uint32_t f = VDXS_FLAG_FULL | (s_i[1] ? 0u : VDXS_FLAG_INEXACT_SUM);
    int tok = p.V - 1;
    double before = 0.0, after = 0.0;
    bool fallback = cs < 0;
    if (!fallback) {
        // Re-read the chunk with contiguous per-thread runs and scan in index order.
        const int64_t cstart = (int64_t)cs * p.chunk;
        const int cn = (int)min((int64_t)p.chunk, (int64_t)p.V - cstart);
        if (npen > 0) build_chunk_bitmap(bitmap, p.chunk, pl.ids, npen, cstart, cn);
        const int R = (p.chunk + NT - 1) / NT;
        const int r0 = tid * R, r1 = min(r0 + R, cn);
        double ls = 0.0;
        for (int i = r0; i < r1; ++i) {
            const float x = pl.apply(i, cstart + i, ld_elem(row, cstart + i));
            float e = (float)exp((double)__fmul_rn(x, p.inv_temp) - Md);
            if (use_min && e < thr) e = 0.0f;
            ls += (double)e;
        }
        double tot2;
        double off = block_excl_scan_d(ls, s_dsh, &tot2) + s_d[2];
        uint32_t jj = 0xFFFFFFFFu;
        double cum = off, bef = 0.0;
        for (int i = r0; i < r1; ++i) {
            const float x = pl.apply(i, cstart + i, ld_elem(row, cstart + i));
            float e = (float)exp((double)__fmul_rn(x, p.inv_temp) - Md);
            if (use_min && e < thr) e = 0.0f;
            bef = cum;
            cum += (double)e;
            if (cum > t) {
                jj = (uint32_t)i;
                break;
            }
        }
        const uint32_t jmin = block_min_u32(jj, sh);
        if (jj == jmin && jj != 0xFFFFFFFFu) {
            s_d[4] = bef;
            s_d[5] = cum;
            s_i[2] = (int)jj;
        }
        __syncthreads();
        if (jmin == 0xFFFFFFFFu) {
            fallback = true;
        } else {
            tok = (int)(cstart + s_i[2]);
            before = s_d[4];
            after = s_d[5];
        }
    }
    if (tid == 0) {
        if (fallback) f |= VDXS_FLAG_FALLBACK;
        const double eps = 1e-6 * S;
        if (fallback || (t - before) <= eps || (after - t) <= eps) f |= VDXS_FLAG_NEAR_BOUNDARY;
        p.tokens[b] = tok;
        if (p.flags) p.flags[b] = f;
        p.row_counter[b] = 0u;
    }
    for (int s = tid; s < p.out_k; s += NT) {
        if (p.out_idx) p.out_idx[(int64_t)b * p.out_k + s] = -1;
        if (p.out_prob) p.out_prob[(int64_t)b * p.out_k + s] = 0.0f;
    }
}

// ---------------------------------------------------------------------------------
// Host side: plans, workspace, launches.
// ---------------------------------------------------------------------------------
static size_t align16(size_t x) { return (x + 15) & ~(size_t)15; }

static int pow2_at_least(int n, int lo) {
    int p = lo;
    while (p < n) p <<= 1;
    return p;
}

static size_t stage2_bytes(int K, int n2) {
    const int P2 = pow2_at_least(K, 32);
    const size_t math = (size_t)24 * P2 + 8 + 16;
    const size_t cands = (size_t)8 * n2;
    return (size_t)8 * K + std::max(math, cands) + 16;
}

static size_t faithful_bytes(int K) {  // sval/sidx, the (value, index) candidate ring, stage-2 tail
    const int P2 = pow2_at_least(K, 32);
    return (size_t)8 * K + (size_t)8 * kFaithfulSlots * kFaithfulSub + 16 + (size_t)16 * P2 + 16;
}

cudaError_t plan_topk(const SampleArgs& a, int smem_optin, LaunchPlan* plan, std::string* err) {
    const int K = a.K;
    const int64_t V = a.V;
    const int pen_stride = a.penalty_on ? (int)std::min<int64_t>(a.hist_stride, kMaxHistory) : 0;
    const size_t esz = a.dtype == VDXS_DTYPE_BF16 ? 2 : 4;
    const bool faithful = a.tie_mode == VDXS_TIES_FAITHFUL && a.path == kTopK && !a.local_emit;
    if (a.B <= kClusterMaxRows && K <= kMaxTopK) {
        // Small batches: one cluster per row when a row's 1/CL fits in shared memory (its
        // stage 2 holds up to kMaxTopK survivors, like the finish kernel's).
        for (const int CL : {kClusterCTAs}) {
            const int64_t L = ((V + CL - 1) / CL + 15) / 16 * 16;
            const int cap = std::max(K, 512);
            size_t xs_area = align16((size_t)L * esz);
            xs_area = std::max(xs_area, align16((size_t)8 * K + 16));  // finish_select's sk / si
            if (faithful) xs_area = std::max(xs_area, align16(faithful_bytes(K)));
            const size_t ncap = (size_t)CL * cap + pen_stride;
            const int P2 = pow2_at_least(K, 32);
            const size_t cand_area = std::max((size_t)8 * ncap, (size_t)24 * P2 + 64);  // also stage 2's work
            const size_t need = kHeadBytes + xs_area + (size_t)4 * kClusterMaxWords + cand_area + 4 * CL + 16;
            if ((int64_t)need + 1024 > smem_optin || L > INT32_MAX) continue;  // 1 KB: the static shared memory
            plan->cluster = true;
            plan->cluster_ctas = CL;
            plan->stream = false;
            plan->chunk = (int)L;
            plan->span = (int)xs_area;
            plan->cand_cap = cap;
            plan->nchunks = 1;
            plan->nspans = 1;
            plan->items = 0;
            plan->smem = align16(need);
            return cudaSuccess;
        }
    }
    if (K <= kMaxTopK) {
        // Stream path: stage 1 on one 16-warp CTA per SM (warps claim row units) + one
        // finish CTA per row.
        int dev = 0, sms = 148;
        cudaGetDevice(&dev);
        cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev);
        const int SE = esz == 4 ? s1_slot_elems<float>() : s1_slot_elems<uint16_t>();
        const int ng = (int)((V + SE - 1) / SE);
        // Row segments of 16 slots (64 KB fp32); the kernel claims them in runs that shrink
        // near the end of the work.
        const int U = std::min(ng, 16);
        const long long units = (long long)a.B * ((ng + U - 1) / U);
        if (units * U >= (1LL << 31)) {
            if (err) *err = "batch x vocab too large for the stream path";
            return cudaErrorInvalidValue;
        }
        // A row's list holds every element at or above the row's final bound, plus
        // candidates taken while the bounds were still rising (about K times the log of
        // the row's units for random orders, more for rows with many ties at the bound).
        // A longer list is incomplete and its row takes the finish kernel's exact fallback.
        // Above top_k 64 a slot's local bound (above 256: none) passes much of a slot, and
        // every warp's first slots of a row go to the list before the row's histogram holds
        // K counts (the raise lands two slots after it starts): with few slots per warp
        // (small batches) those slots are much of the list, which has room for six slots
        // per warp working on the row.
        int dev0 = 0, sms0 = 148;
        cudaGetDevice(&dev0);
        cudaDeviceGetAttribute(&sms0, cudaDevAttrMultiProcessorCount, dev0);
        const int64_t wpr = ((int64_t)sms0 * kS1Warps + a.B - 1) / a.B;
        const int64_t first_wave = K > 64 ? 6 * wpr * SE : 0;
        const int cc = (int)std::min<int64_t>(std::max<int64_t>({32LL * K, 4096, first_wave}), (int64_t)ng * SE);
        const int gather = std::max(K <= 128 ? 4096 : 8192, K + pen_stride);
        size_t s2 = std::max(stage2_bytes(K, gather + pen_stride), faithful ? faithful_bytes(K) : (size_t)0);
        s2 += kHeadBytes;
        const size_t s1 = s1_smem_bytes();
        if ((int64_t)s1 > smem_optin || (int64_t)align16(s2) > smem_optin) {
            if (err) *err = "shared-memory plan exceeds the device limit";
            return cudaErrorInvalidValue;
        }
        plan->chunk = 0;
        plan->nchunks = 1;
        plan->nspans = 1;
        plan->span = 1;
        plan->elems = 0;
        plan->stream = true;
        plan->cand_cap = cc;
        plan->gather_cap = gather;
        // One CTA per SM unless the work is below about four slots per warp.
        const long long slots = (long long)a.B * ng;
        plan->grid = (int)std::max<long long>(1, std::min<long long>((long long)sms, slots / (4LL * kS1Warps)));
        plan->slots = ng;
        plan->unit_slots = U;
        plan->items = a.B;
        plan->smem = s1;
        plan->smem2 = align16(s2);
        return cudaSuccess;
    }
    {
        // top_k above the stream path's maximum: one CTA per row of a persistent grid, each
        // with 24 bytes of global workspace per slot (at most 1 GiB in all). When 32 K <= V
        // the stream kernel runs first and the large kernel selects from its row lists.
        int dev = 0, sms = 148;
        cudaGetDevice(&dev);
        cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev);
        const size_t sm = lk_smem_bytes(K);
        if ((int64_t)sm + 1024 > smem_optin) {
            if (err) *err = "shared-memory plan exceeds the device limit";
            return cudaErrorInvalidValue;
        }
        const int64_t per_cta = 8 * lk_cta_words(K);
        const int64_t by_mem = std::max<int64_t>(1, (1LL << 30) / per_cta);
        plan->large = true;
        plan->stream = false;
        plan->large_grid = (int)std::min<int64_t>({(int64_t)a.B, 2LL * sms, by_mem});
        plan->large_smem = align16(sm);
        plan->chunk = 0;
        plan->nchunks = 1;
        plan->nspans = 1;
        plan->span = 1;
        plan->items = 0;
        plan->cand_cap = 0;
        if (32LL * K <= V) {
            const int SE = esz == 4 ? s1_slot_elems<float>() : s1_slot_elems<uint16_t>();
            const int ng = (int)((V + SE - 1) / SE);
            const int U = std::min(ng, 16);
            const long long units = (long long)a.B * ((ng + U - 1) / U);
            const size_t s1 = s1_smem_bytes();
            if (units * U < (1LL << 31) && (int64_t)s1 <= smem_optin) {
                plan->stream = true;
                const int64_t wpr = ((int64_t)sms * kS1Warps + a.B - 1) / a.B;
                plan->cand_cap = (int)std::min<int64_t>(std::max<int64_t>(32LL * K, 4 * wpr * SE), (int64_t)ng * SE);
                plan->items = a.B;
                const long long slots = (long long)a.B * ng;
                plan->grid = (int)std::max<long long>(1, std::min<long long>((long long)sms, slots / (4LL * kS1Warps)));
                plan->slots = ng;
                plan->unit_slots = U;
                plan->smem = s1;
            }
        }
        return cudaSuccess;
    }
}

cudaError_t plan_full(const SampleArgs& a, LaunchPlan* plan, std::string*) {
    int chunk = 16384;
    const int64_t V = a.V;
    while (chunk > 2048 && (int64_t)a.B * ((V + chunk - 1) / chunk) < 148 * 4) chunk >>= 1;
    if (V <= chunk) chunk = (int)((V + 31) / 32 * 32);
    plan->chunk = chunk;
    plan->nchunks = (int)((V + chunk - 1) / chunk);
    plan->smem = align16((size_t)4 * kShWords + (size_t)4 * (chunk / 32 + 1));
    return cudaSuccess;
}

template <typename P>
static cudaError_t grow(P** ptr, size_t* cap, size_t want, bool zero, cudaStream_t stream) {
    if (*cap >= want && *ptr) return cudaSuccess;
    if (*ptr) {
        cudaError_t e = cudaStreamSynchronize(stream);
        if (e != cudaSuccess) return e;
        cudaFree(*ptr);
        *ptr = nullptr;
        *cap = 0;
    }
    size_t bytes = std::max<size_t>(want, 1) * sizeof(P);
    cudaError_t e = cudaMalloc((void**)ptr, bytes);
    if (e != cudaSuccess) {
        *ptr = nullptr;
        return e;
    }
    if (zero) {
        e = cudaMemsetAsync(*ptr, 0, bytes, stream);
        if (e != cudaSuccess) return e;
    }
    *cap = std::max<size_t>(want, 1);
    return cudaSuccess;
}

cudaError_t ensure_workspace(Workspace& ws, const SampleArgs& a, const LaunchPlan& plan, int ranks,
                             cudaStream_t stream, std::string* err) {
    cudaError_t e;
    const size_t B = (size_t)a.B;
    const size_t nch = (size_t)plan.nchunks;
    if (!ws.err) {
        if ((e = cudaMalloc((void**)&ws.err, sizeof(int32_t))) != cudaSuccess) return e;
        if ((e = cudaMemsetAsync(ws.err, 0, sizeof(int32_t), stream)) != cudaSuccess) return e;
    }
    // Completion counters and row thresholds start at zero and every launch leaves them at zero.
    if ((e = grow(&ws.row_counter, &ws.row_counter_cap, B, true, stream)) != cudaSuccess) return e;
    if ((e = grow(&ws.row_tau, &ws.row_tau_cap, B * kTauStride, true, stream)) != cudaSuccess) return e;
    if (a.path != kFull) {
        if ((e = grow(&ws.cand, &ws.cand_cap, (size_t)plan.items * (size_t)plan.cand_cap, false, stream)) !=
            cudaSuccess)
            return e;
        if (plan.stream) {
            // Per-row histograms and list counts, and the claim counter: zero once here, then
            // left at zero by every call (finish kernel, last stage-1 warp).
            if ((e = grow(&ws.rhist, &ws.rhist_cap, B * (size_t)kRowHistWords, true, stream)) != cudaSuccess) return e;
            if ((e = grow(&ws.row_cnt, &ws.row_cnt_cap, B, true, stream)) != cudaSuccess) return e;
            if (!ws.unit_next) {
                size_t c2 = 0;
                if ((e = grow(&ws.unit_next, &c2, 2, true, stream)) != cudaSuccess) return e;
            }
        }
    } else {
        // fmax: [B*nch] max keys + [B*nch] probability max keys; fsum: [B*nch] sums + [B*nch] stats.
        size_t cap_a = ws.full_cap, cap_b = ws.full_cap;
        if ((e = grow(&ws.fmax, &cap_a, 2 * B * nch, false, stream)) != cudaSuccess) return e;
        if ((e = grow(&ws.fsum, &cap_b, 2 * B * nch, false, stream)) != cudaSuccess) return e;
        ws.full_cap = std::min(cap_a, cap_b);
    }
    if (a.penalty_on) {
        const size_t ps = (size_t)std::min<int64_t>(a.hist_stride, kMaxHistory);
        size_t cap_a = ws.pen_cap, cap_b = ws.pen_cap;
        if ((e = grow(&ws.pen_ids, &cap_a, B * ps, false, stream)) != cudaSuccess) return e;
        if ((e = grow(&ws.pen_vals, &cap_b, B * ps, false, stream)) != cudaSuccess) return e;
        ws.pen_cap = std::min(cap_a, cap_b);
        if ((e = grow(&ws.pen_cnt, &ws.pen_rows_cap, B, false, stream)) != cudaSuccess) return e;
        if (plan.stream || plan.large) {
            // Zero once; the finish kernel (the large top-k kernel) clears the words it set.
            const size_t words = B * (size_t)((a.V + 31) / 32);
            if ((e = grow(&ws.pen_bits, &ws.pen_bits_cap, words, true, stream)) != cudaSuccess) return e;
        }
    }
    if (plan.large &&
        (e = grow(&ws.lk_buf, &ws.lk_cap, (size_t)plan.large_grid * (size_t)lk_cta_words(a.K), false, stream)) !=
            cudaSuccess)
        return e;
    if (a.local_emit) {
        if ((e = grow(&ws.shard_send, &ws.shard_send_cap, B * (size_t)(a.K + 1), false, stream)) != cudaSuccess)
            return e;
        if ((e = grow(&ws.shard_recv, &ws.shard_recv_cap, (size_t)ranks * B * (size_t)(a.K + 1), false,
                      stream)) != cudaSuccess)
            return e;
    }
    (void)err;
    return cudaSuccess;
}

// Scratch of vdxs_sample_noalloc: one fixed array per device, held until the process
// exits. Host code must not use the symbol as a pointer; noalloc_scratch() resolves its
// device address with cudaGetSymbolAddress once per device, with that device current.
static __device__ __align__(256) unsigned char g_noalloc_scratch[kNoAllocScratchBytes];

cudaError_t noalloc_scratch(void** ptr, int* smem_optin) {
    static std::mutex mu;
    static void* addr[64] = {nullptr};
    static int optin[64] = {0};
    int dev = 0;
    cudaError_t e = cudaGetDevice(&dev);
    if (e != cudaSuccess) return e;
    if (dev < 0 || dev >= 64) return cudaErrorInvalidDevice;
    std::lock_guard<std::mutex> lock(mu);
    if (!addr[dev]) {
        void* p = nullptr;
        e = cudaGetSymbolAddress(&p, g_noalloc_scratch);
        if (e != cudaSuccess) return e;
        int o = 0;
        e = cudaDeviceGetAttribute(&o, cudaDevAttrMaxSharedMemoryPerBlockOptin, dev);
        if (e != cudaSuccess) return e;
        addr[dev] = p;
        optin[dev] = o;
    }
    *ptr = addr[dev];
    *smem_optin = optin[dev];
    return cudaSuccess;
}

size_t carve_workspace(Workspace& ws, unsigned char* base, size_t cap, const SampleArgs& a, const LaunchPlan& plan) {
    const size_t B = (size_t)a.B, nch = (size_t)plan.nchunks;
    size_t off = 0;
    Workspace w;
    auto take = [&](size_t bytes) -> unsigned char* {
        unsigned char* p = base + off;
        off += (bytes + 255) & ~(size_t)255;
        return p;
    };
    w.err = (int32_t*)take(sizeof(int32_t));
    w.row_counter = (uint32_t*)take(B * sizeof(uint32_t));
    w.row_counter_cap = B;
    w.row_tau = (uint32_t*)take(B * kTauStride * sizeof(uint32_t));
    w.row_tau_cap = B * kTauStride;
    if (a.path != kFull) {
        w.cand = (uint2*)take((size_t)plan.items * (size_t)plan.cand_cap * sizeof(uint2));
        w.cand_cap = (size_t)plan.items * (size_t)plan.cand_cap;
        if (plan.stream) {
            w.rhist = (uint32_t*)take(B * (size_t)kRowHistWords * sizeof(uint32_t));
            w.rhist_cap = B * (size_t)kRowHistWords;
            w.row_cnt = (uint32_t*)take(B * sizeof(uint32_t));
            w.row_cnt_cap = B;
            w.unit_next = (unsigned long long*)take(2 * sizeof(unsigned long long));
        }
    } else {
        w.fmax = (uint32_t*)take(2 * B * nch * sizeof(uint32_t));
        w.fsum = (double*)take(2 * B * nch * sizeof(double));
        w.full_cap = 2 * B * nch;
    }
    if (a.penalty_on) {
        const size_t ps = (size_t)std::min<int64_t>(a.hist_stride, kMaxHistory);
        w.pen_ids = (int32_t*)take(B * ps * sizeof(int32_t));
        w.pen_vals = (float*)take(B * ps * sizeof(float));
        w.pen_cnt = (int32_t*)take(B * sizeof(int32_t));
        if (plan.stream || plan.large) {
            const size_t words = B * (size_t)((a.V + 31) / 32);
            w.pen_bits = (uint32_t*)take(words * sizeof(uint32_t));
            w.pen_bits_cap = words;
        }
        w.pen_cap = B * ps;
        w.pen_rows_cap = B;
    }
    if (plan.large) {
        w.lk_cap = (size_t)plan.large_grid * (size_t)lk_cta_words(a.K);
        w.lk_buf = (uint64_t*)take(w.lk_cap * sizeof(uint64_t));
    }
    if (off <= cap) ws = w;
    return off;
}

cudaError_t reset_device_state(Workspace& ws, cudaStream_t stream) {
    cudaError_t e = cudaSuccess;
    if (ws.err && (e = cudaMemsetAsync(ws.err, 0, sizeof(int32_t), stream)) != cudaSuccess) return e;
    if (ws.row_counter && (e = cudaMemsetAsync(ws.row_counter, 0, sizeof(uint32_t) * ws.row_counter_cap, stream)) !=
                              cudaSuccess)
        return e;
    if (ws.row_tau && (e = cudaMemsetAsync(ws.row_tau, 0, sizeof(uint32_t) * ws.row_tau_cap, stream)) != cudaSuccess)
        return e;
    if (ws.rhist && (e = cudaMemsetAsync(ws.rhist, 0, sizeof(uint32_t) * ws.rhist_cap, stream)) != cudaSuccess)
        return e;
    if (ws.row_cnt && (e = cudaMemsetAsync(ws.row_cnt, 0, sizeof(uint32_t) * ws.row_cnt_cap, stream)) != cudaSuccess)
        return e;
    if (ws.unit_next && (e = cudaMemsetAsync(ws.unit_next, 0, 2 * sizeof(unsigned long long), stream)) != cudaSuccess)
        return e;
    if (ws.pen_bits && (e = cudaMemsetAsync(ws.pen_bits, 0, sizeof(uint32_t) * ws.pen_bits_cap, stream)) != cudaSuccess)
        return e;
    return cudaSuccess;
}

void free_workspace(Workspace& ws) {
    cudaFree(ws.cand);
    cudaFree(ws.rhist);
    cudaFree(ws.row_cnt);
    cudaFree(ws.unit_next);
    cudaFree(ws.pen_bits);
    cudaFree(ws.row_counter);
    cudaFree(ws.row_tau);
    cudaFree(ws.pen_ids);
    cudaFree(ws.pen_vals);
    cudaFree(ws.pen_cnt);
    cudaFree(ws.fmax);
    cudaFree(ws.fsum);
    cudaFree(ws.shard_send);
    cudaFree(ws.shard_recv);
    cudaFree(ws.lk_buf);
    cudaFree(ws.unembed_logits);
    cudaFree(ws.err);
    cudaFree(ws.d_logits);
    cudaFree(ws.d_hist);
    cudaFree(ws.d_hcnt);
    cudaFree(ws.d_unif);
    cudaFree(ws.d_tok);
    if (ws.h_tok_pinned) cudaFreeHost(ws.h_tok_pinned);
    ws = Workspace();
}

static KParams make_params(const SampleArgs& a, const LaunchPlan& plan, Workspace& ws) {
    KParams p{};
    p.logits = a.logits;
    p.stride = a.stride;
    p.V = a.V;
    p.B = a.B;
    p.chunk = plan.chunk;
    p.nchunks = plan.nchunks;
    p.span = plan.span;
    p.K = a.K;
    p.path = a.path;
    if (a.penalty_on) {
        p.pen_ids = ws.pen_ids;
        p.pen_vals = ws.pen_vals;
        p.pen_cnt = ws.pen_cnt;
        p.pen_stride = (int)std::min<int64_t>(a.hist_stride, kMaxHistory);
        if (plan.stream || plan.large) {
            p.pen_bits = ws.pen_bits;
            p.pen_words = (a.V + 31) / 32;
        }
    }
    p.cand = ws.cand;
    p.cand_cap = plan.cand_cap;
    p.gather_cap = plan.gather_cap;
    p.flat_ng = plan.slots;
    p.unit_slots = plan.unit_slots;
    p.rhist = ws.rhist;
    p.row_cnt = ws.row_cnt;
    p.unit_next = ws.unit_next;
    p.row_counter = ws.row_counter;
    p.row_tau = ws.row_tau;
    p.err = ws.err;
    p.fmax = ws.fmax;
    p.fsum = ws.fsum;
    p.fstat = (uint2*)(ws.fsum ? ws.fsum + (size_t)a.B * plan.nchunks : nullptr);
    p.uniform = a.uniform;
    p.tokens = a.tokens;
    p.flags = a.flags;
    p.out_idx = a.out_idx;
    p.out_prob = a.out_prob;
    p.out_k = a.out_k;
    p.inv_temp = a.inv_temp;
    p.min_p = a.min_p;
    p.top_p = a.top_p;
    p.tie_mode = a.tie_mode;
    p.vocab_offset = a.vocab_offset;
    p.local_emit = a.local_emit ? 1 : 0;
    p.emit_out = ws.shard_send;
    p.lk_buf = ws.lk_buf;
    p.lk_list = plan.large && plan.stream ? 1 : 0;
    return p;
}

// Records the optional profiling event and counts launches (diagnostics only).
static inline cudaError_t mark(const SampleArgs& a, cudaEvent_t ev) {
    return ev ? cudaEventRecord(ev, a.stream) : cudaSuccess;
}
static inline void count(const SampleArgs& a, int n = 1) {
    if (a.launches) *a.launches += n;
}

template <typename T>
static cudaError_t launch_typed(const SampleArgs& a, const LaunchPlan& plan, Workspace& ws, std::string* err) {
    cudaError_t e;
    KParams p = make_params(a, plan, ws);
    if (a.penalty_on) {
        const int ps = p.pen_stride;
        const int P2 = pow2_at_least(std::max(ps, 1), 1);
        const size_t sm = (size_t)4 * P2;
        e = cudaFuncSetAttribute(penalty_prep_kernel<T>, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)sm);
        if (e != cudaSuccess) return e;
        penalty_prep_kernel<T><<<a.B, NT, sm, a.stream>>>((const T*)a.logits, a.stride, a.V, a.vocab_offset, a.hist,
                                                           a.hist_stride, a.hist_count, a.penalty, ws.pen_ids,
                                                           ws.pen_vals, ws.pen_cnt, ps, p.pen_bits, p.pen_words);
        if ((e = cudaGetLastError()) != cudaSuccess) return e;
        count(a);
    }
    (void)err;
    const dim3 grid(plan.nchunks, a.B);
    if (a.path == kFull) {
        e = cudaFuncSetAttribute(full_max_kernel<T>, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)plan.smem);
        if (e != cudaSuccess) return e;
        e = cudaFuncSetAttribute(full_sum_kernel<T>, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)plan.smem);
        if (e != cudaSuccess) return e;
        if ((e = mark(a, a.ev_begin)) != cudaSuccess) return e;
        full_max_kernel<T><<<grid, NT, plan.smem, a.stream>>>(p);
        if ((e = cudaGetLastError()) != cudaSuccess) return e;
        full_sum_kernel<T><<<grid, NT, plan.smem, a.stream>>>(p);
        if ((e = cudaGetLastError()) != cudaSuccess) return e;
        count(a, 2);
        return mark(a, a.ev_end);
    }
    const size_t esz = sizeof(T);
    const bool vec = ((uintptr_t)a.logits % 16 == 0) && (((size_t)a.stride * esz) % 16 == 0);
    if (plan.cluster) {
        const int CL = plan.cluster_ctas;
        void (*kc)(KParams) = vec ? row_cluster_kernel<T, true, kClusterCTAs> : row_cluster_kernel<T, false, kClusterCTAs>;
        if ((e = cudaFuncSetAttribute(kc, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)plan.smem)) != cudaSuccess)
            return e;
        cudaLaunchConfig_t lc = {};
        lc.gridDim = dim3(CL, a.B);
        lc.blockDim = dim3(NT);
        lc.dynamicSmemBytes = plan.smem;
        lc.stream = a.stream;
        cudaLaunchAttribute at[1];
        at[0].id = cudaLaunchAttributeClusterDimension;
        at[0].val.clusterDim.x = CL;
        at[0].val.clusterDim.y = 1;
        at[0].val.clusterDim.z = 1;
        lc.attrs = at;
        lc.numAttrs = 1;
        if ((e = mark(a, a.ev_begin)) != cudaSuccess) return e;
        if ((e = cudaLaunchKernelEx(&lc, kc, p)) != cudaSuccess) return e;
        count(a);
        return mark(a, a.ev_end);
    }
    if (plan.stream) {
        void (*k1)(KParams) = vec ? topk_stream_kernel<T, true> : topk_stream_kernel<T, false>;
        if ((e = cudaFuncSetAttribute(k1, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)plan.smem)) != cudaSuccess)
            return e;
        int sms = 148, dev = 0;
        cudaGetDevice(&dev);
        cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev);
        void (*kf)(KParams) = a.B > 3 * sms ? finish_kernel<T, 4> : finish_kernel<T, 1>;
        if ((e = cudaFuncSetAttribute(kf, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                      (int)plan.smem2)) != cudaSuccess)
            return e;
        if ((e = mark(a, a.ev_begin)) != cudaSuccess) return e;
        if (a.penalty_on) {
            // Programmatic dependent of the penalty prep: its launch overlaps the prep's
            // tail; the kernel waits for the prep grid before it reads the lists.
            cudaLaunchConfig_t lc1 = {};
            lc1.gridDim = dim3(plan.grid);
            lc1.blockDim = dim3(kS1Threads);
            lc1.dynamicSmemBytes = plan.smem;
            lc1.stream = a.stream;
            cudaLaunchAttribute at1[1];
            at1[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
            at1[0].val.programmaticStreamSerializationAllowed = 1;
            lc1.attrs = at1;
            lc1.numAttrs = 1;
            if ((e = cudaLaunchKernelEx(&lc1, k1, p)) != cudaSuccess) return e;
        } else {
            k1<<<plan.grid, kS1Threads, plan.smem, a.stream>>>(p);
            if ((e = cudaGetLastError()) != cudaSuccess) return e;
        }
        if ((e = mark(a, a.ev_end)) != cudaSuccess) return e;
        if (plan.large) {
            // top_k above the stream path's maximum: the large top-k kernel selects from the
            // row lists stage 1 just wrote.
            if ((e = cudaFuncSetAttribute(topk_large_kernel<T>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                          (int)plan.large_smem)) != cudaSuccess)
                return e;
            topk_large_kernel<T><<<plan.large_grid, NT, plan.large_smem, a.stream>>>(p);
            if ((e = cudaGetLastError()) != cudaSuccess) return e;
        } else {
            // Programmatic dependent launch: finish CTAs are scheduled as stage-1 CTAs
            // retire, hiding the launch gap; they wait for the whole grid in the kernel.
            // (A recorded event between the two launches makes it an ordinary launch.)
            cudaLaunchConfig_t lc = {};
            lc.gridDim = dim3(a.B);
            lc.blockDim = dim3(NT);
            lc.dynamicSmemBytes = plan.smem2;
            lc.stream = a.stream;
            cudaLaunchAttribute at[1];
            at[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
            at[0].val.programmaticStreamSerializationAllowed = 1;
            lc.attrs = at;
            lc.numAttrs = 1;
            if ((e = cudaLaunchKernelEx(&lc, kf, p)) != cudaSuccess) return e;
        }
        count(a, 2);
        return cudaSuccess;
    }
    if (plan.large && !plan.stream) {
        if ((e = cudaFuncSetAttribute(topk_large_kernel<T>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                      (int)plan.large_smem)) != cudaSuccess)
            return e;
        if ((e = mark(a, a.ev_begin)) != cudaSuccess) return e;
        topk_large_kernel<T><<<plan.large_grid, NT, plan.large_smem, a.stream>>>(p);
        if ((e = cudaGetLastError()) != cudaSuccess) return e;
        count(a);
        return mark(a, a.ev_end);
    }
    if (err) *err = "no top-k plan for this call";
    return cudaErrorInvalidValue;
}

cudaError_t launch_sample(const SampleArgs& a, const LaunchPlan& plan, Workspace& ws, std::string* err) {
    if (a.dtype == VDXS_DTYPE_BF16) return launch_typed<uint16_t>(a, plan, ws, err);
    return launch_typed<float>(a, plan, ws, err);
}

cudaError_t launch_merge_draw(const SampleArgs& a, int ranks, Workspace& ws, std::string* err) {
    LaunchPlan plan{};
    plan.nchunks = 1;
    KParams p = make_params(a, plan, ws);
    p.local_emit = 0;
    p.tie_mode = VDXS_TIES_CANONICAL;
    const int n2 = ranks * a.K;
    const size_t sm = align16(kHeadBytes + stage2_bytes(a.K, n2));
    cudaError_t e = cudaFuncSetAttribute(merge_draw_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)sm);
    if (e != cudaSuccess) {
        if (err) *err = "merge kernel shared memory request rejected";
        return e;
    }
    merge_draw_kernel<<<a.B, NT, sm, a.stream>>>(p, ws.shard_recv, ranks);
    if ((e = cudaGetLastError()) != cudaSuccess) return e;
    count(a);
    return cudaSuccess;
}

// ---------------------------------------------------------------------------------
// Device-resident decode state: per-row xoshiro256** (Sampler.pas:208-222, 243-248) and
// history ring (Sampler.pas:530-539), one thread per row.
// ---------------------------------------------------------------------------------
__device__ __forceinline__ uint64_t rotl64d(uint64_t x, int k) { return (x << k) | (x >> (64 - k)); }

__global__ void device_uniforms_kernel(uint64_t* prng, int batch, float* out) {
    const int r = blockIdx.x * blockDim.x + threadIdx.x;
    if (r >= batch) return;
    uint64_t* s = prng + (size_t)4 * r;
    uint64_t s0 = s[0], s1 = s[1], s2 = s[2], s3 = s[3];
    const uint64_t result = rotl64d(s1 * 5ull, 7) * 9ull;
    const uint64_t t = s1 << 17;
    s2 ^= s0;
    s3 ^= s1;
    s1 ^= s2;
    s0 ^= s3;
    s2 ^= t;
    s3 = rotl64d(s3, 45);
    s[0] = s0;
    s[1] = s1;
    s[2] = s2;
    s[3] = s3;
    // (result >> 40) / 2^24: a 24-bit integer scaled by a power of two, exact in float.
    out[r] = (float)(result >> 40) * (1.0f / 16777216.0f);
}

__global__ void history_push_kernel(int32_t* hist, int32_t* pos, int32_t* count, int window, const int32_t* tokens,
                                    int batch, const int32_t* stop_ids, int n_stop, int32_t* stopped) {
    const int r = blockIdx.x * blockDim.x + threadIdx.x;
    if (r >= batch) return;
    const int32_t tok = tokens[r];
    if (window > 0) {
        int p = pos[r] % window;
        if (p < 0) p += window;  // a position outside the ring never indexes outside it
        hist[(int64_t)r * window + p] = tok;
        pos[r] = (p + 1) % window;
        if (count[r] < window) count[r] = max(count[r], 0) + 1;
    }
    if (n_stop > 0) {
        bool hit = false;
        for (int j = 0; j < n_stop; ++j) hit |= stop_ids[j] == tok;
        if (hit) stopped[r] = 1;
    }
}

cudaError_t launch_device_uniforms(uint64_t* prng, int batch, float* out, cudaStream_t stream) {
    device_uniforms_kernel<<<(batch + NT - 1) / NT, NT, 0, stream>>>(prng, batch, out);
    return cudaGetLastError();
}

cudaError_t launch_history_push(int32_t* hist, int32_t* pos, int32_t* count, int window, const int32_t* tokens,
                                int batch, const int32_t* stop_ids, int n_stop, int32_t* stopped,
                                cudaStream_t stream) {
    history_push_kernel<<<(batch + NT - 1) / NT, NT, 0, stream>>>(hist, pos, count, window, tokens, batch, stop_ids,
                                                                    n_stop, stopped);
    return cudaGetLastError();
}

}  // namespace vdxs

#ifdef VDXS_TIMING
extern "C" __attribute__((visibility("default"))) int vdxs_debug_network_selftest(int R, const uint64_t* d_in,
                                                                                     uint64_t* d_sorted,
                                                                                     uint64_t* d_merged, int n) {
    const int blocks = (n + 7) / 8;
    if (R == 1) vdxs::warp_network_selftest<1><<<blocks, 256>>>(d_in, d_sorted, d_merged, n);
    else if (R == 2) vdxs::warp_network_selftest<2><<<blocks, 256>>>(d_in, d_sorted, d_merged, n);
    else if (R == 4) vdxs::warp_network_selftest<4><<<blocks, 256>>>(d_in, d_sorted, d_merged, n);
    else return -1;
    return cudaDeviceSynchronize() == cudaSuccess ? 0 : -2;
}
extern "C" __attribute__((visibility("default"))) int vdxs_debug_phase_times(unsigned long long* cycles,
                                                                                unsigned long long* counts,
                                                                                int reset) {
    cudaMemcpyFromSymbol(cycles, vdxs::g_phase_cycles, sizeof(unsigned long long) * 64);
    cudaMemcpyFromSymbol(counts, vdxs::g_phase_count, sizeof(unsigned long long) * 64);
    if (reset) {
        unsigned long long z[64] = {0};
        cudaMemcpyToSymbol(vdxs::g_phase_cycles, z, sizeof(z));
        cudaMemcpyToSymbol(vdxs::g_phase_count, z, sizeof(z));
    }
    return 0;
}
#endif

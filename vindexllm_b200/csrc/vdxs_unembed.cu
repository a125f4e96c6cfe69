// vdxs_unembed.cu - the unembedding matvec in front of the sampler:
// TVdxModel.UnembedToLogits (src/VindexLLM.Model.pas:1258-1271) multiplies the normed
// hidden vector by the tied Q4_0 embedding with shaders/matvec_q4_0.comp (:45-88), and
// the logits go to TVdxSampler.Process.
//
// The shader's arithmetic is reproduced exactly: for each output row, 64 partial sums,
// partial t accumulating elements t, t + 64, ... in order (acc += (qval * scale) * x,
// each operation rounded to fp32, no fused multiply-add), then the pairwise tree over
// strides 32, 16, ..., 1. One warp computes a row: lane l holds partials l (the even
// Q4_0 blocks) and l + 32 (the odd blocks), because element 32j + l of block j belongs
// to partial l when j is even and to partial l + 32 when j is odd.
//
// Layout: the reference's 18-byte blocks are repacked once (q4_0_repack) into
//   nib[row][word][lane]  (uint32): nibble m of word w is element `lane` of block 8w+m;
//   scales[row][block]    (fp16, padded to a multiple of 8 blocks per row),
// so a warp reads a row's nibbles as coalesced 128-byte lines and its scales as 16-byte
// broadcasts: the same 1440 bytes per row of 2560 elements as the Q4_0 blocks.
#include "vdxs_internal.h"

#include <cuda_fp16.h>
#include <cuda_runtime.h>

#include <algorithm>

namespace vdxs {

int q4_0_words_per_lane(int in_dim);

namespace {

constexpr unsigned FULLMASK = 0xFFFFFFFFu;
constexpr int kUThreads = 256;
constexpr int kUWarps = kUThreads / 32;

__global__ void q4_0_repack_kernel(const uint8_t* __restrict__ src, int nb, int nw, int out_dim,
                                   uint32_t* __restrict__ nib, uint16_t* __restrict__ scales) {
    const int64_t total = (int64_t)out_dim * nw * 32;
    for (int64_t t = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; t < total; t += (int64_t)gridDim.x * blockDim.x) {
        const int lane = (int)(t & 31);
        const int64_t rw = t >> 5;
        const int w = (int)(rw % nw);
        const int64_t row = rw / nw;
        const uint8_t* rb = src + row * (int64_t)nb * 18;
        uint32_t word = 0u;
#pragma unroll
        for (int m = 0; m < 8; ++m) {
            const int j = 8 * w + m;
            uint32_t q = 8u;  // padding blocks: never read
            if (j < nb) {
                const uint32_t raw = rb[(int64_t)j * 18 + 2 + (lane & 15)];
                q = lane < 16 ? (raw & 15u) : (raw >> 4);
            }
            word |= q << (4 * m);
        }
        nib[t] = word;
        if (lane < 8) {
            const int j = 8 * w + lane;
            scales[row * (int64_t)nw * 8 + j] =
                j < nb ? (uint16_t)(rb[(int64_t)j * 18] | (rb[(int64_t)j * 18 + 1] << 8)) : (uint16_t)0;
        }
    }
}

// Packed fp32 pairs (sm_100 f32x2): both halves rounded to nearest, exactly as two
// scalar operations.
__device__ __forceinline__ uint64_t pk2(float lo, float hi) {
    uint64_t d;
    asm("mov.b64 %0, {%1, %2};" : "=l"(d) : "f"(lo), "f"(hi));
    return d;
}
__device__ __forceinline__ uint64_t mul2(uint64_t a, uint64_t b) {
    uint64_t d;
    asm("mul.rn.f32x2 %0, %1, %2;" : "=l"(d) : "l"(a), "l"(b));
    return d;
}
__device__ __forceinline__ uint64_t add2(uint64_t a, uint64_t b) {
    uint64_t d;
    asm("add.rn.f32x2 %0, %1, %2;" : "=l"(d) : "l"(a), "l"(b));
    return d;
}
__device__ __forceinline__ float lo2(uint64_t v) { return __uint_as_float((uint32_t)v); }
__device__ __forceinline__ float hi2(uint64_t v) { return __uint_as_float((uint32_t)(v >> 32)); }

// Each lane carries its two partial sums (even blocks, odd blocks) as one packed pair, so
// a block pair costs two scalar multiplies and one packed add per input vector (a packed
// multiply feeding a packed add was contracted into a fused multiply-add by the
// compiler, which changes the rounding the shader's sums have). The input
// vectors sit in shared memory as pairs (x[64k + l], x[64k + 32 + l]); a missing odd
// block (an odd block count) has x = 0, weight 0 and adds +0.0, which leaves a
// round-to-nearest sum started at +0 unchanged.
template <int B, int NW>
__global__ void __launch_bounds__(kUThreads) q4_0_matvec_kernel(const uint32_t* __restrict__ nib,
                                                                const uint16_t* __restrict__ scales,
                                                                const float* __restrict__ x, int in_dim,
                                                                int out_dim, float* __restrict__ out) {
    extern __shared__ float2 xs2[];  // [B][npairs][32]
    const int nb = in_dim >> 5, nw = (nb + 7) >> 3, npairs = (nb + 1) >> 1;
    for (int i = threadIdx.x; i < B * npairs * 32; i += kUThreads) {
        const int l = i & 31, k = (i >> 5) % npairs, b = (i >> 5) / npairs;
        const int e0 = 64 * k + l, e1 = e0 + 32;
        xs2[i] = make_float2(x[(int64_t)b * in_dim + e0], e1 < in_dim ? x[(int64_t)b * in_dim + e1] : 0.0f);
    }
    __syncthreads();
    const int lane = threadIdx.x & 31;
    const int warps = gridDim.x * kUWarps;
    const uint64_t kMagic8 = pk2(-8388616.0f, -8388616.0f);  // -(2^23 + 8)
    // A row's words are read kWChunk at a time, all loads of a chunk issued before any is
    // used; lane c of the warp also loads the chunk's c-th group of eight scales, which
    // reaches the other lanes by shuffles.
    constexpr int kWChunk = 16;
    for (int row = blockIdx.x * kUWarps + (threadIdx.x >> 5); row < out_dim; row += warps) {
        const uint32_t* nr = nib + (int64_t)row * nw * 32 + lane;
        const uint4* sr = reinterpret_cast<const uint4*>(scales + (int64_t)row * nw * 8);
        uint64_t acc[B];
#pragma unroll
        for (int b = 0; b < B; ++b) acc[b] = 0ull;  // (+0, +0)
        // One block pair (2k, 2k + 1): nibbles m, m + 1 of `word`, scales in `sp`.
        auto pair = [&](uint32_t word, int m, uint32_t sp, int k) {
            // nibble - 8 for both blocks: 2^23 + nibble as a float, minus 2^23 + 8.
            const float fa = __uint_as_float(0x4B000000u | ((word >> (4 * m)) & 15u));
            const float fb = __uint_as_float(0x4B000000u | ((word >> (4 * m + 4)) & 15u));
            const uint64_t q = add2(pk2(fa, fb), kMagic8);
            const float s0 = __half2float(__ushort_as_half((unsigned short)(sp & 0xFFFFu)));
            const float s1 = __half2float(__ushort_as_half((unsigned short)(sp >> 16)));
            const uint64_t qs = mul2(q, pk2(s0, s1));  // exact
            const float2* xk = xs2 + k * 32 + lane;
#pragma unroll
            for (int b = 0; b < B; ++b) {
                const float2 xv = xk[b * npairs * 32];
                // Scalar products (.rn: never contracted into a fused multiply-add with the
                // sum), then one packed add.
                const float t0 = __fmul_rn(lo2(qs), xv.x);
                const float t1 = __fmul_rn(hi2(qs), xv.y);
                acc[b] = add2(acc[b], pk2(t0, t1));
            }
        };
        if constexpr (NW > 0) {
            // Words per lane known at compile time: all loads first, then fully unrolled
            // pairs; only the last word can hold padding blocks.
            uint32_t words[NW];
#pragma unroll
            for (int c = 0; c < NW; ++c) words[c] = __ldg(nr + c * 32);
            const uint4 s4 = lane < NW ? __ldg(sr + lane) : make_uint4(0u, 0u, 0u, 0u);
#pragma unroll
            for (int c = 0; c < NW; ++c) {
                const uint32_t sw[4] = {__shfl_sync(FULLMASK, s4.x, c), __shfl_sync(FULLMASK, s4.y, c),
                                        __shfl_sync(FULLMASK, s4.z, c), __shfl_sync(FULLMASK, s4.w, c)};
#pragma unroll
                for (int m = 0; m < 8; m += 2) {
                    const int k = 4 * c + (m >> 1);
                    if (c < NW - 1 || k < npairs) pair(words[c], m, sw[m >> 1], k);
                }
            }
        } else {
            for (int w0 = 0; w0 < nw; w0 += kWChunk) {
                const int nc = min(kWChunk, nw - w0);
                uint32_t words[kWChunk];
#pragma unroll
                for (int c = 0; c < kWChunk; ++c) words[c] = c < nc ? __ldg(nr + (w0 + c) * 32) : 0u;
                const uint4 s4 = lane < nc ? __ldg(sr + w0 + lane) : make_uint4(0u, 0u, 0u, 0u);
#pragma unroll
                for (int c = 0; c < kWChunk; ++c) {
                    if (c >= nc) break;
                    const int w = w0 + c;
                    const uint32_t sw[4] = {__shfl_sync(FULLMASK, s4.x, c), __shfl_sync(FULLMASK, s4.y, c),
                                            __shfl_sync(FULLMASK, s4.z, c), __shfl_sync(FULLMASK, s4.w, c)};
#pragma unroll
                    for (int m = 0; m < 8; m += 2) {
                        const int k = 4 * w + (m >> 1);
                        if (k < npairs) pair(words[c], m, sw[m >> 1], k);
                    }
                }
            }
        }
#pragma unroll
        for (int b = 0; b < B; ++b) {
            // Stride 32: partial[l] + partial[l + 32]; then strides 16 .. 1.
            float p = __fadd_rn(lo2(acc[b]), hi2(acc[b]));
#pragma unroll
            for (int s = 16; s > 0; s >>= 1) p = __fadd_rn(p, __shfl_down_sync(FULLMASK, p, s));
            if (lane == 0) out[(int64_t)b * out_dim + row] = p;
        }
    }
}

template <int B, int NW>
cudaError_t launch_matvec_nw(const uint32_t* nib, const uint16_t* scales, const float* x, int in_dim, int out_dim,
                             float* out, cudaStream_t stream) {
    const size_t smem = (size_t)B * (((in_dim >> 5) + 1) / 2) * 32 * sizeof(float2);
    void (*kern)(const uint32_t*, const uint16_t*, const float*, int, int, float*) = q4_0_matvec_kernel<B, NW>;
    cudaError_t e = cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem);
    if (e != cudaSuccess) return e;
    int dev = 0, sms = 148, per_sm = 1;
    cudaGetDevice(&dev);
    cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev);
    e = cudaOccupancyMaxActiveBlocksPerMultiprocessor(&per_sm, kern, kUThreads, smem);
    if (e != cudaSuccess) return e;
    const int64_t want = ((int64_t)out_dim + kUWarps - 1) / kUWarps;
    const int grid = (int)std::max<int64_t>(1, std::min<int64_t>(want, (int64_t)sms * std::max(per_sm, 1)));
    kern<<<grid, kUThreads, smem, stream>>>(nib, scales, x, in_dim, out_dim, out);
    return cudaGetLastError();
}

// Words per lane specialised for the hidden sizes 1152, 2560 and 3840 (5, 10, 15).
template <int B>
cudaError_t launch_matvec(const uint32_t* nib, const uint16_t* scales, const float* x, int in_dim, int out_dim,
                          float* out, cudaStream_t stream) {
    switch (q4_0_words_per_lane(in_dim)) {
        case 5: return launch_matvec_nw<B, 5>(nib, scales, x, in_dim, out_dim, out, stream);
        case 10: return launch_matvec_nw<B, 10>(nib, scales, x, in_dim, out_dim, out, stream);
        case 15: return launch_matvec_nw<B, 15>(nib, scales, x, in_dim, out_dim, out, stream);
        default: return launch_matvec_nw<B, 0>(nib, scales, x, in_dim, out_dim, out, stream);
    }
}

}  // namespace

int q4_0_words_per_lane(int in_dim) { return ((in_dim >> 5) + 7) >> 3; }

int unembed_chunk_rows(int in_dim) {
    // The chunk's input vectors live in shared memory as float2 pairs of 64-element
    // groups (at most kUnembedSmemBytes).
    const size_t per_row = (size_t)(((in_dim >> 5) + 1) / 2) * 32 * 8;
    return std::min(kMaxUnembedBatch, (int)(kUnembedSmemBytes / std::max<size_t>(per_row, 1)));
}

size_t q4_0_packed_bytes(int in_dim, int out_dim) {
    const size_t nw = (size_t)q4_0_words_per_lane(in_dim);
    return (size_t)out_dim * nw * (32 * 4 + 8 * 2);
}

cudaError_t q4_0_repack(const uint8_t* src, int in_dim, int out_dim, uint32_t* nib, uint16_t* scales,
                        cudaStream_t stream) {
    const int nb = in_dim >> 5, nw = q4_0_words_per_lane(in_dim);
    const int64_t total = (int64_t)out_dim * nw * 32;
    const int grid = (int)std::min<int64_t>((total + 255) / 256, 148 * 16);
    q4_0_repack_kernel<<<grid, 256, 0, stream>>>(src, nb, nw, out_dim, nib, scales);
    return cudaGetLastError();
}

cudaError_t q4_0_matvec(const uint32_t* nib, const uint16_t* scales, int in_dim, int out_dim, const float* x,
                        int batch, float* out, cudaStream_t stream, int* launches) {
    // Batches above kMaxUnembedBatch are cut into chunks (the weights are read per chunk).
    const int per = unembed_chunk_rows(in_dim);
    if (per < 1) return cudaErrorInvalidValue;
    for (int b0 = 0; b0 < batch;) {
        // Chunks of 8, 4, 2 or 1 rows (at most `per`).
        const int left = std::min(per, batch - b0);
        const int nbch = left >= 8 ? 8 : left >= 4 ? 4 : left >= 2 ? 2 : 1;
        const float* xb = x + (int64_t)b0 * in_dim;
        float* ob = out + (int64_t)b0 * out_dim;
        cudaError_t e;
        switch (nbch) {
            case 1: e = launch_matvec<1>(nib, scales, xb, in_dim, out_dim, ob, stream); break;
            case 2: e = launch_matvec<2>(nib, scales, xb, in_dim, out_dim, ob, stream); break;
            case 4: e = launch_matvec<4>(nib, scales, xb, in_dim, out_dim, ob, stream); break;
            default: e = launch_matvec<8>(nib, scales, xb, in_dim, out_dim, ob, stream); break;
        }
        if (e != cudaSuccess) return e;
        if (launches) ++*launches;
        b0 += nbch;
    }
    return cudaSuccess;
}

}  // namespace vdxs

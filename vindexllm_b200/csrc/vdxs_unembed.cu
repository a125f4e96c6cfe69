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

template <int B>
__global__ void __launch_bounds__(kUThreads) q4_0_matvec_kernel(const uint32_t* __restrict__ nib,
                                                                const uint16_t* __restrict__ scales,
                                                                const float* __restrict__ x, int in_dim,
                                                                int out_dim, float* __restrict__ out) {
    extern __shared__ float xs[];  // [B][in_dim]
    const int nb = in_dim >> 5, nw = (nb + 7) >> 3;
    for (int i = threadIdx.x; i < B * in_dim; i += kUThreads) xs[i] = x[i];
    __syncthreads();
    const int lane = threadIdx.x & 31;
    const int warps = gridDim.x * kUWarps;
    for (int row = blockIdx.x * kUWarps + (threadIdx.x >> 5); row < out_dim; row += warps) {
        const uint32_t* nr = nib + (int64_t)row * nw * 32 + lane;
        const uint4* sr = reinterpret_cast<const uint4*>(scales + (int64_t)row * nw * 8);
        float acc_even[B], acc_odd[B];
#pragma unroll
        for (int b = 0; b < B; ++b) acc_even[b] = acc_odd[b] = 0.0f;
        for (int w = 0; w < nw; ++w) {
            const uint32_t word = __ldg(nr + w * 32);
            const uint4 s4 = __ldg(sr + w);
            const uint32_t sw[4] = {s4.x, s4.y, s4.z, s4.w};
#pragma unroll
            for (int m = 0; m < 8; ++m) {
                const int j = 8 * w + m;
                if (j < nb) {
                    const uint16_t hb = (uint16_t)(sw[m >> 1] >> (16 * (m & 1)));
                    const float scale = __half2float(__ushort_as_half(hb));
                    const float qval = (float)((int)((word >> (4 * m)) & 15u) - 8);
                    const float qs = __fmul_rn(qval, scale);  // exact
                    const float* xj = xs + 32 * j + lane;
#pragma unroll
                    for (int b = 0; b < B; ++b) {
                        const float t = __fmul_rn(qs, xj[b * in_dim]);
                        if (m & 1) acc_odd[b] = __fadd_rn(acc_odd[b], t);
                        else acc_even[b] = __fadd_rn(acc_even[b], t);
                    }
                }
            }
        }
#pragma unroll
        for (int b = 0; b < B; ++b) {
            // Stride 32: partial[l] + partial[l + 32]; then strides 16 .. 1.
            float p = __fadd_rn(acc_even[b], acc_odd[b]);
#pragma unroll
            for (int s = 16; s > 0; s >>= 1) p = __fadd_rn(p, __shfl_down_sync(FULLMASK, p, s));
            if (lane == 0) out[(int64_t)b * out_dim + row] = p;
        }
    }
}

template <int B>
cudaError_t launch_matvec(const uint32_t* nib, const uint16_t* scales, const float* x, int in_dim, int out_dim,
                          float* out, cudaStream_t stream) {
    const size_t smem = (size_t)B * in_dim * sizeof(float);
    cudaError_t e = cudaFuncSetAttribute(q4_0_matvec_kernel<B>, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem);
    if (e != cudaSuccess) return e;
    int dev = 0, sms = 148, per_sm = 1;
    cudaGetDevice(&dev);
    cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev);
    e = cudaOccupancyMaxActiveBlocksPerMultiprocessor(&per_sm, q4_0_matvec_kernel<B>, kUThreads, smem);
    if (e != cudaSuccess) return e;
    const int64_t want = ((int64_t)out_dim + kUWarps - 1) / kUWarps;
    const int grid = (int)std::max<int64_t>(1, std::min<int64_t>(want, (int64_t)sms * std::max(per_sm, 1)));
    q4_0_matvec_kernel<B><<<grid, kUThreads, smem, stream>>>(nib, scales, x, in_dim, out_dim, out);
    return cudaGetLastError();
}

}  // namespace

int q4_0_words_per_lane(int in_dim) { return ((in_dim >> 5) + 7) >> 3; }

int unembed_chunk_rows(int in_dim) {
    // The chunk's input vectors live in shared memory (at most kUnembedSmemBytes).
    return std::min(kMaxUnembedBatch, (int)(kUnembedSmemBytes / ((size_t)4 * std::max(in_dim, 1))));
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
    for (int b0 = 0; b0 < batch; b0 += per) {
        const int nbch = std::min(per, batch - b0);
        const float* xb = x + (int64_t)b0 * in_dim;
        float* ob = out + (int64_t)b0 * out_dim;
        cudaError_t e;
        switch (nbch) {
            case 1: e = launch_matvec<1>(nib, scales, xb, in_dim, out_dim, ob, stream); break;
            case 2: e = launch_matvec<2>(nib, scales, xb, in_dim, out_dim, ob, stream); break;
            case 3: e = launch_matvec<3>(nib, scales, xb, in_dim, out_dim, ob, stream); break;
            case 4: e = launch_matvec<4>(nib, scales, xb, in_dim, out_dim, ob, stream); break;
            case 5: e = launch_matvec<5>(nib, scales, xb, in_dim, out_dim, ob, stream); break;
            case 6: e = launch_matvec<6>(nib, scales, xb, in_dim, out_dim, ob, stream); break;
            case 7: e = launch_matvec<7>(nib, scales, xb, in_dim, out_dim, ob, stream); break;
            default: e = launch_matvec<8>(nib, scales, xb, in_dim, out_dim, ob, stream); break;
        }
        if (e != cudaSuccess) return e;
        if (launches) ++*launches;
    }
    return cudaSuccess;
}

}  // namespace vdxs

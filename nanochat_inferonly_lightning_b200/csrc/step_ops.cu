// The two small passes at the ends of a decode step, so that a graph-captured step is all on this
// library:
//  * the embedding gather fused with the RMSNorm that follows it (reference
//    kernels/ops.cu:9-20 then kernels/rmsnorm.cu:9-56, called at src/model.cpp:158-162);
//  * greedy sampling, the first maximum of each row of logits (src/engine.cpp:88-95), on the
//    device so the token never leaves it between steps.
#include <cstdint>

#include "../../include/nanochat_attn.h"
#include "nc_common.cuh"
#include "sm100_ptx.cuh"

namespace nc {

namespace {

constexpr int kEmbedThreads = 256;
constexpr int kArgmaxThreads = 1024;
constexpr int kStatusTokenRange = 0x800;  // a token id outside [0, vocab): row written as zeros

// out[r] = RMSNorm(table[tokens[r]]): one CTA per row, 16-byte loads, fp32 sum of squares,
// rsqrt(sum / dim + 1e-6), one bf16 rounding (the reference's rmsnorm on the gathered row).
__global__ void __launch_bounds__(kEmbedThreads)
    embed_rmsnorm_kernel(bf16* __restrict__ out, const bf16* __restrict__ table,
                         const int* __restrict__ tokens, int dim, int vocab, int* status) {
    // The GEMM that consumes `out` may start streaming its weights now (it waits for this grid
    // before reading `out`).
    griddep_launch_dependents();
    __shared__ float red[kEmbedThreads / 32];
    const int r = blockIdx.x;
    const int tok = tokens[r];
    bf16* dst = out + (size_t)r * dim;
    const int nvec = dim / 8;
    if (tok < 0 || tok >= vocab) {
        if (threadIdx.x == 0) atomicOr(status, kStatusTokenRange);
        for (int i = threadIdx.x; i < nvec; i += kEmbedThreads)
            reinterpret_cast<uint4*>(dst)[i] = make_uint4(0u, 0u, 0u, 0u);
        return;
    }
    const uint4* src = reinterpret_cast<const uint4*>(table + (size_t)tok * dim);
    // dim <= 8 * 4 * kEmbedThreads: at most four vectors per thread, held in registers.
    uint4 v[4];
    float ss = 0.f;
#pragma unroll
    for (int j = 0; j < 4; ++j) {
        const int i = threadIdx.x + j * kEmbedThreads;
        v[j] = i < nvec ? src[i] : make_uint4(0u, 0u, 0u, 0u);
        float f[8];
        bf16x8_to_f32(v[j], f);
#pragma unroll
        for (int e = 0; e < 8; ++e) ss = __fmaf_rn(f[e], f[e], ss);
    }
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) ss += __shfl_xor_sync(0xFFFFFFFFu, ss, o);
    if ((threadIdx.x & 31) == 0) red[threadIdx.x >> 5] = ss;
    __syncthreads();
    float tot = 0.f;
#pragma unroll
    for (int w = 0; w < kEmbedThreads / 32; ++w) tot += red[w];
    const float scale = rsqrtf(tot / (float)dim + kNormEps);
#pragma unroll
    for (int j = 0; j < 4; ++j) {
        const int i = threadIdx.x + j * kEmbedThreads;
        if (i < nvec) {
            float f[8];
            bf16x8_to_f32(v[j], f);
#pragma unroll
            for (int e = 0; e < 8; ++e) f[e] *= scale;
            reinterpret_cast<uint4*>(dst)[i] = f32_to_bf16x8(f);
        }
    }
}

// Keeps (value, index) of the larger value; on equal values the smaller index, so the result
// is the first maximum whatever the reduction order.
__device__ __forceinline__ void better(float& v, int& i, float v2, int i2) {
    if (v2 > v || (v2 == v && i2 < i)) {
        v = v2;
        i = i2;
    }
}

// out[r] = first index of the maximum of row r: one CTA per row; each thread scans 8-wide
// vectors in increasing index order with a strict '>' (so it keeps its first maximum), then a
// warp and a block reduction that prefer the smaller index on ties.
__global__ void __launch_bounds__(kArgmaxThreads)
    argmax_rows_kernel(int* __restrict__ out, const bf16* __restrict__ logits, int cols) {
    __shared__ float sv[kArgmaxThreads / 32];
    __shared__ int si[kArgmaxThreads / 32];
    const bf16* row = logits + (size_t)blockIdx.x * cols;
    float best = -INFINITY;
    int bi = 0x7FFFFFFF;
    for (int c = threadIdx.x * 8; c < cols; c += kArgmaxThreads * 8) {
        float f[8];
        bf16x8_to_f32(*reinterpret_cast<const uint4*>(row + c), f);
#pragma unroll
        for (int e = 0; e < 8; ++e)
            if (bi == 0x7FFFFFFF || f[e] > best) {  // the thread's first element, then strict '>'
                best = f[e];
                bi = c + e;
            }
    }
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) {
        const float v2 = __shfl_xor_sync(0xFFFFFFFFu, best, o);
        const int i2 = __shfl_xor_sync(0xFFFFFFFFu, bi, o);
        better(best, bi, v2, i2);
    }
    if ((threadIdx.x & 31) == 0) {
        sv[threadIdx.x >> 5] = best;
        si[threadIdx.x >> 5] = bi;
    }
    __syncthreads();
    if (threadIdx.x < 32) {
        best = sv[threadIdx.x];
        bi = si[threadIdx.x];
#pragma unroll
        for (int o = 16; o > 0; o >>= 1) {
            const float v2 = __shfl_xor_sync(0xFFFFFFFFu, best, o);
            const int i2 = __shfl_xor_sync(0xFFFFFFFFu, bi, o);
            better(best, bi, v2, i2);
        }
        if (threadIdx.x == 0) out[blockIdx.x] = bi;
    }
}

}  // namespace

}  // namespace nc

extern "C" {

int nc_embed_rmsnorm(void* out, const void* table, const int* tokens, int rows, int dim,
                     int vocab, cudaStream_t stream) {
    using namespace nc;
    if (rows < 0 || dim < 8 || (dim & 7) || dim > 8 * 4 * kEmbedThreads || vocab < 1)
        return NC_ERR_INVALID_ARG;
    if (rows == 0) return NC_OK;
    if (!out || !table || !tokens) return NC_ERR_INVALID_ARG;
    if ((reinterpret_cast<uintptr_t>(out) & 15) || (reinterpret_cast<uintptr_t>(table) & 15))
        return NC_ERR_MISALIGNED;
    int* status = nullptr;
    int st = internal_status_word(&status);
    if (st) return st;
    embed_rmsnorm_kernel<<<rows, kEmbedThreads, 0, stream>>>(
        static_cast<bf16*>(out), static_cast<const bf16*>(table), tokens, dim, vocab, status);
    cudaError_t e = cudaGetLastError();
    return e == cudaSuccess ? NC_OK : internal_cuda_fail(e);
}

int nc_argmax_rows(int* out, const void* logits, int rows, int cols, cudaStream_t stream) {
    using namespace nc;
    if (rows < 0 || cols < 8 || (cols & 7)) return NC_ERR_INVALID_ARG;
    if (rows == 0) return NC_OK;
    if (!out || !logits) return NC_ERR_INVALID_ARG;
    if (reinterpret_cast<uintptr_t>(logits) & 15) return NC_ERR_MISALIGNED;
    argmax_rows_kernel<<<rows, kArgmaxThreads, 0, stream>>>(out, static_cast<const bf16*>(logits),
                                                            cols);
    cudaError_t e = cudaGetLastError();
    return e == cudaSuccess ? NC_OK : internal_cuda_fail(e);
}

}  // extern "C"

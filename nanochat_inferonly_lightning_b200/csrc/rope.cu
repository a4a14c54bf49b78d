// RoPE, fused RoPE + parameter-free QK-RMSNorm, and the fused RoPE + QK-norm + KV-append
// pass that writes keys and values straight into the KV cache.
//
// Replaces reference kernels/rope.cu (init_rope_tables :14-30, rope_kernel/apply_rope :34-68,
// rope_rmsnorm_kernel/apply_rope_rmsnorm :74-158) and the two cudaMemcpyAsync cache appends
// in src/model.cpp:122-131.
//
// Mapping: one half-warp per (position, head) row, 16 lanes x 16-byte loads = one 256-byte
// head row, so a warp moves two full rows per instruction (fully coalesced).  The pair
// partner (dim i <-> i+64) sits eight lanes away and is fetched with one shuffle per word.
#include <cmath>
#include <mutex>
#include <vector>

#include "nc_common.cuh"

namespace nc {

namespace {

// cos/sin table (10.5 MB per device), filled by upload_rope_table().
__device__ float2 g_rope_cs[kRopeMaxSeq * kHalfDim];

constexpr int kRopeThreads = 256;   // 16 half-warps per block
constexpr int kRowsPerHalfWarp = 2;  // rows per half-warp: all loads issued before any math

template <int MODE>
__global__ void __launch_bounds__(kRopeThreads) rope_rows_kernel(RopeArgs a) {
    const int hw = (blockIdx.x * kRopeThreads + threadIdx.x) >> 4;
    const int sub = threadIdx.x & 15;
    const unsigned mask = (threadIdx.x & 16) ? 0xFFFF0000u : 0x0000FFFFu;
    const int nrows = a.seq_len * a.heads;
    const int row0 = hw * kRowsPerHalfWarp;
    if (row0 >= nrows) return;  // whole half-warps leave together
    bool has[kRowsPerHalfWarp];
    size_t off[kRowsPerHalfWarp];
    int pos[kRowsPerHalfWarp];
#pragma unroll
    for (int r = 0; r < kRowsPerHalfWarp; ++r) {
        const int row = row0 + r;
        has[r] = row < nrows;
        off[r] = (size_t)(has[r] ? row : row0) * kHeadDim + 8 * sub;
        pos[r] = a.start_pos + (has[r] ? row : row0) / a.heads;
    }
    if (MODE == kRopeNormAppend) {
        uint4 qr[kRowsPerHalfWarp], kr[kRowsPerHalfWarp], vr[kRowsPerHalfWarp];
#pragma unroll
        for (int r = 0; r < kRowsPerHalfWarp; ++r) {
            qr[r] = *reinterpret_cast<const uint4*>(a.q + off[r]);
            kr[r] = *reinterpret_cast<const uint4*>(a.k + off[r]);
            vr[r] = *reinterpret_cast<const uint4*>(a.v + off[r]);
        }
#pragma unroll
        for (int r = 0; r < kRowsPerHalfWarp; ++r) {
            float y[8];
            rope_norm_row(a.rope_cs, qr[r], sub, mask, pos[r], true, y);
            const uint4 qo = f32_to_bf16x8(y);
            rope_norm_row(a.rope_cs, kr[r], sub, mask, pos[r], true, y);
            const uint4 ko = f32_to_bf16x8(y);
            if (has[r]) {
                *reinterpret_cast<uint4*>(a.q + off[r]) = qo;
                *reinterpret_cast<uint4*>(a.k_dst + off[r]) = ko;
                *reinterpret_cast<uint4*>(a.v_dst + off[r]) = vr[r];
            }
        }
    } else {
        uint4 xr[kRowsPerHalfWarp];
#pragma unroll
        for (int r = 0; r < kRowsPerHalfWarp; ++r) xr[r] = *reinterpret_cast<const uint4*>(a.q + off[r]);
#pragma unroll
        for (int r = 0; r < kRowsPerHalfWarp; ++r) {
            float y[8];
            rope_norm_row(a.rope_cs, xr[r], sub, mask, pos[r], MODE == kRopeNorm, y);
            if (has[r]) *reinterpret_cast<uint4*>(a.q + off[r]) = f32_to_bf16x8(y);
        }
    }
}

}  // namespace

cudaError_t launch_rope(RopeMode mode, const RopeArgs& a, cudaStream_t stream) {
    const long long rows = (long long)a.seq_len * a.heads;
    if (rows <= 0) return cudaSuccess;
    const long long halfwarps = (rows + kRowsPerHalfWarp - 1) / kRowsPerHalfWarp;
    const long long threads = halfwarps * 16;
    const unsigned blocks = (unsigned)((threads + kRopeThreads - 1) / kRopeThreads);
    switch (mode) {
        case kRopeOnly:
            rope_rows_kernel<kRopeOnly><<<blocks, kRopeThreads, 0, stream>>>(a);
            break;
        case kRopeNorm:
            rope_rows_kernel<kRopeNorm><<<blocks, kRopeThreads, 0, stream>>>(a);
            break;
        case kRopeNormAppend:
            rope_rows_kernel<kRopeNormAppend><<<blocks, kRopeThreads, 0, stream>>>(a);
            break;
    }
    return cudaGetLastError();
}

// Host-side table, computed once per process with the same fp32 libm calls and the same
// expression order as the reference (kernels/rope.cu:18-26), so the device tables are
// bit-identical to the reference's d_cos_table / d_sin_table.
const std::vector<float2>& rope_table_host() {
    static std::vector<float2> table;
    static std::once_flag once;
    std::call_once(once, [] {
        table.resize((size_t)kRopeMaxSeq * kHalfDim);
        for (int pos = 0; pos < kRopeMaxSeq; pos++) {
            for (int i = 0; i < kHalfDim; i++) {
                float freq = 1.0f / powf(kRopeBase, (2.0f * i) / kHeadDim);
                float angle = pos * freq;
                table[(size_t)pos * kHalfDim + i] = make_float2(cosf(angle), sinf(angle));
            }
        }
    });
    return table;
}

cudaError_t upload_rope_table(const float2** device_table) {
    const auto& t = rope_table_host();
    cudaError_t e = cudaMemcpyToSymbol(g_rope_cs, t.data(), t.size() * sizeof(float2));
    if (e != cudaSuccess) return e;
    void* p = nullptr;
    e = cudaGetSymbolAddress(&p, g_rope_cs);
    *device_table = static_cast<const float2*>(p);
    return e;
}

}  // namespace nc

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

constexpr int kRopeThreads = 256;  // 16 rows per block

template <int MODE>
__global__ void __launch_bounds__(kRopeThreads) rope_rows_kernel(RopeArgs a) {
    const int gtid = blockIdx.x * kRopeThreads + threadIdx.x;
    const int row = gtid >> 4;  // (position, head) row handled by this half-warp
    const int sub = threadIdx.x & 15;
    const unsigned mask = (threadIdx.x & 16) ? 0xFFFF0000u : 0x0000FFFFu;
    const int nrows = a.seq_len * a.heads;
    if (row >= nrows) return;  // whole half-warps leave together
    const int s = row / a.heads;
    const int pos = a.start_pos + s;
    const size_t off = (size_t)row * kHeadDim + 8 * sub;

    if (MODE == kRopeNormAppend) {
        // Issue all three loads before any math.
        const uint4 qr = *reinterpret_cast<const uint4*>(a.q + off);
        const uint4 kr = *reinterpret_cast<const uint4*>(a.k + off);
        const uint4 vr = *reinterpret_cast<const uint4*>(a.v + off);
        float y[8];
        rope_norm_row(a.rope_cs, qr, sub, mask, pos, true, y);
        *reinterpret_cast<uint4*>(a.q + off) = f32_to_bf16x8(y);
        rope_norm_row(a.rope_cs, kr, sub, mask, pos, true, y);
        *reinterpret_cast<uint4*>(a.k_dst + off) = f32_to_bf16x8(y);
        *reinterpret_cast<uint4*>(a.v_dst + off) = vr;
    } else {
        const uint4 xr = *reinterpret_cast<const uint4*>(a.q + off);
        float y[8];
        rope_norm_row(a.rope_cs, xr, sub, mask, pos, MODE == kRopeNorm, y);
        *reinterpret_cast<uint4*>(a.q + off) = f32_to_bf16x8(y);
    }
}

}  // namespace

cudaError_t launch_rope(RopeMode mode, const RopeArgs& a, cudaStream_t stream) {
    const long long rows = (long long)a.seq_len * a.heads;
    if (rows <= 0) return cudaSuccess;
    const long long threads = rows * 16;
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

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
#include <algorithm>
#include <cmath>
#include <mutex>
#include <vector>

#include "nc_common.cuh"

namespace nc {

namespace {

// cos/sin table (10.5 MB per device), filled by upload_rope_table().
__device__ float2 g_rope_cs[kRopeMaxSeq * kHalfDim];

constexpr int kRopeThreads = 256;  // 16 half-warps per block
constexpr int kRopeBlocksPerSm = 4;

// One (position, head) row's inputs for one lane: 16 bytes of q (or x), k and v.
struct RowIn {
    uint4 q, k, v;
};

template <int MODE>
__device__ __forceinline__ RowIn load_row(const RopeArgs& a, size_t off) {
    RowIn r;
    r.q = __ldcs(reinterpret_cast<const uint4*>(a.q + off));
    if (MODE == kRopeNormAppend) {
        r.k = __ldcs(reinterpret_cast<const uint4*>(a.k + off));
        r.v = __ldcs(reinterpret_cast<const uint4*>(a.v + off));
    }
    return r;
}

// Persistent, grid-stride streaming pass: each half-warp walks rows row, row + stride, ...
// and issues the loads of its next row before it computes the current one, so every lane
// keeps two rows of loads in flight.
template <int MODE>
__global__ void __launch_bounds__(kRopeThreads) rope_rows_kernel(RopeArgs a) {
    const int hw = (blockIdx.x * kRopeThreads + threadIdx.x) >> 4;
    const int stride = (gridDim.x * kRopeThreads) >> 4;
    const int sub = threadIdx.x & 15;
    const unsigned mask = (threadIdx.x & 16) ? 0xFFFF0000u : 0x0000FFFFu;
    const int nrows = a.seq_len * a.heads;
    int row = hw;
    if (row >= nrows) return;  // whole half-warps leave together
    RowIn cur = load_row<MODE>(a, (size_t)row * kHeadDim + 8 * sub);
    for (; row < nrows; row += stride) {
        const int next = row + stride;
        RowIn nxt;
        if (next < nrows) nxt = load_row<MODE>(a, (size_t)next * kHeadDim + 8 * sub);
        const size_t off = (size_t)row * kHeadDim + 8 * sub;
        const int pos = a.start_pos + row / a.heads;
        float y[8];
        if (MODE == kRopeNormAppend) {
            rope_norm_row(a.rope_cs, cur.q, sub, mask, pos, true, y);
            __stcs(reinterpret_cast<uint4*>(a.q + off), f32_to_bf16x8(y));
            rope_norm_row(a.rope_cs, cur.k, sub, mask, pos, true, y);
            *reinterpret_cast<uint4*>(a.k_dst + off) = f32_to_bf16x8(y);
            *reinterpret_cast<uint4*>(a.v_dst + off) = cur.v;
        } else {
            rope_norm_row(a.rope_cs, cur.q, sub, mask, pos, MODE == kRopeNorm, y);
            *reinterpret_cast<uint4*>(a.q + off) = f32_to_bf16x8(y);
        }
        cur = nxt;
    }
}

}  // namespace

cudaError_t launch_rope(RopeMode mode, const RopeArgs& a, cudaStream_t stream) {
    const long long rows = (long long)a.seq_len * a.heads;
    if (rows <= 0) return cudaSuccess;
    static int sms[64] = {};
    int dev = 0;
    cudaError_t e = cudaGetDevice(&dev);
    if (e != cudaSuccess) return e;
    if (dev < 0 || dev >= 64) return cudaErrorInvalidDevice;
    if (!sms[dev]) {
        e = cudaDeviceGetAttribute(&sms[dev], cudaDevAttrMultiProcessorCount, dev);
        if (e != cudaSuccess) return e;
    }
    // Enough half-warps for every row, capped at a full persistent wave.
    const long long need = (rows * 16 + kRopeThreads - 1) / kRopeThreads;
    const unsigned blocks = (unsigned)std::min<long long>(need, (long long)sms[dev] * kRopeBlocksPerSm);
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

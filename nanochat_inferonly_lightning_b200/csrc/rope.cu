// RoPE, fused RoPE + parameter-free QK-RMSNorm, and the fused RoPE + QK-norm + KV-append
// pass that writes keys and values straight into the KV cache.
//
// Replaces reference kernels/rope.cu (init_rope_tables :14-30, rope_kernel/apply_rope :34-68,
// rope_rmsnorm_kernel/apply_rope_rmsnorm :74-158) and the two cudaMemcpyAsync cache appends
// in src/model.cpp:122-131.
//
// Mapping: eight lanes per (position, head) row.  Lane s owns the rotation pairs
// (i, i + 64) for i in [8s, 8s + 8): it loads dims [8s, 8s + 8) and [64 + 8s, 64 + 8s + 8)
// with two 16-byte loads, so the rotation needs no data from other lanes and the 128-dim
// RMS norm is a three-step butterfly over the row's eight lanes.  A warp covers four rows
// per instruction; each row half is one contiguous 128-byte segment (coalesced).
#include <algorithm>
#include <cmath>
#include <mutex>
#include <vector>

#include "nc_common.cuh"
#include "sm100_ptx.cuh"

namespace nc {

namespace {

// cos/sin table (10.5 MB per device), filled by upload_rope_table().
__device__ float2 g_rope_cs[kRopeMaxSeq * kHalfDim];

constexpr int kRopeThreads = 256;  // 32 rows per block

// One row's inputs for one lane: the low and high 16-byte slices of q (or x), k and v, and
// the lane's eight (cos, sin) pairs of the row's position.
struct RowIn {
    uint4 qlo, qhi, klo, khi, vlo, vhi;
    float4 cs[4];
};

template <int MODE>
__device__ __forceinline__ RowIn load_row(const RopeArgs& a, size_t off, int pos, int s8) {
    RowIn r;
    const float4* cs = reinterpret_cast<const float4*>(a.rope_cs + (size_t)pos * kHalfDim + 8 * s8);
#pragma unroll
    for (int i = 0; i < 4; ++i) r.cs[i] = __ldg(cs + i);
    r.qlo = __ldcs(reinterpret_cast<const uint4*>(a.q + off));
    r.qhi = __ldcs(reinterpret_cast<const uint4*>(a.q + off + 64));
    if (MODE == kRopeNormAppend) {
        r.klo = __ldcs(reinterpret_cast<const uint4*>(a.k + off));
        r.khi = __ldcs(reinterpret_cast<const uint4*>(a.k + off + 64));
        r.vlo = __ldcs(reinterpret_cast<const uint4*>(a.v + off));
        r.vhi = __ldcs(reinterpret_cast<const uint4*>(a.v + off + 64));
    }
    return r;
}

// RoPE (+ optional RMS norm) of one lane's 16 values.  Same per-element arithmetic as the
// reference (kernels/rope.cu:105-107, :137): y_lo = x_lo*c + x_hi*s, y_hi = x_hi*c - x_lo*s,
// then y * rsqrt(mean(y^2) + 1e-6), the sum of squares taken as two 8-term fma chains (low
// and high dims) added, then a butterfly over the row's eight lanes (`gmask`).
__device__ __forceinline__ void rope_norm_pairs(const float4 (&cs)[4], uint4 lo, uint4 hi,
                                                unsigned gmask, bool norm, uint4& out_lo,
                                                uint4& out_hi) {
    float xl[8], xh[8];
    bf16x8_to_f32(lo, xl);
    bf16x8_to_f32(hi, xh);
    float c[8], sn[8];
#pragma unroll
    for (int i = 0; i < 4; ++i) {
        const float4 t = cs[i];
        c[2 * i] = t.x;
        sn[2 * i] = t.y;
        c[2 * i + 1] = t.z;
        sn[2 * i + 1] = t.w;
    }
    float yl[8], yh[8];
#pragma unroll
    for (int e = 0; e < 8; ++e) {
        yl[e] = __fmaf_rn(xl[e], c[e], xh[e] * sn[e]);
        yh[e] = __fmaf_rn(xh[e], c[e], -(xl[e] * sn[e]));
    }
    if (norm) {
        float sl = 0.f, sh = 0.f;
#pragma unroll
        for (int e = 0; e < 8; ++e) {
            sl = __fmaf_rn(yl[e], yl[e], sl);
            sh = __fmaf_rn(yh[e], yh[e], sh);
        }
        float ss = sl + sh;
        ss += __shfl_xor_sync(gmask, ss, 4);
        ss += __shfl_xor_sync(gmask, ss, 2);
        ss += __shfl_xor_sync(gmask, ss, 1);
        const float r = rsqrtf(ss * (1.0f / kHeadDim) + kNormEps);
#pragma unroll
        for (int e = 0; e < 8; ++e) {
            yl[e] *= r;
            yh[e] *= r;
        }
    }
    out_lo = f32_to_bf16x8(yl);
    out_hi = f32_to_bf16x8(yh);
}

// Element offset of row `row` (lane slice s8) in k_dst / v_dst: sequence row / rps at its row
// row % rps from start_pos, in a contiguous slot (dst_stride apart) or through the page table.
// -1 when the page id is out of range (recorded in the status word).
__device__ __forceinline__ long long dst_offset(const RopeArgs& a, int row, int rps, int s8) {
    const int b = row / rps, r = row % rps;
    if (!a.page_table) return (long long)b * a.dst_stride + (long long)r * kHeadDim + 8 * s8;
    const int pos = a.start_pos + r / a.heads;
    const int page = a.page_table[(size_t)b * a.pages_per_seq + pos / a.page_rows];
    if (page < 0 || page >= a.num_pages) {
        if (s8 == 0) atomicOr(a.status, kStatusBounds);
        return -1;
    }
    return (((long long)page * a.page_rows + pos % a.page_rows) * a.heads + r % a.heads) * kHeadDim +
           8 * s8;
}

// Persistent, grid-stride streaming pass: each 8-lane group walks rows row, row + stride,
// ... and issues the loads of its next row (data and cos/sin) before it computes the
// current one.  Raw inputs
// are read with evict-first loads; outputs use ordinary stores so that they stay in L2 for
// the attention kernel that reads them next.
template <int MODE>
__global__ void __launch_bounds__(kRopeThreads) rope_rows_kernel(RopeArgs a) {
    // Lets a kernel launched after this one with programmatic stream serialization (the
    // prefill attention kernel) start its setup early; it still waits for this grid to
    // complete before it reads any of this pass's outputs.
    asm volatile("griddepcontrol.launch_dependents;");
    const int grp = (blockIdx.x * kRopeThreads + threadIdx.x) >> 3;
    const int stride = (gridDim.x * kRopeThreads) >> 3;
    const int s8 = threadIdx.x & 7;
    const unsigned gmask = 0xFFu << (threadIdx.x & 24);
    const int rps = a.seq_len * a.heads;  // rows per sequence
    const int nrows = rps * a.batch;
    int row = grp;
    if (row >= nrows) return;  // whole 8-lane groups leave together
    RowIn cur = load_row<MODE>(a, (size_t)row * kHeadDim + 8 * s8,
                               a.start_pos + (row % rps) / a.heads, s8);
    for (; row < nrows; row += stride) {
        const int next = row + stride;
        RowIn nxt;
        if (next < nrows)
            nxt = load_row<MODE>(a, (size_t)next * kHeadDim + 8 * s8,
                                 a.start_pos + (next % rps) / a.heads, s8);
        const size_t off = (size_t)row * kHeadDim + 8 * s8;
        uint4 ol, oh;
        if (MODE == kRopeNormAppend) {
            rope_norm_pairs(cur.cs, cur.qlo, cur.qhi, gmask, true, ol, oh);
            *reinterpret_cast<uint4*>(a.q + off) = ol;
            *reinterpret_cast<uint4*>(a.q + off + 64) = oh;
            rope_norm_pairs(cur.cs, cur.klo, cur.khi, gmask, true, ol, oh);
            const long long doff = dst_offset(a, row, rps, s8);
            if (doff >= 0) {
                *reinterpret_cast<uint4*>(a.k_dst + doff) = ol;
                *reinterpret_cast<uint4*>(a.k_dst + doff + 64) = oh;
                *reinterpret_cast<uint4*>(a.v_dst + doff) = cur.vlo;
                *reinterpret_cast<uint4*>(a.v_dst + doff + 64) = cur.vhi;
            }
        } else {
            rope_norm_pairs(cur.cs, cur.qlo, cur.qhi, gmask, MODE == kRopeNorm, ol, oh);
            *reinterpret_cast<uint4*>(a.q + off) = ol;
            *reinterpret_cast<uint4*>(a.q + off + 64) = oh;
        }
        cur = nxt;
    }
}

template <int MODE>
cudaError_t launch_rope_mode(const RopeArgs& a, long long rows, int dev, cudaStream_t stream) {
    // Persistent wave: as many blocks as are resident at once on the device (occupancy
    // queried once per device), or fewer when there are fewer rows.
    static int wave[64] = {};
    if (!wave[dev]) {
        int sms = 0, per_sm = 0;
        cudaError_t e = cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev);
        if (e != cudaSuccess) return e;
        e = cudaOccupancyMaxActiveBlocksPerMultiprocessor(&per_sm, rope_rows_kernel<MODE>,
                                                          kRopeThreads, 0);
        if (e != cudaSuccess) return e;
        wave[dev] = sms * std::max(per_sm, 1);
    }
    const long long need = (rows * 8 + kRopeThreads - 1) / kRopeThreads;
    const unsigned blocks = (unsigned)std::min<long long>(need, wave[dev]);
    rope_rows_kernel<MODE><<<blocks, kRopeThreads, 0, stream>>>(a);
    return cudaGetLastError();
}

}  // namespace

cudaError_t launch_rope(RopeMode mode, const RopeArgs& a, cudaStream_t stream) {
    const long long rows = (long long)a.seq_len * a.heads * a.batch;
    if (rows <= 0) return cudaSuccess;
    int dev = 0;
    cudaError_t e = cudaGetDevice(&dev);
    if (e != cudaSuccess) return e;
    if (dev < 0 || dev >= 64) return cudaErrorInvalidDevice;
    switch (mode) {
        case kRopeOnly: return launch_rope_mode<kRopeOnly>(a, rows, dev, stream);
        case kRopeNorm: return launch_rope_mode<kRopeNorm>(a, rows, dev, stream);
        case kRopeNormAppend: return launch_rope_mode<kRopeNormAppend>(a, rows, dev, stream);
    }
    return cudaErrorInvalidValue;
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

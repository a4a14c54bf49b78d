// Shared device helpers and the launch entry points that the host API layer calls.
#pragma once

#include <cuda_bf16.h>
#include <cuda_runtime.h>
#include <cstddef>
#include <cstdint>

namespace nc {

// Model geometry fixed by the reference engine (src/config.h:12, :17).
constexpr int kHeadDim = 128;
constexpr int kHalfDim = kHeadDim / 2;
constexpr int kRopeMaxSeq = 2048 * 10;  // positions covered by the cos/sin table
constexpr float kRopeBase = 10000.0f;
constexpr float kNormEps = 1e-6f;
constexpr float kLog2e = 1.4426950408889634f;

using bf16 = __nv_bfloat16;

// ---------------------------------------------------------------------------------------
// small device utilities
// ---------------------------------------------------------------------------------------
__device__ __forceinline__ uint4 ldg_stream(const void* p) {
    uint4 r;
    asm volatile("ld.global.nc.L1::no_allocate.v4.u32 {%0,%1,%2,%3}, [%4];"
                 : "=r"(r.x), "=r"(r.y), "=r"(r.z), "=r"(r.w)
                 : "l"(p));
    return r;
}

__device__ __forceinline__ void bf16x8_to_f32(const uint4& v, float (&f)[8]) {
    const uint32_t w[4] = {v.x, v.y, v.z, v.w};
#pragma unroll
    for (int i = 0; i < 4; ++i) {
        f[2 * i] = __uint_as_float(w[i] << 16);
        f[2 * i + 1] = __uint_as_float(w[i] & 0xFFFF0000u);
    }
}

__device__ __forceinline__ uint32_t pack_bf16x2(float lo, float hi) {
    __nv_bfloat162 h = __floats2bfloat162_rn(lo, hi);
    return *reinterpret_cast<uint32_t*>(&h);
}

__device__ __forceinline__ uint4 f32_to_bf16x8(const float (&f)[8]) {
    uint4 r;
    r.x = pack_bf16x2(f[0], f[1]);
    r.y = pack_bf16x2(f[2], f[3]);
    r.z = pack_bf16x2(f[4], f[5]);
    r.w = pack_bf16x2(f[6], f[7]);
    return r;
}

__device__ __forceinline__ float fast_exp2(float x) {
    float y;
    asm("ex2.approx.ftz.f32 %0, %1;" : "=f"(y) : "f"(x));
    return y;
}

// 2^x on the FMA pipe, for x <= 8 (anything below -127 gives 0): range reduction
// x = n + f with n = round(x) and f in [-1/2, 1/2] (the 1.5 * 2^23 rounding trick), a cubic
// for 2^f, and n added straight into the exponent bits.  The cubic 1 + c1 f + c2 f^2 + c3 f^3
// is a minimax fit of 2^f on [-1/2, 1/2] with the constant term pinned to 1 (made for this
// kernel; max relative error 1.0e-4, against 3.9e-3 for one bf16 half-ulp), so x = -127
// yields exactly +0.  Used for part of the softmax exponentials to relieve the MUFU pipe.
__device__ __forceinline__ float exp2_poly(float x) {
    x = fmaxf(x, -127.0f);
    const float r = x + 12582912.0f;
    const float f = x - (r - 12582912.0f);
    float p = __fmaf_rn(0.05500893f, f, 0.24221095f);
    p = __fmaf_rn(p, f, 0.6932829f);
    p = __fmaf_rn(p, f, 1.0f);
    return __int_as_float(__float_as_int(p) + ((__float_as_int(r) - 0x4B400000) << 23));
}

// Packed pairs of fp32 (Blackwell f32x2 arithmetic: one instruction, two lanes of work).
__device__ __forceinline__ uint64_t f2_pack(float lo, float hi) {
    uint64_t r;
    asm("mov.b64 %0, {%1, %2};" : "=l"(r) : "f"(lo), "f"(hi));
    return r;
}
__device__ __forceinline__ void f2_unpack(uint64_t v, float& lo, float& hi) {
    asm("mov.b64 {%0, %1}, %2;" : "=f"(lo), "=f"(hi) : "l"(v));
}
__device__ __forceinline__ uint64_t f2_fma(uint64_t a, uint64_t b, uint64_t c) {
    uint64_t r;
    asm("fma.rn.f32x2 %0, %1, %2, %3;" : "=l"(r) : "l"(a), "l"(b), "l"(c));
    return r;
}
__device__ __forceinline__ uint64_t f2_add(uint64_t a, uint64_t b) {
    uint64_t r;
    asm("add.rn.f32x2 %0, %1, %2;" : "=l"(r) : "l"(a), "l"(b));
    return r;
}

// exp2_poly on a packed pair (same method and coefficients); the clamp and the exponent
// insertion are per element.  Because 0x4B400000 << 23 wraps to 0 in 32 bits, adding
// (rounded << 23) to the polynomial's bits inserts the integer part directly.
__device__ __forceinline__ void exp2_poly2(float x0, float x1, float& p0, float& p1) {
    x0 = fmaxf(x0, -127.0f);
    x1 = fmaxf(x1, -127.0f);
    const uint64_t x = f2_pack(x0, x1);
    const uint64_t magic = f2_pack(12582912.0f, 12582912.0f);
    const uint64_t nmagic = f2_pack(-12582912.0f, -12582912.0f);
    const uint64_t r = f2_add(x, magic);
    const uint64_t n = f2_add(r, nmagic);
    float n0, n1;
    f2_unpack(n, n0, n1);
    const uint64_t f = f2_add(x, f2_pack(-n0, -n1));
    uint64_t q = f2_fma(f2_pack(0.05500893f, 0.05500893f), f, f2_pack(0.24221095f, 0.24221095f));
    q = f2_fma(q, f, f2_pack(0.6932829f, 0.6932829f));
    q = f2_fma(q, f, f2_pack(1.0f, 1.0f));
    float q0, q1, r0, r1;
    f2_unpack(q, q0, q1);
    f2_unpack(r, r0, r1);
    p0 = __int_as_float(__float_as_int(q0) + (__float_as_int(r0) << 23));
    p1 = __int_as_float(__float_as_int(q1) + (__float_as_int(r1) << 23));
}

// RoPE (+ optional parameter-free RMSNorm) of one 128-wide head row held by a half-warp:
// lane `sub` (0..15) owns dims [8*sub, 8*sub+8).  Half-split pairing (dim i with i+64,
// reference kernels/rope.cu:95-97) puts a lane's partner at sub^8.  `mask` is the
// half-warp's shuffle mask.  Rotation: y0 = x0*c + x1*s, y1 = x1*c - x0*s
// (kernels/rope.cu:105-107); the norm is y * rsqrt(mean(y^2) + 1e-6) (kernels/rope.cu:137).
// `cs` is the interleaved cos/sin table: cs[pos * 64 + i] = (cos(pos*f_i), sin(pos*f_i)).
__device__ __forceinline__ void rope_norm_row(const float2* __restrict__ cs_table,
                                              const uint4 raw, int sub, unsigned mask, int pos,
                                              bool norm, float (&y)[8]) {
    uint4 pr;
    pr.x = __shfl_xor_sync(mask, raw.x, 8);
    pr.y = __shfl_xor_sync(mask, raw.y, 8);
    pr.z = __shfl_xor_sync(mask, raw.z, 8);
    pr.w = __shfl_xor_sync(mask, raw.w, 8);
    float xo[8], xp[8];
    bf16x8_to_f32(raw, xo);
    bf16x8_to_f32(pr, xp);
    const float4* cs = reinterpret_cast<const float4*>(cs_table + (size_t)pos * kHalfDim +
                                                       8 * (sub & 7));
    float c[8], s[8];
#pragma unroll
    for (int i = 0; i < 4; ++i) {
        const float4 t = __ldg(cs + i);
        c[2 * i] = t.x;
        s[2 * i] = t.y;
        c[2 * i + 1] = t.z;
        s[2 * i + 1] = t.w;
    }
    if (sub < 8) {
#pragma unroll
        for (int e = 0; e < 8; ++e) y[e] = __fmaf_rn(xo[e], c[e], xp[e] * s[e]);
    } else {
#pragma unroll
        for (int e = 0; e < 8; ++e) y[e] = __fmaf_rn(xo[e], c[e], -(xp[e] * s[e]));
    }
    if (norm) {
        float ss = 0.f;
#pragma unroll
        for (int e = 0; e < 8; ++e) ss = __fmaf_rn(y[e], y[e], ss);
        ss += __shfl_xor_sync(mask, ss, 8);
        ss += __shfl_xor_sync(mask, ss, 4);
        ss += __shfl_xor_sync(mask, ss, 2);
        ss += __shfl_xor_sync(mask, ss, 1);
        const float r = rsqrtf(ss * (1.0f / kHeadDim) + kNormEps);
#pragma unroll
        for (int e = 0; e < 8; ++e) y[e] *= r;
    }
}

// ---------------------------------------------------------------------------------------
// launch entry points (defined in rope.cu / decode.cu / prefill.cu)
// ---------------------------------------------------------------------------------------
enum RopeMode : int { kRopeOnly = 0, kRopeNorm = 1, kRopeNormAppend = 2 };

struct RopeArgs {
    const float2* rope_cs;  // device cos/sin table
    bf16* q;              // [rows, heads, 128]; modified in place
    const bf16* k;        // append mode: [rows, heads, 128] pre-RoPE keys
    const bf16* v;        // append mode: [rows, heads, 128] values
    bf16* k_dst;          // append mode: destination rows (cache row start_pos)
    bf16* v_dst;
    int seq_len;
    int heads;
    int start_pos;
    // Append mode over several sequences: q, k, v hold batch x seq_len rows, sequence b's
    // rows go to k_dst / v_dst + b * dst_stride elements (its cache, from row start_pos).
    int batch = 1;
    long long dst_stride = 0;
    // Paged destination (page_table != null): k_dst / v_dst are pools
    // [num_pages][page_rows][heads][128]; position p of sequence b goes to row p % page_rows of
    // page page_table[b * pages_per_seq + p / page_rows].  A page id outside [0, num_pages) ORs
    // 0x400 into *status and the row is not written.
    const int* page_table = nullptr;
    int pages_per_seq = 0, page_rows = 0, num_pages = 0;
    int* status = nullptr;
};

cudaError_t launch_rope(RopeMode mode, const RopeArgs& a, cudaStream_t stream);
// Uploads the table to the current device and returns its device address there.
cudaError_t upload_rope_table(const float2** device_table);

struct DecodeArgs {
    const float2* rope_cs;        // device cos/sin table (fused RoPE only)
    bf16* out;                    // [B, heads*128]
    const bf16* q;                // [B, heads, 128]
    const bf16* k_new;            // [B, heads, 128] pre-RoPE key of the new token, or null
    const bf16* v_new;            // [B, heads, 128] value of the new token, or null
    bf16* const* k_cache;         // device array [B] of per-sequence K bases, or null
    bf16* const* v_cache;
    bf16* k_single;               // single-sequence mode (B == 1): K base, used if k_cache null
    bf16* v_single;
    const int* kv_len;            // device [B] visible keys, or null (then n_visible_single)
    int n_visible_single;
    int max_kv_len;               // host bound on kv_len[b]; sized the grid and workspace
    int batch;
    int heads;
    int q_raw;                    // 1: q is pre-RoPE and gets RoPE + QK-norm in the kernel
    // Paged cache (page_table != null): row r of sequence b is row r % page_rows of page
    // page_table[b * pages_per_seq + r / page_rows] of k_pool / v_pool, pools laid out
    // [num_pages][page_rows][heads][128]; k_cache / v_cache / k_single are then unused.
    bf16* k_pool;
    bf16* v_pool;
    const int* page_table;
    int page_rows;                // multiple of 16
    int pages_per_seq;
    int num_pages;
    int head_layout;              // 1: per-head layout (decode_use_head_layout)
    int overlap;                  // 1: per-head layout launched as a programmatic dependent
                                  // launch; cache rows, lengths and pointer tables are read
                                  // before griddepcontrol.wait (q, k_new, v_new after it)
    float scale_log2;             // softmax scale * log2(e)
    int split_len;                // keys per split (multiple of 16)
    int max_splits;
    float* part_o;                // [B, max_splits, heads, 128]
    float2* part_ml;              // [B, max_splits, heads]
    unsigned* counters;           // decode_counter_words(B, heads), zero between launches
    int* status;                  // device status word (argument violations seen on device)
};

cudaError_t launch_decode(const DecodeArgs& a, cudaStream_t stream);
// Small decode calls run the per-head layout: one CTA per (split, head, sequence) with at
// most kDecodeHeadSplit keys per split.  It is chosen for at most kDecodeHeadMaxBatch sequences
// and, with automatic splits, at most kDecodeHeadMaxKeys keys in total (batch * max_kv_len).
// With the cache rows staged in shared memory (six CTAs per SM), measured at 8 sequences of
// cfg3's lengths (longest ~2048): 22.1 / 18.5 / 26.7 us against 24.7 / 22.3 / 29.1 for the
// streaming layout, and at 8 x 4096 keys 65.3 against 59.6, so the bound is 8 x 2048.  Up to
// 16 sequences: cfg3's 8-way shards of 9-10 sequences take 22.7-22.9 us against 25.7-26.0 on
// the streaming layout, 12 x 1024 keys 29.0 against 35.1, 16 x 300 17.2 against 18.7 (evenly
// long 9-12 sequences of 600-850 keys lose 0.7-1.6 us).  An explicit split length above
// kDecodeHeadSplit selects the streaming layout.
constexpr int kDecodeHeadMaxBatch = 16;
constexpr int kDecodeHeadSplit = 64;
constexpr long long kDecodeHeadMaxKeys = 16384;
inline bool decode_use_head_layout(int batch, int max_kv_len, int split_len) {
    if (batch > kDecodeHeadMaxBatch) return false;
    if (split_len) return split_len <= kDecodeHeadSplit;
    return (long long)batch * max_kv_len <= kDecodeHeadMaxKeys;
}
// Per-head calls with 2..16 splits combine them inside a thread-block cluster (distributed
// shared memory), without global partials, tickets or workspace; not when the call overlaps
// the kernel before it (programmatic dependent launch).  Above 8 splits only while the call
// has few clusters to place (batch x splits <= 64): each cluster must fit whole in one GPC
// beside the other CTAs.  Measured (one call, cold cache): 8 x 1024 keys (16 splits) 26.8 us
// with clusters against 22.7 with the global combine, 8 x 700 (11) 20.7 / 18.5, 4 x 1024
// 16.7 / 16.6, but 1 x 1024 8.8 / 10.3 and 2 x 600 (10) 9.2 / 10.6.
constexpr int kDecodeHeadMaxCluster = 16;
inline bool decode_head_cluster(int max_splits, int batch, bool overlap) {
    if (overlap || max_splits < 2 || max_splits > kDecodeHeadMaxCluster) return false;
    return max_splits <= 8 || (long long)batch * max_splits <= 64;
}
size_t decode_workspace_bytes(int batch, int max_splits, int heads);
// 32-bit words at the start of the decode workspace: two work-queue words, then one split
// ticket per (sequence, head).  All zero between launches.
size_t decode_counter_words(int batch, int heads);

struct PrefillArgs {
    bf16* out;                    // [B, seq_q, heads*128]
    const bf16* q;                // [B, seq_q, heads, 128]
    const bf16* k;                // K rows of sequence b start at k + b*kv_batch_stride
    const bf16* v;
    long long kv_batch_stride;    // elements between sequences (0 when B == 1)
    int kv_rows;                  // rows addressable per sequence (tensor-map extent)
    const int* kv_offset_dev;     // device [B] offsets, or null (then kv_offset / kv_len)
    int kv_offset;
    int kv_len;
    int batch;
    int seq_q;
    int heads;
    float scale;
    int* status;                  // device status word for bounded waits
    // Paged cache (page_table != null): k / v are pools [num_pages][page_rows][heads][128],
    // page_rows a multiple of 128, and key row r of sequence b is row r % page_rows of page
    // page_table[b * pages_per_seq + r / page_rows].
    const int* page_table;
    int page_rows;
    int pages_per_seq;
    int num_pages;
};

cudaError_t launch_prefill(const PrefillArgs& a, cudaStream_t stream);

// Host-side per-device state owned by api.cu, for other entry points of the library:
// the RoPE table's device address (uploaded on first use) and the kernel status word.
// Both return an nc_status.
int internal_rope_table(const float2** table);
int internal_status_word(int** status);
// Records `e` as this thread's last CUDA error and returns NC_ERR_CUDA.
int internal_cuda_fail(cudaError_t e);
// Keys per split that nc_decode_attention picks for `batch` sequences of up to `max_kv_len`
// keys when the caller passes split_len 0.
int internal_auto_split_len(int batch, int max_kv_len);

}  // namespace nc

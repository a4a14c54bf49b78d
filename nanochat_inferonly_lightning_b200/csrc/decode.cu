// Split-KV flash-decoding over the KV cache, with RoPE + QK-norm of the query and the
// RoPE + QK-norm + append of the new token's key/value fused into the same pass.
//
// Replaces the seq_q == 1 use of reference kernels/flash_attention.cu:19-171 (one CTA per
// head streaming every key with 2-byte loads), and, in the fused form, also
// apply_rope_rmsnorm(q), apply_rope_rmsnorm(k) and the two cache-append copies of
// src/model.cpp:119-131.
//
// Layout: K/V cache rows are [heads, 128] bf16 (4352 B for 17 heads).  Grid (split, seq):
// each CTA owns `split_len` consecutive keys of one sequence and all heads; warp h = head h.
// Inside a warp, lanes 0-15 take even keys and 16-31 odd keys; lane (sub = lane & 15) owns
// dims [8*sub, 8*sub+8), so every load is a 16-byte vector and each half-warp reads one whole
// 256-byte head row.  Eight keys per warp are in flight per iteration (4 K + 4 V loads per
// lane).  Each half-warp keeps its own online-softmax state (max in log2 units, sum, 8
// accumulators); the halves merge at the end, and splits merge through a small fp32
// workspace in the last CTA of each sequence to finish (atomic ticket, self-resetting).
#include "nc_common.cuh"

namespace nc {

namespace {

constexpr int kUnroll = 4;  // keys per half-warp per iteration
constexpr int kStatusDecodeBound = 0x200;  // a kv_len exceeded max_kv_len
constexpr float kNegInf = -__builtin_huge_valf();

__device__ __forceinline__ float dot8(const float (&q)[8], const uint4 kv) {
    float k[8];
    bf16x8_to_f32(kv, k);
    float s = 0.f;
#pragma unroll
    for (int e = 0; e < 8; ++e) s = __fmaf_rn(q[e], k[e], s);
    return s;
}

__global__ void __launch_bounds__(1024) decode_kernel(DecodeArgs a) {
    const int b = blockIdx.y;
    const int split = blockIdx.x;
    const int h = threadIdx.x >> 5;
    const int lane = threadIdx.x & 31;
    const int half = lane >> 4;
    const int sub = lane & 15;
    const unsigned hmask = half ? 0xFFFF0000u : 0x0000FFFFu;
    const int H = a.heads;
    const size_t rowstride = (size_t)H * kHeadDim;

    int L = a.kv_len ? a.kv_len[b] : a.n_visible_single;
    bf16* out_row = a.out + (size_t)b * rowstride;
    if (L <= 0) {
        // No visible key: the reference's 0/0 yields NaN (flash_attention.cu:155).
        if (split == 0 && half == 0) {
            const uint4 nan4 = make_uint4(0x7FC07FC0u, 0x7FC07FC0u, 0x7FC07FC0u, 0x7FC07FC0u);
            *reinterpret_cast<uint4*>(out_row + h * kHeadDim + 8 * sub) = nan4;
        }
        return;
    }
    if (L > a.max_kv_len) {
        // kv_len[b] above the caller's bound (which sized the grid and the workspace): clamp,
        // so no access leaves the promised rows, and flag it.
        if (split == 0 && threadIdx.x == 0 && a.status) atomicOr(a.status, kStatusDecodeBound);
        L = a.max_kv_len;
    }
    const int n_splits = (L + a.split_len - 1) / a.split_len;
    if (split >= n_splits) return;
    const int ks = split * a.split_len;
    const int ke = min(L, ks + a.split_len);
    const bool fuse_new = a.k_new != nullptr;
    const bool owns_new = fuse_new && (split == n_splits - 1);
    const int ke_stream = owns_new ? ke - 1 : ke;  // the new key is handled from registers

    bf16* Kb = a.k_cache ? a.k_cache[b] : a.k_single;
    bf16* Vb = a.v_cache ? a.v_cache[b] : a.v_single;
    const size_t head_off = (size_t)h * kHeadDim + 8 * sub;
    const int pos = L - 1;  // position of the query token

    // Query: optional RoPE + QK-norm, rounded to bf16 like the unfused path, then
    // pre-scaled so dot products come out in log2 units.
    float qf[8];
    {
        const uint4 qr = *reinterpret_cast<const uint4*>(a.q + (size_t)b * rowstride + head_off);
        if (a.q_raw) {
            float y[8];
            rope_norm_row(a.rope_cs, qr, sub, hmask, pos, true, y);
            bf16x8_to_f32(f32_to_bf16x8(y), qf);
        } else {
            bf16x8_to_f32(qr, qf);
        }
#pragma unroll
        for (int e = 0; e < 8; ++e) qf[e] *= a.scale_log2;
    }

    float m = kNegInf, l = 0.f, acc[8];
#pragma unroll
    for (int e = 0; e < 8; ++e) acc[e] = 0.f;

    const bf16* kp = Kb + head_off;
    const bf16* vp = Vb + head_off;
    for (int k0 = ks; k0 < ke_stream; k0 += 2 * kUnroll) {
        uint4 kr[kUnroll], vr[kUnroll];
        bool valid[kUnroll];
#pragma unroll
        for (int i = 0; i < kUnroll; ++i) {
            const int key = k0 + 2 * i + half;
            valid[i] = key < ke_stream;
            kr[i] = valid[i] ? ldg_stream(kp + (size_t)key * rowstride) : make_uint4(0, 0, 0, 0);
        }
#pragma unroll
        for (int i = 0; i < kUnroll; ++i) {
            const int key = k0 + 2 * i + half;
            vr[i] = valid[i] ? ldg_stream(vp + (size_t)key * rowstride) : make_uint4(0, 0, 0, 0);
        }
        float s[kUnroll];
#pragma unroll
        for (int i = 0; i < kUnroll; ++i) s[i] = dot8(qf, kr[i]);
#pragma unroll
        for (int i = 0; i < kUnroll; ++i) {
            s[i] += __shfl_xor_sync(0xFFFFFFFFu, s[i], 8);
            s[i] += __shfl_xor_sync(0xFFFFFFFFu, s[i], 4);
            s[i] += __shfl_xor_sync(0xFFFFFFFFu, s[i], 2);
            s[i] += __shfl_xor_sync(0xFFFFFFFFu, s[i], 1);
            if (!valid[i]) s[i] = kNegInf;
        }
        float mx = s[0];
#pragma unroll
        for (int i = 1; i < kUnroll; ++i) mx = fmaxf(mx, s[i]);
        const float m_new = fmaxf(m, mx);
        const float mu = (m_new == kNegInf) ? 0.f : m_new;
        const float alpha = fast_exp2(m - mu);
        float p[kUnroll], psum = 0.f;
#pragma unroll
        for (int i = 0; i < kUnroll; ++i) {
            p[i] = fast_exp2(s[i] - mu);
            psum += p[i];
        }
        l = __fmaf_rn(l, alpha, psum);
#pragma unroll
        for (int e = 0; e < 8; ++e) acc[e] *= alpha;
#pragma unroll
        for (int i = 0; i < kUnroll; ++i) {
            float v[8];
            bf16x8_to_f32(vr[i], v);
#pragma unroll
            for (int e = 0; e < 8; ++e) acc[e] = __fmaf_rn(p[i], v[e], acc[e]);
        }
        m = m_new;
    }

    if (owns_new) {
        // New token: RoPE + QK-norm of its key, append K and V to the cache, and add its
        // contribution (lanes of half 0 only; half 1 contributes nothing for this key).
        const size_t in_off = (size_t)b * rowstride + head_off;
        const uint4 kr = *reinterpret_cast<const uint4*>(a.k_new + in_off);
        const uint4 vr = *reinterpret_cast<const uint4*>(a.v_new + in_off);
        float y[8];
        rope_norm_row(a.rope_cs, kr, sub, hmask, pos, true, y);
        const uint4 kn = f32_to_bf16x8(y);
        if (half == 0) {
            *reinterpret_cast<uint4*>(Kb + (size_t)pos * rowstride + head_off) = kn;
            *reinterpret_cast<uint4*>(Vb + (size_t)pos * rowstride + head_off) = vr;
        }
        float s = dot8(qf, kn);
        s += __shfl_xor_sync(0xFFFFFFFFu, s, 8);
        s += __shfl_xor_sync(0xFFFFFFFFu, s, 4);
        s += __shfl_xor_sync(0xFFFFFFFFu, s, 2);
        s += __shfl_xor_sync(0xFFFFFFFFu, s, 1);
        if (half == 0) {
            const float m_new = fmaxf(m, s);
            const float alpha = fast_exp2(m - m_new);
            const float p = fast_exp2(s - m_new);
            l = __fmaf_rn(l, alpha, p);
            float v[8];
            bf16x8_to_f32(vr, v);
#pragma unroll
            for (int e = 0; e < 8; ++e) acc[e] = __fmaf_rn(p, v[e], acc[e] * alpha);
            m = m_new;
        }
    }

    // Merge the two half-warps (same dims, disjoint keys).
    {
        const float m_o = __shfl_xor_sync(0xFFFFFFFFu, m, 16);
        const float l_o = __shfl_xor_sync(0xFFFFFFFFu, l, 16);
        const float M = fmaxf(m, m_o);
        const float mu = (M == kNegInf) ? 0.f : M;
        const float wa = fast_exp2(m - mu), wb = fast_exp2(m_o - mu);
        l = l * wa + l_o * wb;
#pragma unroll
        for (int e = 0; e < 8; ++e) {
            const float o = __shfl_xor_sync(0xFFFFFFFFu, acc[e], 16);
            acc[e] = acc[e] * wa + o * wb;
        }
        m = M;
    }

    if (n_splits == 1) {
        if (half == 0) {
            const float inv = 1.0f / l;
            float o[8];
#pragma unroll
            for (int e = 0; e < 8; ++e) o[e] = acc[e] * inv;
            *reinterpret_cast<uint4*>(out_row + head_off) = f32_to_bf16x8(o);
        }
        return;
    }

    // Partial result of this split.
    const size_t pidx = ((size_t)b * a.max_splits + split) * H + h;
    if (half == 0) {
        float4* po = reinterpret_cast<float4*>(a.part_o + pidx * kHeadDim + 8 * sub);
        __stcg(po, make_float4(acc[0], acc[1], acc[2], acc[3]));
        __stcg(po + 1, make_float4(acc[4], acc[5], acc[6], acc[7]));
        if (sub == 0) __stcg(a.part_ml + pidx, make_float2(m, l));
    }
    __threadfence();
    __syncthreads();
    __shared__ unsigned s_ticket;
    if (threadIdx.x == 0) s_ticket = atomicAdd(a.counters + b, 1u);
    __syncthreads();
    if (s_ticket != (unsigned)(n_splits - 1)) return;

    // Last CTA of this sequence: combine every split.  Warp h = head h; lanes read the
    // split maxima in parallel, then each lane owns dims [4*lane, 4*lane+4) and keeps eight
    // splits' partial rows in flight per round.
    __threadfence();
    if (threadIdx.x == 0) a.counters[b] = 0u;  // ready for the next launch
    const size_t base = (size_t)b * a.max_splits * H + h;  // (b, split 0, h); split stride H
    float M = kNegInf;
    for (int sp = lane; sp < n_splits; sp += 32) M = fmaxf(M, __ldcg(a.part_ml + base + (size_t)sp * H).x);
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) M = fmaxf(M, __shfl_xor_sync(0xFFFFFFFFu, M, o));
    const float mu = (M == kNegInf) ? 0.f : M;
    float den = 0.f, o4[4] = {0.f, 0.f, 0.f, 0.f};
    for (int sp0 = 0; sp0 < n_splits; sp0 += 8) {
        float2 ml[8];
        float4 v[8];
#pragma unroll
        for (int i = 0; i < 8; ++i) {
            const int sp = sp0 + i;
            if (sp < n_splits) {
                const size_t pi = base + (size_t)sp * H;
                ml[i] = __ldcg(a.part_ml + pi);
                v[i] = __ldcg(reinterpret_cast<const float4*>(a.part_o + pi * kHeadDim) + lane);
            } else {
                ml[i] = make_float2(kNegInf, 0.f);
                v[i] = make_float4(0.f, 0.f, 0.f, 0.f);
            }
        }
#pragma unroll
        for (int i = 0; i < 8; ++i) {
            const float w = fast_exp2(ml[i].x - mu);
            den = __fmaf_rn(ml[i].y, w, den);
            o4[0] = __fmaf_rn(v[i].x, w, o4[0]);
            o4[1] = __fmaf_rn(v[i].y, w, o4[1]);
            o4[2] = __fmaf_rn(v[i].z, w, o4[2]);
            o4[3] = __fmaf_rn(v[i].w, w, o4[3]);
        }
    }
    const float inv = 1.0f / den;
    uint2 r;
    r.x = pack_bf16x2(o4[0] * inv, o4[1] * inv);
    r.y = pack_bf16x2(o4[2] * inv, o4[3] * inv);
    *reinterpret_cast<uint2*>(out_row + (size_t)h * kHeadDim + 4 * lane) = r;
}

}  // namespace

size_t decode_workspace_bytes(int batch, int max_splits, int heads) {
    const size_t n = (size_t)batch * max_splits * heads;
    size_t bytes = ((size_t)batch * sizeof(unsigned) + 255) & ~(size_t)255;  // counters
    bytes = (bytes + n * sizeof(float2) + 255) & ~(size_t)255;                 // part_ml
    bytes += n * kHeadDim * sizeof(float);                                     // part_o
    return (bytes + 255) & ~(size_t)255;
}

cudaError_t launch_decode(const DecodeArgs& a, cudaStream_t stream) {
    if (a.batch <= 0) return cudaSuccess;
    dim3 grid(a.max_splits, a.batch);
    decode_kernel<<<grid, a.heads * 32, 0, stream>>>(a);
    return cudaGetLastError();
}

}  // namespace nc

// Split-KV flash-decoding over the KV cache, with RoPE + QK-norm of the query and the
// RoPE + QK-norm + append of the new token's key/value fused into the same pass.
//
// Replaces the seq_q == 1 use of reference kernels/flash_attention.cu:19-171 (one CTA per
// head streaming every key with 2-byte loads), and, in the fused form, also
// apply_rope_rmsnorm(q), apply_rope_rmsnorm(k) and the two cache-append copies of
// src/model.cpp:119-131.
//
// Work items are (sequence, split): `split_len` consecutive keys of one sequence, all heads.
// The kernel is persistent (at most one CTA per SM, never more CTAs than items).  Lane 0 of
// the last warp is the producer: its first item is its CTA index, further items (when there
// are more items than CTAs) come from a global atomic counter; it streams each item's K and V rows (a cache row
// holds every head, heads*256 contiguous bytes, so R rows are one contiguous block) into a
// three-stage shared-memory ring with bulk asynchronous copies (cp.async.bulk, completion on
// an mbarrier).  The bytes in flight per SM are therefore set by the ring (three stages of
// 2*R rows, ~200 KB), not by registers.  Warp h (< heads) consumes head h: half-warp 0 takes
// even rows and half-warp 1 odd rows of each stage, lane `sub` reads dims [8*sub, 8*sub+8) of
// its head with 16-byte shared-memory loads, and keeps an online softmax (max in log2 units,
// sum, 8 fp32 accumulators).  At the end of an item the halves merge, and the split either
// writes the output directly (single-split sequence) or a partial result; the last split of
// each (sequence, head) to finish (per-head atomic ticket, self-resetting) combines them.
#include <cooperative_groups.h>

#include <algorithm>

#include "nc_common.cuh"
#include "sm100_ptx.cuh"

namespace nc {

namespace {

constexpr int kStages = 3;
constexpr int kStatusDecodeBound = 0x200;  // a kv_len exceeded max_kv_len
constexpr float kNegInf = -__builtin_huge_valf();
constexpr int kQueueWords = 2;  // counters[0]: next work item; counters[1]: CTAs done fetching

// Stage header, written by the producer before it arms the stage's full barrier.
struct StageHdr {
    int b;           // sequence, or -1: no more work
    int first;       // first row of this stage (absolute key index)
    int nrows;       // rows in this stage (0 for an item made of the new key only)
    int item_first;  // 1 if this stage starts an item
    int item_last;   // 1 if this stage ends an item
    int split;
    int n_splits;
    int L;           // visible keys of the sequence
};

struct __align__(8) DecTail {
    uint64_t full[kStages];
    uint64_t empty[kStages];
    StageHdr hdr[kStages];
    int abort;
};

__device__ __forceinline__ void bulk_g2s(void* dst, const void* src, uint32_t bytes, uint64_t* bar) {
    asm volatile(
        "cp.async.bulk.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1], %2, [%3];" ::"r"(
            smem_u32(dst)),
        "l"(src), "r"(bytes), "r"(smem_u32(bar))
        : "memory");
}

__device__ __forceinline__ float dot8(const float (&q)[8], const uint4 kv) {
    float k[8];
    bf16x8_to_f32(kv, k);
    float s = 0.f;
#pragma unroll
    for (int e = 0; e < 8; ++e) s = __fmaf_rn(q[e], k[e], s);
    return s;
}

__device__ __forceinline__ int raw_len(const DecodeArgs& a, int b) {
    return a.kv_len ? a.kv_len[b] : a.n_visible_single;
}

// Start of cache row r of sequence b, K (v == false) or V.  Contiguous caches: the sequence's
// base + r rows.  Paged caches: the row's page from the page table; a page id outside
// [0, num_pages) sets kStatusBounds and yields null (callers then skip the access).
template <bool PAGED>
__device__ __forceinline__ bf16* kv_row(const DecodeArgs& a, bool v, int b, int r) {
    const size_t rowstride = (size_t)a.heads * kHeadDim;
    if (PAGED) {
        const int page = a.page_table[(size_t)b * a.pages_per_seq + r / a.page_rows];
        if (page < 0 || page >= a.num_pages) {
            atomicOr(a.status, kStatusBounds);
            return nullptr;
        }
        return (v ? a.v_pool : a.k_pool) +
               ((size_t)page * a.page_rows + (r % a.page_rows)) * rowstride;
    }
    bf16* base = v ? (a.v_cache ? a.v_cache[b] : a.v_single)
                   : (a.k_cache ? a.k_cache[b] : a.k_single);
    return base + (size_t)r * rowstride;
}

// MAX_THREADS selects the register budget: (heads + 1) warps must fit in it.
template <int MAX_THREADS, bool PAGED>
__global__ void __launch_bounds__(MAX_THREADS, 1) decode_kernel(DecodeArgs a, int rows_per_stage) {
    // A GEMM launched after this kernel with programmatic dependent launch (the output
    // projection) may start streaming its weights now; it waits for this grid to complete
    // before it reads anything this kernel writes.
    asm volatile("griddepcontrol.launch_dependents;");
    extern __shared__ uint8_t smem_raw[];
    uint8_t* smem = reinterpret_cast<uint8_t*>(
        (reinterpret_cast<uintptr_t>(smem_raw) + 127) & ~static_cast<uintptr_t>(127));
    const int H = a.heads;
    const size_t rowstride = (size_t)H * kHeadDim;  // elements
    const uint32_t rowbytes = (uint32_t)rowstride * 2;
    const int R = rows_per_stage;
    const uint32_t stage_bytes = 2u * R * rowbytes;  // K rows then V rows
    DecTail* tail = reinterpret_cast<DecTail*>(smem + kStages * stage_bytes);
    volatile int* abort_flag = &tail->abort;
    const int warp = threadIdx.x >> 5;
    const int lane = threadIdx.x & 31;

    if (threadIdx.x == 0) {
        for (int s = 0; s < kStages; ++s) {
            mbar_init(&tail->full[s], 1);
            mbar_init(&tail->empty[s], (uint32_t)H);
        }
        tail->abort = 0;
        fence_mbar_init();
    }
    __syncthreads();

    const int total_items = a.max_splits * a.batch;  // split-major virtual items

    if (warp == H) {
        // -------------------------------------------------------------- producer
        if (lane == 0) {
            unsigned n = 0;  // stages armed by this CTA
            bool ok = true;
            // Slot of stage n; waits until the consumers released its previous use.
            auto acquire_slot = [&](int& s) -> bool {
                s = (int)(n % kStages);
                const unsigned use = n / kStages;
                return use == 0 ||
                       mbar_wait(&tail->empty[s], (use - 1) & 1, abort_flag, a.status, 0x21);
            };
            // The first item is the CTA's own index; only when there are more items than CTAs
            // do CTAs take further items from the queue (and then all of them reset it below).
            const bool queue = total_items > (int)gridDim.x;
            for (int first_item = 1;; first_item = 0) {
                int i;
                if (first_item) {
                    i = (int)blockIdx.x;
                } else {
                    if (!queue) break;
                    i = (int)gridDim.x + (int)atomicAdd(a.counters, 1u);
                }
                if (i >= total_items) break;
                const int split = i / a.batch;
                const int b = i - split * a.batch;
                const int Lraw = raw_len(a, b);
                const int L = min(Lraw, a.max_kv_len);
                const int n_splits = L > 0 ? (L + a.split_len - 1) / a.split_len : 1;
                if (split >= n_splits) continue;
                if (split == 0 && Lraw > a.max_kv_len) atomicOr(a.status, kStatusDecodeBound);
                const int ks = split * a.split_len;
                const int ke = max(0, min(L, ks + a.split_len));
                const bool owns_new = a.k_new != nullptr && L > 0 && ke == L;
                const int ke_s = owns_new ? ke - 1 : ke;  // the new key comes from registers
                // Stages of up to R rows; with a paged cache a stage never crosses a page.
                for (int r0 = ks, first = 1, nr = 0; first || r0 < ke_s; r0 += nr, first = 0) {
                    nr = max(0, min(R, ke_s - r0));
                    if (PAGED) nr = min(nr, a.page_rows - r0 % a.page_rows);
                    const bf16* krow = nr > 0 ? kv_row<PAGED>(a, false, b, r0) : nullptr;
                    const bf16* vrow = nr > 0 ? kv_row<PAGED>(a, true, b, r0) : nullptr;
                    int s;
                    if (!(ok = acquire_slot(s))) break;
                    StageHdr& hd = tail->hdr[s];
                    hd.b = b;
                    hd.first = r0;
                    hd.nrows = nr;
                    hd.item_first = first;
                    hd.item_last = (r0 + nr >= ke_s) ? 1 : 0;
                    hd.split = split;
                    hd.n_splits = n_splits;
                    hd.L = L;
                    uint8_t* dst = smem + (size_t)s * stage_bytes;
                    if (nr > 0 && krow && vrow) {
                        mbar_arrive_expect_tx(&tail->full[s], 2u * nr * rowbytes);
                        bulk_g2s(dst, krow, nr * rowbytes, &tail->full[s]);
                        bulk_g2s(dst + (size_t)R * rowbytes, vrow, nr * rowbytes, &tail->full[s]);
                    } else {
                        hd.nrows = 0;  // nothing copied (no rows, or a bad page id)
                        mbar_arrive(&tail->full[s]);
                    }
                    ++n;
                }
                if (!ok) break;
            }
            // Tell the consumers there is no more work (one more stage, header b = -1).
            int s;
            if (ok && (ok = acquire_slot(s))) {
                tail->hdr[s].b = -1;
                mbar_arrive(&tail->full[s]);
                ++n;
            }
            // Leave the queue ready for the next launch once every CTA has stopped fetching.
            if (queue) {
                __threadfence();
                if (atomicAdd(a.counters + 1, 1u) == gridDim.x - 1) {
                    a.counters[0] = 0u;
                    a.counters[1] = 0u;
                }
            }
            // Do not leave with copies still landing: the data stages armed last are
            // released by the consumers before they exit (the terminator is not released).
            const unsigned data_stages = ok ? n - 1 : n;
            for (unsigned x = 0; x < (unsigned)kStages && x < data_stages; ++x) {
                const unsigned m_ = data_stages - 1 - x;
                mbar_wait(&tail->empty[m_ % kStages], (m_ / kStages) & 1, abort_flag, a.status, 0x22);
            }
        }
        __syncwarp();
    } else if (warp < H) {
        // -------------------------------------------------------------- consumers (head h)
        const int h = warp;
        const int half = lane >> 4;
        const int sub = lane & 15;
        const unsigned hmask = half ? 0xFFFF0000u : 0x0000FFFFu;
        const uint32_t head_off_b = (uint32_t)(h * kHeadDim + 8 * sub) * 2;  // bytes in a row
        float qf[8], acc[8], m = kNegInf, l = 0.f;
#pragma unroll
        for (int e = 0; e < 8; ++e) qf[e] = acc[e] = 0.f;
        // The query of sequence qf_b, scaled and (fused form) after RoPE + QK-norm.  It only
        // depends on the sequence, so it is kept across that sequence's items, and the CTA's
        // first item (its own index) is known up front: that query is prepared while the
        // producer's first copies are in flight.
        int qf_b = -1;
        auto load_query = [&](int b, int L) {
            const size_t qoff = (size_t)b * rowstride + (size_t)h * kHeadDim + 8 * sub;
            const uint4 qr = *reinterpret_cast<const uint4*>(a.q + qoff);
            if (a.q_raw) {
                float y[8];
                rope_norm_row(a.rope_cs, qr, sub, hmask, max(L - 1, 0), true, y);
                bf16x8_to_f32(f32_to_bf16x8(y), qf);  // bf16 like the unfused path
            } else {
                bf16x8_to_f32(qr, qf);
            }
#pragma unroll
            for (int e = 0; e < 8; ++e) qf[e] *= a.scale_log2;
            qf_b = b;
        };
        if ((int)blockIdx.x < total_items) {
            const int b0 = (int)blockIdx.x % a.batch;
            load_query(b0, min(raw_len(a, b0), a.max_kv_len));
        }
        // The new token's key (after RoPE + QK-norm) and value, prepared at the start of the
        // item that ends at it, and used after the item's cached rows.
        uint4 new_k = make_uint4(0u, 0u, 0u, 0u), new_v = new_k;
        unsigned n = 0;
        for (;;) {
            const int s = (int)(n % kStages);
            if (!__all_sync(0xFFFFFFFFu, mbar_wait(&tail->full[s], (n / kStages) & 1, abort_flag,
                                                   a.status, 0x23)))
                break;
            const StageHdr hd = tail->hdr[s];
            if (hd.b < 0) break;
            const int b = hd.b;
            const size_t qoff = (size_t)b * rowstride + (size_t)h * kHeadDim + 8 * sub;
            if (hd.item_first) {
                m = kNegInf;
                l = 0.f;
#pragma unroll
                for (int e = 0; e < 8; ++e) acc[e] = 0.f;
                if (b != qf_b) load_query(b, hd.L);
                const int ke0 = min(hd.L, hd.split * a.split_len + a.split_len);
                if (a.k_new != nullptr && hd.L > 0 && ke0 == hd.L) {
                    const uint4 kr = *reinterpret_cast<const uint4*>(a.k_new + qoff);
                    new_v = *reinterpret_cast<const uint4*>(a.v_new + qoff);
                    float y[8];
                    rope_norm_row(a.rope_cs, kr, sub, hmask, hd.L - 1, true, y);
                    new_k = f32_to_bf16x8(y);
                }
            }
            // Rows of this stage: half-warp `half` takes rows half, half + 2, ...
            const uint8_t* sk = smem + (size_t)s * stage_bytes + head_off_b;
            const uint8_t* sv = sk + (size_t)R * rowbytes;
            // Each half-warp takes kRH rows per step (rows half, half + 2, ...), so that a step's
            // dot products, shuffle reductions and exponentials are kRH independent chains and
            // one online-softmax update covers 2 * kRH rows.  Four rows under the 576-thread
            // register budget, two under the 1024-thread one.
            constexpr int kRH = MAX_THREADS <= 576 ? 4 : 2;
            for (int r0 = 0; r0 < hd.nrows; r0 += 2 * kRH) {
                uint4 kr[kRH], vr[kRH];
                bool valid[kRH];
#pragma unroll
                for (int i = 0; i < kRH; ++i) {
                    const int r = r0 + 2 * i + half;
                    valid[i] = r < hd.nrows;
                    const int rr = valid[i] ? r : 0;
                    kr[i] = *reinterpret_cast<const uint4*>(sk + (size_t)rr * rowbytes);
                    vr[i] = *reinterpret_cast<const uint4*>(sv + (size_t)rr * rowbytes);
                }
                float sc[kRH];
#pragma unroll
                for (int i = 0; i < kRH; ++i) sc[i] = dot8(qf, kr[i]);
#pragma unroll
                for (int i = 0; i < kRH; ++i) {
                    sc[i] += __shfl_xor_sync(0xFFFFFFFFu, sc[i], 8);
                    sc[i] += __shfl_xor_sync(0xFFFFFFFFu, sc[i], 4);
                    sc[i] += __shfl_xor_sync(0xFFFFFFFFu, sc[i], 2);
                    sc[i] += __shfl_xor_sync(0xFFFFFFFFu, sc[i], 1);
                    if (!valid[i]) sc[i] = kNegInf;
                }
                float bm = sc[0];
#pragma unroll
                for (int i = 1; i < kRH; ++i) bm = fmaxf(bm, sc[i]);
                const float m_new = fmaxf(m, bm);
                const float mu = (m_new == kNegInf) ? 0.f : m_new;
                const float alpha = fast_exp2(m - mu);
                float pr[kRH];
#pragma unroll
                for (int i = 0; i < kRH; ++i) pr[i] = fast_exp2(sc[i] - mu);
                float psum = pr[0] + pr[1];
                if (kRH == 4) psum += pr[2] + pr[3];
                l = __fmaf_rn(l, alpha, psum);
#pragma unroll
                for (int e = 0; e < 8; ++e) acc[e] *= alpha;
#pragma unroll
                for (int i = 0; i < kRH; ++i) {
                    float v[8];
                    bf16x8_to_f32(vr[i], v);
#pragma unroll
                    for (int e = 0; e < 8; ++e) acc[e] = __fmaf_rn(pr[i], v[e], acc[e]);
                }
                m = m_new;
            }
            __syncwarp();
            if (lane == 0) mbar_arrive(&tail->empty[s]);
            ++n;
            if (!hd.item_last) continue;

            // ---- end of item
            const int L = hd.L;
            bf16* out_row = a.out + (size_t)b * rowstride + (size_t)h * kHeadDim;
            if (L <= 0) {
                // No visible key: the reference's 0/0 yields NaN (flash_attention.cu:155).
                if (half == 0)
                    *reinterpret_cast<uint4*>(out_row + 8 * sub) =
                        make_uint4(0x7FC07FC0u, 0x7FC07FC0u, 0x7FC07FC0u, 0x7FC07FC0u);
                continue;
            }
            const int ks = hd.split * a.split_len;
            const int ke = min(L, ks + a.split_len);
            if (a.k_new != nullptr && ke == L) {
                // New token (position L-1): RoPE + QK-norm of its key, append K and V to the
                // cache, add its contribution (lanes of half 0 only).
                const int pos = L - 1;
                const uint4 kn = new_k;  // prepared at the start of this item
                const uint4 vr = new_v;
                if (half == 0) {
                    bf16* kd = kv_row<PAGED>(a, false, b, pos);
                    bf16* vd = kv_row<PAGED>(a, true, b, pos);
                    const size_t hoff = (size_t)h * kHeadDim + 8 * sub;
                    if (kd && vd) {
                        *reinterpret_cast<uint4*>(kd + hoff) = kn;
                        *reinterpret_cast<uint4*>(vd + hoff) = vr;
                    }
                }
                float sc = dot8(qf, kn);
                sc += __shfl_xor_sync(0xFFFFFFFFu, sc, 8);
                sc += __shfl_xor_sync(0xFFFFFFFFu, sc, 4);
                sc += __shfl_xor_sync(0xFFFFFFFFu, sc, 2);
                sc += __shfl_xor_sync(0xFFFFFFFFu, sc, 1);
                if (half == 0) {
                    const float m_new = fmaxf(m, sc);
                    const float alpha = fast_exp2(m - m_new);
                    const float pr = fast_exp2(sc - m_new);
                    l = __fmaf_rn(l, alpha, pr);
                    float v[8];
                    bf16x8_to_f32(vr, v);
#pragma unroll
                    for (int e = 0; e < 8; ++e) acc[e] = __fmaf_rn(pr, v[e], acc[e] * alpha);
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
            if (hd.n_splits == 1) {
                if (half == 0) {
                    const float inv = 1.0f / l;
                    float o[8];
#pragma unroll
                    for (int e = 0; e < 8; ++e) o[e] = acc[e] * inv;
                    *reinterpret_cast<uint4*>(out_row + 8 * sub) = f32_to_bf16x8(o);
                }
                continue;
            }
            // Partial result of this split, then the per-(sequence, head) ticket.
            const size_t pidx = ((size_t)b * a.max_splits + hd.split) * H + h;
            if (half == 0) {
                float4* po = reinterpret_cast<float4*>(a.part_o + pidx * kHeadDim + 8 * sub);
                __stcg(po, make_float4(acc[0], acc[1], acc[2], acc[3]));
                __stcg(po + 1, make_float4(acc[4], acc[5], acc[6], acc[7]));
                if (sub == 0) __stcg(a.part_ml + pidx, make_float2(m, l));
            }
            __threadfence();
            __syncwarp();
            unsigned ticket = 0;
            unsigned* ctr = a.counters + kQueueWords + (size_t)b * H + h;
            if (lane == 0) ticket = atomicAdd(ctr, 1u);
            ticket = __shfl_sync(0xFFFFFFFFu, ticket, 0);
            if (ticket != (unsigned)(hd.n_splits - 1)) continue;
            // Last split of (b, h): combine.  Lane owns dims [4*lane, 4*lane+4).
            __threadfence();
            if (lane == 0) *ctr = 0u;  // ready for the next launch
            const size_t base = (size_t)b * a.max_splits * H + h;
            const int ns = hd.n_splits;
            // Lane j holds (max, sum) of splits j, j + 32, ...; the first group's stays in a
            // register for the second pass.
            float2 ml0 = make_float2(kNegInf, 0.f);
            if (lane < ns) ml0 = __ldcg(a.part_ml + base + (size_t)lane * H);
            float M = ml0.x;
            for (int sp = lane + 32; sp < ns; sp += 32)
                M = fmaxf(M, __ldcg(a.part_ml + base + (size_t)sp * H).x);
#pragma unroll
            for (int o = 16; o > 0; o >>= 1) M = fmaxf(M, __shfl_xor_sync(0xFFFFFFFFu, M, o));
            const float mu = (M == kNegInf) ? 0.f : M;
            float den = 0.f, o4[4] = {0.f, 0.f, 0.f, 0.f};
            // kDepth partial outputs per round trip to L2 (fewer under the 1024-thread register
            // budget); each split's weight comes from the lane that holds it.
            constexpr int kDepth = MAX_THREADS <= 576 ? 8 : 4;
            for (int g0 = 0; g0 < ns; g0 += 32) {
                float2 ml = ml0;
                if (g0 > 0)
                    ml = g0 + lane < ns ? __ldcg(a.part_ml + base + (size_t)(g0 + lane) * H)
                                        : make_float2(kNegInf, 0.f);
                const float w = fast_exp2(ml.x - mu);  // 0 for a missing split (-inf)
                float lw = ml.y * w;
#pragma unroll
                for (int o = 16; o > 0; o >>= 1) lw += __shfl_xor_sync(0xFFFFFFFFu, lw, o);
                den += lw;
                const int cnt = min(32, ns - g0);
                for (int sp0 = 0; sp0 < cnt; sp0 += kDepth) {
                    float4 v[kDepth];
#pragma unroll
                    for (int i = 0; i < kDepth; ++i) {
                        const int sp = sp0 + i;
                        v[i] = sp < cnt ? __ldcg(reinterpret_cast<const float4*>(
                                              a.part_o + (base + (size_t)(g0 + sp) * H) * kHeadDim) + lane)
                                        : make_float4(0.f, 0.f, 0.f, 0.f);
                    }
#pragma unroll
                    for (int i = 0; i < kDepth; ++i) {
                        const float wi = __shfl_sync(0xFFFFFFFFu, w, (sp0 + i) & 31);
                        o4[0] = __fmaf_rn(v[i].x, wi, o4[0]);
                        o4[1] = __fmaf_rn(v[i].y, wi, o4[1]);
                        o4[2] = __fmaf_rn(v[i].z, wi, o4[2]);
                        o4[3] = __fmaf_rn(v[i].w, wi, o4[3]);
                    }
                }
            }
            const float inv = 1.0f / den;
            uint2 r;
            r.x = pack_bf16x2(o4[0] * inv, o4[1] * inv);
            r.y = pack_bf16x2(o4[2] * inv, o4[3] * inv);
            *reinterpret_cast<uint2*>(out_row + 4 * lane) = r;
        }
    }
    __syncthreads();
}

// Per-head layout for small batches: one CTA of four warps per (split, head, sequence), at most
// kDecodeHeadSplit = 64 keys per split.  Every warp issues the copies of its 16 rows at once
// (a half-warp copies one row's 256 bytes of this head, 16 bytes per lane, by cp.async into
// shared memory, each lane into its own slots), so a split costs one DRAM round trip and there
// is no queue or staging ring; with a few sequences this puts work on every SM within one
// launch latency.  Staging the rows in shared memory rather than registers keeps the kernel
// at 80 registers, six CTAs per SM: 50 % more bytes in flight than four (measured on the cfg5
// decode step: 1.395 ms against 1.515 with register-held rows).  Same per-row arithmetic as decode_kernel
// (fused RoPE + QK-norm of q and of the new key, online softmax in log2 units, four rows per
// half-warp step); the four warps merge through shared memory, and, with several splits, the
// last split of each (sequence, head) to finish combines them (per-head ticket, self-resetting).
//
// CLUSTER: the splits of one (sequence, head) form one thread-block cluster (grid x = cluster x
// = the call's split count, at most 16).  Each CTA leaves its merged partial (max, sum, 128
// unnormalised outputs) in its own shared memory; after a cluster barrier, CTA 0 of the cluster
// combines them over distributed shared memory, in split order, and writes the output, and a
// second barrier keeps every CTA resident until it has read them.  No global partials, no
// tickets, no workspace.  CTAs past a sequence's split count (a shorter sequence of the batch)
// only take part in the two barriers.
template <bool PAGED, bool CLUSTER>
__global__ void __launch_bounds__(128, 6) decode_head_kernel(DecodeArgs a) {
    asm volatile("griddepcontrol.launch_dependents;");  // as in decode_kernel
    __shared__ float sm_o[4][kHeadDim];
    __shared__ float2 sm_ml[4];
    // Cache rows in flight: each thread's 8 K and 8 V slices land here by cp.async (16 bytes
    // each, slot [k/v][i][thread]); only the thread that copied a slot reads it.
    __shared__ __align__(16) uint4 sm_kv[2][8][128];
    __shared__ __align__(16) float cl_o[kHeadDim];  // CLUSTER: this split's partial
    __shared__ float2 cl_ml;
    const int split = blockIdx.x, h = blockIdx.y, b = blockIdx.z;
    const int warp = threadIdx.x >> 5;
    const int lane = threadIdx.x & 31;
    const int half = lane >> 4;
    const int sub = lane & 15;
    const unsigned hmask = half ? 0xFFFF0000u : 0x0000FFFFu;
    const int H = a.heads;
    const size_t rowstride = (size_t)H * kHeadDim;
    const size_t qoff = (size_t)b * rowstride + (size_t)h * kHeadDim + 8 * sub;
    // The sequence's length and this warp's cache base (or page id) first, loaded together,
    // then this split's cache rows: none of them is written by the kernel that precedes an
    // overlapped launch (a.overlap), so they are read before griddepcontrol.wait; the query
    // and the new key and value come after it.
    const int T = a.split_len;
    // This warp's rows start at w0 (half-warp `half` takes w0 + half, w0 + half + 2, ...); the
    // 16 rows are consecutive in the cache (a paged cache's pages hold a multiple of 16 rows,
    // and w0 is a multiple of 16), so one base or page id per warp.
    const int w0 = split * T + 16 * warp;
    const int Lraw = raw_len(a, b);
    // Without an overlapped launch the query has no producer still running: load it with the
    // rest, so that its RoPE + QK-norm overlaps the cache loads.
    uint4 qr = make_uint4(0u, 0u, 0u, 0u);
    if (!a.overlap) qr = *reinterpret_cast<const uint4*>(a.q + qoff);
    const bf16* kbase = nullptr;
    const bf16* vbase = nullptr;
    int page = 0;
    if (PAGED) {
        const int pidx = w0 / a.page_rows;
        page = pidx < a.pages_per_seq ? a.page_table[(size_t)b * a.pages_per_seq + pidx] : -1;
    } else {
        kbase = a.k_cache ? a.k_cache[b] : a.k_single;
        vbase = a.v_cache ? a.v_cache[b] : a.v_single;
    }
    const int L = min(Lraw, a.max_kv_len);
    const int n_splits = L > 0 ? (L + T - 1) / T : 1;
    if (split == 0 && h == 0 && threadIdx.x == 0 && Lraw > a.max_kv_len)
        atomicOr(a.status, kStatusDecodeBound);
    bf16* out_row = a.out + (size_t)b * rowstride + (size_t)h * kHeadDim;
    if (CLUSTER) {
        // Uniform across the CTA: a split past the sequence's count, or no visible key (the
        // reference's 0/0 yields NaN, flash_attention.cu:155), contributes nothing but its
        // part in the cluster barriers.
        if (split >= n_splits || L <= 0) {
            griddep_wait();
            if (L <= 0 && split == 0 && warp == 0 && half == 0)
                *reinterpret_cast<uint4*>(out_row + 8 * sub) =
                    make_uint4(0x7FC07FC0u, 0x7FC07FC0u, 0x7FC07FC0u, 0x7FC07FC0u);
            cooperative_groups::this_cluster().sync();
            cooperative_groups::this_cluster().sync();
            return;
        }
    } else {
        if (split >= n_splits) return;  // uniform across the CTA
        if (L <= 0) {
            griddep_wait();
            // No visible key: the reference's 0/0 yields NaN (flash_attention.cu:155).
            if (warp == 0 && half == 0)
                *reinterpret_cast<uint4*>(out_row + 8 * sub) =
                    make_uint4(0x7FC07FC0u, 0x7FC07FC0u, 0x7FC07FC0u, 0x7FC07FC0u);
            return;
        }
    }
    const int ks = split * T;
    const int ke = min(L, ks + T);
    const bool owns_new = a.k_new != nullptr && ke == L;
    const int ke_s = owns_new ? ke - 1 : ke;  // the new key comes from registers

    const int w1 = min(ke_s, w0 + 16);  // this warp's rows are [w0, w1)
    const bf16* kb = nullptr;
    const bf16* vb = nullptr;
    if (w0 < w1) {
        if (!PAGED) {
            kb = kbase + (size_t)w0 * rowstride;
            vb = vbase + (size_t)w0 * rowstride;
        } else if (page >= 0 && page < a.num_pages) {
            const size_t prow = (size_t)page * a.page_rows + (w0 % a.page_rows);
            kb = a.k_pool + prow * rowstride;
            vb = a.v_pool + prow * rowstride;
        } else {
            atomicOr(a.status, kStatusBounds);
        }
    }
#pragma unroll
    for (int i = 0; i < 8; ++i) {
        const int r = w0 + 2 * i + half;
        if (r < w1 && kb && vb) {
            const size_t off = (size_t)(r - w0) * rowstride + (size_t)h * kHeadDim + 8 * sub;
            asm volatile("cp.async.cg.shared.global [%0], [%1], 16;" ::"r"(smem_u32(&sm_kv[0][i][threadIdx.x])),
                         "l"(kb + off) : "memory");
            asm volatile("cp.async.cg.shared.global [%0], [%1], 16;" ::"r"(smem_u32(&sm_kv[1][i][threadIdx.x])),
                         "l"(vb + off) : "memory");
        } else {
            sm_kv[0][i][threadIdx.x] = sm_kv[1][i][threadIdx.x] = make_uint4(0u, 0u, 0u, 0u);
        }
    }
    asm volatile("cp.async.commit_group;" ::: "memory");
    griddep_wait();  // no-op unless launched as a programmatic dependent launch
    if (a.overlap) qr = *reinterpret_cast<const uint4*>(a.q + qoff);
    float qf[8];
    {
        if (a.q_raw) {
            float y[8];
            rope_norm_row(a.rope_cs, qr, sub, hmask, L - 1, true, y);
            bf16x8_to_f32(f32_to_bf16x8(y), qf);  // bf16 like the unfused path
        } else {
            bf16x8_to_f32(qr, qf);
        }
#pragma unroll
        for (int e = 0; e < 8; ++e) qf[e] *= a.scale_log2;
    }
    // New token (position L-1), warp 0 of the CTA that owns it: RoPE + QK-norm of its key,
    // append K and V to the cache (lanes of half 0), add its contribution below.
    uint4 new_k = make_uint4(0u, 0u, 0u, 0u), new_v = new_k;
    if (owns_new && warp == 0) {
        const uint4 kraw = *reinterpret_cast<const uint4*>(a.k_new + qoff);
        new_v = *reinterpret_cast<const uint4*>(a.v_new + qoff);
        float y[8];
        rope_norm_row(a.rope_cs, kraw, sub, hmask, L - 1, true, y);
        new_k = f32_to_bf16x8(y);
        if (half == 0) {
            bf16* kd = kv_row<PAGED>(a, false, b, L - 1);
            bf16* vd = kv_row<PAGED>(a, true, b, L - 1);
            const size_t hoff = (size_t)h * kHeadDim + 8 * sub;
            if (kd && vd) {
                *reinterpret_cast<uint4*>(kd + hoff) = new_k;
                *reinterpret_cast<uint4*>(vd + hoff) = new_v;
            }
        }
    }

    float m = kNegInf, l = 0.f, acc[8];
#pragma unroll
    for (int e = 0; e < 8; ++e) acc[e] = 0.f;
    asm volatile("cp.async.wait_all;" ::: "memory");
#pragma unroll
    for (int s4 = 0; s4 < 2; ++s4) {
        float sc[4];
#pragma unroll
        for (int i = 0; i < 4; ++i) {
            const int idx = 4 * s4 + i;
            sc[i] = dot8(qf, sm_kv[0][idx][threadIdx.x]);
            sc[i] += __shfl_xor_sync(0xFFFFFFFFu, sc[i], 8);
            sc[i] += __shfl_xor_sync(0xFFFFFFFFu, sc[i], 4);
            sc[i] += __shfl_xor_sync(0xFFFFFFFFu, sc[i], 2);
            sc[i] += __shfl_xor_sync(0xFFFFFFFFu, sc[i], 1);
            if (!(w0 + 2 * idx + half < w1)) sc[i] = kNegInf;
        }
        const float bm = fmaxf(fmaxf(sc[0], sc[1]), fmaxf(sc[2], sc[3]));
        const float m_new = fmaxf(m, bm);
        const float mu = (m_new == kNegInf) ? 0.f : m_new;
        const float alpha = fast_exp2(m - mu);
        float pr[4];
#pragma unroll
        for (int i = 0; i < 4; ++i) pr[i] = fast_exp2(sc[i] - mu);
        l = __fmaf_rn(l, alpha, (pr[0] + pr[1]) + (pr[2] + pr[3]));
#pragma unroll
        for (int e = 0; e < 8; ++e) acc[e] *= alpha;
#pragma unroll
        for (int i = 0; i < 4; ++i) {
            float v[8];
            bf16x8_to_f32(sm_kv[1][4 * s4 + i][threadIdx.x], v);
#pragma unroll
            for (int e = 0; e < 8; ++e) acc[e] = __fmaf_rn(pr[i], v[e], acc[e]);
        }
        m = m_new;
    }
    if (owns_new && warp == 0) {
        float sc = dot8(qf, new_k);
        sc += __shfl_xor_sync(0xFFFFFFFFu, sc, 8);
        sc += __shfl_xor_sync(0xFFFFFFFFu, sc, 4);
        sc += __shfl_xor_sync(0xFFFFFFFFu, sc, 2);
        sc += __shfl_xor_sync(0xFFFFFFFFu, sc, 1);
        if (half == 0) {
            const float m_new = fmaxf(m, sc);
            const float alpha = fast_exp2(m - m_new);
            const float pr = fast_exp2(sc - m_new);
            l = __fmaf_rn(l, alpha, pr);
            float v[8];
            bf16x8_to_f32(new_v, v);
#pragma unroll
            for (int e = 0; e < 8; ++e) acc[e] = __fmaf_rn(pr, v[e], acc[e] * alpha);
            m = m_new;
        }
    }
    // Merge the two half-warps (same dims, disjoint keys), then the four warps.
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
    if (half == 0) {
#pragma unroll
        for (int e = 0; e < 8; ++e) sm_o[warp][8 * sub + e] = acc[e];
    }
    if (lane == 0) sm_ml[warp] = make_float2(m, l);
    __syncthreads();
    if (CLUSTER) {
        if (warp == 0) {
            float M = kNegInf;
#pragma unroll
            for (int w = 0; w < 4; ++w) M = fmaxf(M, sm_ml[w].x);
            const float mu = (M == kNegInf) ? 0.f : M;
            float den = 0.f, o4[4] = {0.f, 0.f, 0.f, 0.f};
#pragma unroll
            for (int w = 0; w < 4; ++w) {
                const float wt = fast_exp2(sm_ml[w].x - mu);
                den = __fmaf_rn(sm_ml[w].y, wt, den);
#pragma unroll
                for (int i = 0; i < 4; ++i) o4[i] = __fmaf_rn(sm_o[w][4 * lane + i], wt, o4[i]);
            }
            *reinterpret_cast<float4*>(&cl_o[4 * lane]) = make_float4(o4[0], o4[1], o4[2], o4[3]);
            if (lane == 0) cl_ml = make_float2(M, den);
        }
        cooperative_groups::cluster_group cluster = cooperative_groups::this_cluster();
        cluster.sync();  // release / acquire: every split's partial is visible
        if (split == 0 && warp == 0) {
            // The same arithmetic, in the same split order, as the global combine of up to 8
            // splits below.
            float2 ml[16];
            float4 v[16];
#pragma unroll
            for (int i = 0; i < 16; ++i) {
                const bool okr = i < n_splits;
                ml[i] = okr ? *cluster.map_shared_rank(&cl_ml, i) : make_float2(kNegInf, 0.f);
                v[i] = okr ? *reinterpret_cast<const float4*>(cluster.map_shared_rank(&cl_o[4 * lane], i))
                           : make_float4(0.f, 0.f, 0.f, 0.f);
            }
            float Mf = kNegInf;
#pragma unroll
            for (int i = 0; i < 16; ++i) Mf = fmaxf(Mf, ml[i].x);
            const float muf = (Mf == kNegInf) ? 0.f : Mf;
            float df = 0.f, of[4] = {0.f, 0.f, 0.f, 0.f};
#pragma unroll
            for (int i = 0; i < 16; ++i) {
                const float w = fast_exp2(ml[i].x - muf);
                df = __fmaf_rn(ml[i].y, w, df);
                of[0] = __fmaf_rn(v[i].x, w, of[0]);
                of[1] = __fmaf_rn(v[i].y, w, of[1]);
                of[2] = __fmaf_rn(v[i].z, w, of[2]);
                of[3] = __fmaf_rn(v[i].w, w, of[3]);
            }
            const float invf = 1.0f / df;
            uint2 rf;
            rf.x = pack_bf16x2(of[0] * invf, of[1] * invf);
            rf.y = pack_bf16x2(of[2] * invf, of[3] * invf);
            *reinterpret_cast<uint2*>(out_row + 4 * lane) = rf;
        }
        cluster.sync();  // no CTA leaves while CTA 0 still reads its shared memory
        return;
    }
    // Warp 0 merges the four warps into this split's (max, sum, output) and, with several
    // splits, stores it and takes the ticket of its (sequence, head).  The other warps wait
    // for the outcome: above 8 splits the last split's combine is shared by all four warps.
    __shared__ int sm_last;
    unsigned* ctr = a.counters + kQueueWords + (size_t)b * H + h;
    if (warp == 0) {
        // Warp 0: lane owns dims [4*lane, 4*lane+4).
        float M = kNegInf;
#pragma unroll
        for (int w = 0; w < 4; ++w) M = fmaxf(M, sm_ml[w].x);
        const float mu = (M == kNegInf) ? 0.f : M;
        float den = 0.f, o4[4] = {0.f, 0.f, 0.f, 0.f};
#pragma unroll
        for (int w = 0; w < 4; ++w) {
            const float wt = fast_exp2(sm_ml[w].x - mu);
            den = __fmaf_rn(sm_ml[w].y, wt, den);
#pragma unroll
            for (int i = 0; i < 4; ++i) o4[i] = __fmaf_rn(sm_o[w][4 * lane + i], wt, o4[i]);
        }
        if (n_splits == 1) {
            const float inv = 1.0f / den;
            uint2 r;
            r.x = pack_bf16x2(o4[0] * inv, o4[1] * inv);
            r.y = pack_bf16x2(o4[2] * inv, o4[3] * inv);
            *reinterpret_cast<uint2*>(out_row + 4 * lane) = r;
        } else {
            // Partial result of this split (max, sum, unnormalised output), then the ticket.
            const size_t pidx = ((size_t)b * a.max_splits + split) * H + h;
            __stcg(reinterpret_cast<float4*>(a.part_o + pidx * kHeadDim) + lane,
                   make_float4(o4[0], o4[1], o4[2], o4[3]));
            if (lane == 0) __stcg(a.part_ml + pidx, make_float2(M, den));
            __threadfence();
            __syncwarp();
            unsigned ticket = 0;
            if (lane == 0) ticket = atomicAdd(ctr, 1u);
            ticket = __shfl_sync(0xFFFFFFFFu, ticket, 0);
            if (lane == 0) sm_last = ticket == (unsigned)(n_splits - 1) ? 1 : 0;
        }
    }
    if (n_splits == 1) return;  // uniform across the CTA
    __syncthreads();            // sm_last written; warp 0 has read sm_o / sm_ml
    if (!sm_last) return;       // uniform: only the last split of (b, h) combines
    __threadfence();
    if (threadIdx.x == 0) *ctr = 0u;  // ready for the next launch
    const size_t base = (size_t)b * a.max_splits * H + h;
    if (n_splits <= 8) {
        if (warp != 0) return;
        // Up to 8 splits (up to 512 keys): every partial is loaded in one round trip.
        float4 v[8];
        float2 ml[8];
#pragma unroll
        for (int i = 0; i < 8; ++i) {
            const bool ok = i < n_splits;
            v[i] = ok ? __ldcg(reinterpret_cast<const float4*>(
                           a.part_o + (base + (size_t)i * H) * kHeadDim) + lane)
                      : make_float4(0.f, 0.f, 0.f, 0.f);
            ml[i] = ok ? __ldcg(a.part_ml + base + (size_t)i * H) : make_float2(kNegInf, 0.f);
        }
        float Mf = kNegInf;
#pragma unroll
        for (int i = 0; i < 8; ++i) Mf = fmaxf(Mf, ml[i].x);
        const float muf = (Mf == kNegInf) ? 0.f : Mf;
        float df = 0.f, of[4] = {0.f, 0.f, 0.f, 0.f};
#pragma unroll
        for (int i = 0; i < 8; ++i) {
            const float w = fast_exp2(ml[i].x - muf);
            df = __fmaf_rn(ml[i].y, w, df);
            of[0] = __fmaf_rn(v[i].x, w, of[0]);
            of[1] = __fmaf_rn(v[i].y, w, of[1]);
            of[2] = __fmaf_rn(v[i].z, w, of[2]);
            of[3] = __fmaf_rn(v[i].w, w, of[3]);
        }
        const float invf = 1.0f / df;
        uint2 rf;
        rf.x = pack_bf16x2(of[0] * invf, of[1] * invf);
        rf.y = pack_bf16x2(of[2] * invf, of[3] * invf);
        *reinterpret_cast<uint2*>(out_row + 4 * lane) = rf;
        return;
    }
    // More than 8 splits: warp w combines splits w, w + 4, w + 8, ... , four per round trip
    // (two round trips for up to 32 splits), merged online, then warp 0 merges the
    // four warps' results.  Lane owns dims [4*lane, 4*lane+4).
    {
        float Mw = kNegInf, dw = 0.f, ow[4] = {0.f, 0.f, 0.f, 0.f};
        for (int c0 = warp; c0 < n_splits; c0 += 16) {
            float4 v[4];
            float2 ml[4];
#pragma unroll
            for (int i = 0; i < 4; ++i) {
                const int sp = c0 + 4 * i;
                const bool ok = sp < n_splits;
                v[i] = ok ? __ldcg(reinterpret_cast<const float4*>(
                                a.part_o + (base + (size_t)sp * H) * kHeadDim) + lane)
                          : make_float4(0.f, 0.f, 0.f, 0.f);
                ml[i] = ok ? __ldcg(a.part_ml + base + (size_t)sp * H) : make_float2(kNegInf, 0.f);
            }
            float Mc = kNegInf;
#pragma unroll
            for (int i = 0; i < 4; ++i) Mc = fmaxf(Mc, ml[i].x);
            const float Mn = fmaxf(Mw, Mc);
            const float mun = (Mn == kNegInf) ? 0.f : Mn;
            const float sc = fast_exp2(Mw - mun);  // 0 while nothing is merged (Mw = -inf)
            dw *= sc;
#pragma unroll
            for (int k = 0; k < 4; ++k) ow[k] *= sc;
#pragma unroll
            for (int i = 0; i < 4; ++i) {
                const float w = fast_exp2(ml[i].x - mun);
                dw = __fmaf_rn(ml[i].y, w, dw);
                ow[0] = __fmaf_rn(v[i].x, w, ow[0]);
                ow[1] = __fmaf_rn(v[i].y, w, ow[1]);
                ow[2] = __fmaf_rn(v[i].z, w, ow[2]);
                ow[3] = __fmaf_rn(v[i].w, w, ow[3]);
            }
            Mw = Mn;
        }
        if (lane == 0) sm_ml[warp] = make_float2(Mw, dw);
        *reinterpret_cast<float4*>(&sm_o[warp][4 * lane]) = make_float4(ow[0], ow[1], ow[2], ow[3]);
    }
    __syncthreads();
    if (warp != 0) return;
    float Mf = kNegInf;
#pragma unroll
    for (int w = 0; w < 4; ++w) Mf = fmaxf(Mf, sm_ml[w].x);
    const float muf = (Mf == kNegInf) ? 0.f : Mf;
    float df = 0.f, of[4] = {0.f, 0.f, 0.f, 0.f};
#pragma unroll
    for (int w = 0; w < 4; ++w) {
        const float wt = fast_exp2(sm_ml[w].x - muf);
        df = __fmaf_rn(sm_ml[w].y, wt, df);
#pragma unroll
        for (int i = 0; i < 4; ++i) of[i] = __fmaf_rn(sm_o[w][4 * lane + i], wt, of[i]);
    }
    const float invf = 1.0f / df;
    uint2 rf;
    rf.x = pack_bf16x2(of[0] * invf, of[1] * invf);
    rf.y = pack_bf16x2(of[2] * invf, of[3] * invf);
    *reinterpret_cast<uint2*>(out_row + 4 * lane) = rf;
}

}  // namespace

// Rows per ring stage for a head count: three stages of K and V rows within ~216 KB.
int decode_rows_per_stage(int heads) {
    const int rowbytes = heads * kHeadDim * 2;
    int r = (216 * 1024) / (kStages * 2 * rowbytes);
    r = std::min(r, 16) & ~1;
    return std::max(r, 2);
}

size_t decode_smem_bytes(int heads) {
    const size_t rowbytes = (size_t)heads * kHeadDim * 2;
    return 128 + (size_t)kStages * 2 * decode_rows_per_stage(heads) * rowbytes + sizeof(DecTail);
}

size_t decode_counter_words(int batch, int heads) {
    return kQueueWords + (size_t)batch * heads;
}

size_t decode_workspace_bytes(int batch, int max_splits, int heads) {
    const size_t n = (size_t)batch * max_splits * heads;
    size_t bytes = (decode_counter_words(batch, heads) * sizeof(unsigned) + 255) & ~(size_t)255;
    bytes = (bytes + n * sizeof(float2) + 255) & ~(size_t)255;  // part_ml
    bytes += n * kHeadDim * sizeof(float);                      // part_o
    return (bytes + 255) & ~(size_t)255;
}

cudaError_t launch_decode(const DecodeArgs& a, cudaStream_t stream) {
    if (a.batch <= 0) return cudaSuccess;
    static int sms[64] = {};
    static bool attr[64] = {};
    int dev = 0;
    cudaError_t e = cudaGetDevice(&dev);
    if (e != cudaSuccess) return e;
    if (dev < 0 || dev >= 64) return cudaErrorInvalidDevice;
    if (!sms[dev]) {
        e = cudaDeviceGetAttribute(&sms[dev], cudaDevAttrMultiProcessorCount, dev);
        if (e != cudaSuccess) return e;
    }
    if (!attr[dev]) {
        size_t most = 0;  // the opt-in must cover every head count the kernel accepts
        for (int hh = 1; hh <= 31; ++hh) most = std::max(most, decode_smem_bytes(hh));
        e = cudaSuccess;
        for (auto fn : {decode_kernel<576, false>, decode_kernel<1024, false>,
                        decode_kernel<576, true>, decode_kernel<1024, true>})
            if (e == cudaSuccess)
                e = cudaFuncSetAttribute(fn, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                         (int)most);
        if (e != cudaSuccess) return e;
        attr[dev] = true;
    }
    const bool paged = a.page_table != nullptr;
    if (a.head_layout) {
        // The splits of a (sequence, head) combine inside one thread-block cluster when there
        // are 2..16 of them (above 8 needs the non-portable cluster size), except for an
        // overlapped launch: its CTAs start beside the still-running GEMM, which a cluster,
        // placed whole inside one GPC, would hold back (measured: the engine's decode step
        // 1.69 ms with clusters against 1.50 without).
        const bool cluster = decode_head_cluster(a.max_splits, a.batch, a.overlap != 0);
        static bool cl_attr[64] = {};
        if (cluster && !cl_attr[dev]) {
            for (auto fn : {decode_head_kernel<false, true>, decode_head_kernel<true, true>}) {
                e = cudaFuncSetAttribute(fn, cudaFuncAttributeNonPortableClusterSizeAllowed, 1);
                if (e != cudaSuccess) return e;
            }
            cl_attr[dev] = true;
        }
        cudaLaunchConfig_t cfg = {};
        cfg.gridDim = dim3((unsigned)a.max_splits, (unsigned)a.heads, (unsigned)a.batch);
        cfg.blockDim = dim3(128);
        cfg.stream = stream;
        cudaLaunchAttribute at[2];
        int n = 0;
        if (a.overlap) {
            at[n].id = cudaLaunchAttributeProgrammaticStreamSerialization;
            at[n].val.programmaticStreamSerializationAllowed = 1;
            ++n;
        }
        if (cluster) {
            at[n].id = cudaLaunchAttributeClusterDimension;
            at[n].val.clusterDim.x = (unsigned)a.max_splits;
            at[n].val.clusterDim.y = 1;
            at[n].val.clusterDim.z = 1;
            ++n;
        }
        cfg.attrs = at;
        cfg.numAttrs = n;
        if (cluster)
            return paged ? cudaLaunchKernelEx(&cfg, decode_head_kernel<true, true>, a)
                         : cudaLaunchKernelEx(&cfg, decode_head_kernel<false, true>, a);
        return paged ? cudaLaunchKernelEx(&cfg, decode_head_kernel<true, false>, a)
                     : cudaLaunchKernelEx(&cfg, decode_head_kernel<false, false>, a);
    }
    const long long items = (long long)a.max_splits * a.batch;
    const unsigned grid = (unsigned)std::max<long long>(1, std::min<long long>(items, sms[dev]));
    const int threads = (a.heads + 1) * 32;  // one warp per head + the producer warp
    const size_t smem = decode_smem_bytes(a.heads);
    const int R = decode_rows_per_stage(a.heads);
    if (threads <= 576) {
        if (paged) decode_kernel<576, true><<<grid, threads, smem, stream>>>(a, R);
        else decode_kernel<576, false><<<grid, threads, smem, stream>>>(a, R);
    } else {
        if (paged) decode_kernel<1024, true><<<grid, threads, smem, stream>>>(a, R);
        else decode_kernel<1024, false><<<grid, threads, smem, stream>>>(a, R);
    }
    return cudaGetLastError();
}

}  // namespace nc

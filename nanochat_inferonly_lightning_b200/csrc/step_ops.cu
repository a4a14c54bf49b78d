// The two small passes at the ends of a decode step, so that a graph-captured step is all on this
// library:
//  * the embedding gather fused with the RMSNorm that follows it (reference
//    kernels/ops.cu:9-20 then kernels/rmsnorm.cu:9-56, called at src/model.cpp:158-162);
//  * sampling on the device, so the token never leaves it between steps: greedy (the first
//    maximum of each row, src/engine.cpp:88-95) and temperature / top-k / top-p sampling
//    (src/engine.cpp:62-131) with the uniform draw supplied by the caller.
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

// ---------------------------------------------------------------------------------------
// Sampling (src/engine.cpp:88-131) on the device, one CTA of 1024 threads per row; thread t
// owns the contiguous slice [t * ept, (t + 1) * ept) of the row, so thread order is index
// order.
// ---------------------------------------------------------------------------------------
constexpr int kSampleThreads = 1024;
constexpr int kSampleMaxK = 1024;

// bf16 bits -> 16-bit key ordered like the value (larger value, larger key); -0 counts as +0.
__device__ __forceinline__ uint32_t order_key(uint32_t h) {
    if (h == 0x8000u) h = 0u;
    return (h & 0x8000u) ? (~h & 0xFFFFu) : (h | 0x8000u);
}
__device__ __forceinline__ float key_value(uint32_t key) {
    const uint32_t h = (key & 0x8000u) ? (key & 0x7FFFu) : (~key & 0xFFFFu);
    return __uint_as_float(h << 16);
}

// Exclusive prefix sum of one int per thread over the block (1024 threads); *total gets the sum.
__device__ int block_exclusive_scan(int v, int* warp_sums, int* total) {
    const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
    int x = v;
#pragma unroll
    for (int o = 1; o < 32; o <<= 1) {
        const int y = __shfl_up_sync(0xFFFFFFFFu, x, o);
        if (lane >= o) x += y;
    }
    if (lane == 31) warp_sums[warp] = x;
    __syncthreads();
    if (warp == 0) {
        int w = warp_sums[lane];
#pragma unroll
        for (int o = 1; o < 32; o <<= 1) {
            const int y = __shfl_up_sync(0xFFFFFFFFu, w, o);
            if (lane >= o) w += y;
        }
        warp_sums[lane] = w;  // inclusive over warps
    }
    __syncthreads();
    const int base = warp > 0 ? warp_sums[warp - 1] : 0;
    *total = warp_sums[31];
    __syncthreads();  // warp_sums is reused by the next call
    return base + x - v;
}

// Exclusive prefix sum of one float per thread over the block (1024 threads); *total gets the
// sum.  Same structure as block_exclusive_scan.
__device__ float block_exclusive_scan_f(float v, float* warp_sums, float* total) {
    const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
    float x = v;
#pragma unroll
    for (int o = 1; o < 32; o <<= 1) {
        const float y = __shfl_up_sync(0xFFFFFFFFu, x, o);
        if (lane >= o) x += y;
    }
    if (lane == 31) warp_sums[warp] = x;
    __syncthreads();
    if (warp == 0) {
        float w = warp_sums[lane];
#pragma unroll
        for (int o = 1; o < 32; o <<= 1) {
            const float y = __shfl_up_sync(0xFFFFFFFFu, w, o);
            if (lane >= o) w += y;
        }
        warp_sums[lane] = w;
    }
    __syncthreads();
    const float base = warp > 0 ? warp_sums[warp - 1] : 0.f;
    *total = warp_sums[31];
    __syncthreads();
    return base + x - v;
}

struct SampleSmem {
    unsigned long long cand[kSampleMaxK];  // (key << 32) | (0xFFFFFFFF - index)
    float q[kSampleMaxK];                  // normalised probability of each candidate
    int hist[256];
    int warp_sums[32];
    float fred[32];
    int b1, above1, kstar, c_gt;
    int found;
};

// ---------------------------------------------------------------------------------------
// Top-p over the whole row (Engine::top_p_filter with top_k off, src/engine.cpp:68-84, then
// the renormalisation and the draw, :114-131), without a sort.  A probability is a monotone
// function of its bf16 logit, so the reference's descending sort orders the row by 16-bit key
// (equal keys by ascending index: the order its sort leaves unspecified; -0 counts as +0), and
// all members of one key have the same probability.  One pass counts the members of every key
// (65536 16-bit counters, 128 KB of shared memory); the mass of a key is then its count times
// its probability, in fixed point (units of 2^-62, a probability being at most 1), so every
// sum below is exact and independent of the order of the threads.  The keys' masses summed
// over 256 buckets of 256 keys locate the bucket where the running mass (from the top) first
// exceeds top_p, the masses of that bucket's keys locate the key, and the members of that key
// needed to pass top_p are counted off; the draw r is located in the kept prefix the same way,
// and a last pass over the row finds the chosen member's index.  The reference sums in fp32,
// in order: the two agree except where top_p or r lies within that summation error of an
// interval edge.
// ---------------------------------------------------------------------------------------
constexpr size_t kTopPCountBytes = 65536 * sizeof(uint16_t);
constexpr int kTopPMaxDev = 64;  // devices whose shared-memory attribute is tracked

struct TopPSmem {
    int warp_sums[32];
    float fred[32];
    int cnt1[256], cnt2[256];  // per bucket: members of the 256 keys of a high byte / of one key
    unsigned long long mass1[256], mass2[256];
    int xb;
    unsigned long long xmass;
    int found, all_equal;
};

// Fixed-point mass of one member of key `key` (units of 2^-62).
__device__ __forceinline__ unsigned long long key_mass(uint32_t key, float mx, float temperature,
                                                       float sum) {
    const float q = expf((key_value(key) - mx) / temperature) / sum;
    return (unsigned long long)(q * 0x1p62f);
}

// Warp 0: walking the 256 buckets of (cnt, mass) from 255 down, the first bucket at which the
// running mass exceeds `target`; sm.xb = that bucket (-1 if the total does not), sm.xmass = the
// mass of the buckets above it (the total when there is none).  Lane l scans buckets 255 - 8l
// down to 248 - 8l.
__device__ void bucket_crossing(TopPSmem& sm, const int* cnt, const unsigned long long* mass,
                                unsigned long long target) {
    const int lane = threadIdx.x & 31;
    unsigned long long m = 0;
#pragma unroll
    for (int i = 0; i < 8; ++i) m += mass[255 - 8 * lane - i];
    unsigned long long mi = m;  // inclusive scan over the lanes
#pragma unroll
    for (int o = 1; o < 32; o <<= 1) {
        const unsigned long long y = __shfl_up_sync(0xFFFFFFFFu, mi, o);
        if (lane >= o) mi += y;
    }
    const unsigned long long total = __shfl_sync(0xFFFFFFFFu, mi, 31);
    const unsigned hit = __ballot_sync(0xFFFFFFFFu, mi > target);
    if (hit == 0u) {
        if (lane == 0) {
            sm.xb = -1;
            sm.xmass = total;
        }
        return;
    }
    if (lane == __ffs(hit) - 1) {
        unsigned long long cum = mi - m;
        int b = 255 - 8 * lane;
        for (int i = 0; i < 7; ++i, --b) {  // the crossing lies in this lane's eight buckets
            if (cum + mass[b] > target) break;
            cum += mass[b];
        }
        sm.xb = b;
        sm.xmass = cum;
    }
    (void)cnt;
}

// Every thread: the crossing of `target` in (cnt, mass), searched by warp 0.
__device__ void block_crossing(TopPSmem& sm, const int* cnt, const unsigned long long* mass,
                               unsigned long long target, int* b, unsigned long long* above) {
    __syncthreads();  // (cnt, mass) written; earlier readers of sm.xb done
    if (threadIdx.x < 32) bucket_crossing(sm, cnt, mass, target);
    __syncthreads();
    *b = sm.xb;
    *above = sm.xmass;
}

__global__ void __launch_bounds__(kSampleThreads)
    sample_top_p_kernel(int* __restrict__ out, const bf16* __restrict__ logits, int vocab,
                        float temperature, float top_p, const float* __restrict__ uniforms) {
    extern __shared__ __align__(16) uint32_t kcnt[];  // 65536 16-bit counters, two per word
    __shared__ TopPSmem sm;
    const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
    const bf16* row = logits + (size_t)blockIdx.x * vocab;
    const int ept = (((vocab + kSampleThreads - 1) / kSampleThreads) + 7) & ~7;
    const int c0 = min(tid * ept, vocab), c1 = min(c0 + ept, vocab);
    for (int i = tid; i < 32768; i += kSampleThreads) kcnt[i] = 0u;
    // maximum logit and the softmax denominator, as sample_rows_kernel computes them
    float mx = -INFINITY;
    for (int c = c0; c < c1; c += 8) {
        float f[8];
        bf16x8_to_f32(*reinterpret_cast<const uint4*>(row + c), f);
#pragma unroll
        for (int e = 0; e < 8; ++e) mx = fmaxf(mx, f[e]);
    }
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) mx = fmaxf(mx, __shfl_xor_sync(0xFFFFFFFFu, mx, o));
    if (lane == 0) sm.fred[warp] = mx;
    __syncthreads();
    mx = sm.fred[0];
    for (int w = 1; w < 32; ++w) mx = fmaxf(mx, sm.fred[w]);
    __syncthreads();
    float sum = 0.f;
    for (int c = c0; c < c1; c += 8) {
        float f[8];
        bf16x8_to_f32(*reinterpret_cast<const uint4*>(row + c), f);
#pragma unroll
        for (int e = 0; e < 8; ++e) sum += expf((f[e] - mx) / temperature);
    }
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) sum += __shfl_xor_sync(0xFFFFFFFFu, sum, o);
    if (lane == 0) sm.fred[warp] = sum;
    __syncthreads();
    sum = 0.f;
    for (int w = 0; w < 32; ++w) sum += sm.fred[w];
    // members per key.  A 16-bit counter overflows only when all 65536 entries share one key:
    // that row is flagged and handled with its single key below.
    const uint32_t key0 = order_key(__bfloat16_as_ushort(row[0]));
    bool same = true;
    for (int c = c0; c < c1; c += 8) {
        const uint4 v = *reinterpret_cast<const uint4*>(row + c);
        const uint32_t w4[4] = {v.x, v.y, v.z, v.w};
#pragma unroll
        for (int e = 0; e < 8; ++e) {
            const uint32_t key = order_key((w4[e >> 1] >> (16 * (e & 1))) & 0xFFFFu);
            same &= key == key0;
            atomicAdd(&kcnt[key >> 1], 1u << (16 * (key & 1)));
        }
    }
    const bool all_equal = __syncthreads_and(same) != 0;
    auto count_of = [&](uint32_t key) -> int {
        if (all_equal) return key == key0 ? vocab : 0;
        return (int)((kcnt[key >> 1] >> (16 * (key & 1))) & 0xFFFFu);
    };
    // level 1: thread t sums keys [64t, 64t + 64); four threads make one bucket (high byte)
    {
        int n = 0;
        unsigned long long m = 0;
        for (int i = 0; i < 64; ++i) {
            const uint32_t key = (uint32_t)(64 * tid + i);
            const int cn = count_of(key);
            if (cn) {
                n += cn;
                m += (unsigned long long)cn * key_mass(key, mx, temperature, sum);
            }
        }
#pragma unroll
        for (int o = 1; o < 4; o <<= 1) {
            n += __shfl_xor_sync(0xFFFFFFFFu, n, o);
            m += __shfl_xor_sync(0xFFFFFFFFu, m, o);
        }
        if ((tid & 3) == 0) {
            sm.cnt1[tid >> 2] = n;
            sm.mass1[tid >> 2] = m;
        }
    }
    // level 2 of high byte hb: one key per bucket (threads 0..255)
    auto fill_level2 = [&](int hb) {
        __syncthreads();  // earlier readers of cnt2 / mass2 done
        if (tid < 256) {
            const uint32_t key = ((uint32_t)hb << 8) | (uint32_t)tid;
            const int cn = count_of(key);
            sm.cnt2[tid] = cn;
            sm.mass2[tid] = cn ? (unsigned long long)cn * key_mass(key, mx, temperature, sum) : 0ull;
        }
    };
    const unsigned long long P = (unsigned long long)((double)top_p * 0x1p62);
    int b1;
    unsigned long long above1;
    block_crossing(sm, sm.cnt1, sm.mass1, P, &b1, &above1);
    unsigned long long S2 = above1;  // mass of the kept prefix (no cut: the total)
    int kc = -1;                     // key of the group the cut falls in (-1: no cut)
    int jc = 0;                      // members of key kc kept
    if (b1 >= 0) {
        fill_level2(b1);
        int b2;
        unsigned long long above2;
        block_crossing(sm, sm.cnt2, sm.mass2, P - above1, &b2, &above2);
        if (b2 >= 0) {  // always: bucket b1's mass carries the running sum past P
            kc = (b1 << 8) | b2;
            const unsigned long long above_c = above1 + above2;
            const int gc = sm.cnt2[b2];
            const unsigned long long qc = sm.mass2[b2] / (unsigned long long)gc;
            jc = (int)((P - above_c) / qc) + 1;  // the first member whose running sum exceeds P
            if (jc > gc) jc = gc;
            S2 = above_c + (unsigned long long)jc * qc;
        }
    }
    // The draw: the first entry of the prefix whose running sum exceeds r * S2 (the reference
    // compares r with running sums of p / S2); r < 1 keeps the target inside the prefix.
    unsigned long long T = (unsigned long long)((double)uniforms[blockIdx.x] * (double)S2);
    if (T >= S2) T = S2 > 0 ? S2 - 1 : 0;
    int br;
    unsigned long long above_r1;
    block_crossing(sm, sm.cnt1, sm.mass1, T, &br, &above_r1);
    int kr = kc, jr = jc - 1;  // fallback (not reached): the prefix's last member
    if (br >= 0) {
        if (br != b1) fill_level2(br);
        int b2;
        unsigned long long above2;
        block_crossing(sm, sm.cnt2, sm.mass2, T - above_r1, &b2, &above2);
        if (b2 >= 0) {
            kr = (br << 8) | b2;
            const int g = sm.cnt2[b2];
            const unsigned long long q = sm.mass2[b2] / (unsigned long long)g;
            jr = (int)((T - above_r1 - above2) / q);
            const int lim = kr == kc ? jc : g;
            if (jr > lim - 1) jr = lim - 1;
        }
    }
    // index of member jr (in ascending index order) of key kr
    int n = 0;
    if (kr >= 0)
        for (int c = c0; c < c1; ++c) n += order_key(__bfloat16_as_ushort(row[c])) == (uint32_t)kr;
    int tot;
    const int base = block_exclusive_scan(n, sm.warp_sums, &tot);
    if (tid == 0) sm.found = 0;
    __syncthreads();
    if (kr >= 0 && base <= jr && jr < base + n) {
        int k = base;
        for (int c = c0; c < c1; ++c) {
            if (order_key(__bfloat16_as_ushort(row[c])) == (uint32_t)kr) {
                if (k == jr) {
                    sm.found = c;
                    break;
                }
                ++k;
            }
        }
    }
    __syncthreads();
    if (tid == 0) out[blockIdx.x] = sm.found;
}

__global__ void __launch_bounds__(kSampleThreads)
    sample_rows_kernel(int* __restrict__ out, const bf16* __restrict__ logits, int vocab,
                       float temperature, int top_k, float top_p,
                       const float* __restrict__ uniforms) {
    __shared__ SampleSmem sm;
    const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
    const bf16* row = logits + (size_t)blockIdx.x * vocab;
    const int ept = (((vocab + kSampleThreads - 1) / kSampleThreads) + 7) & ~7;
    const int c0 = min(tid * ept, vocab), c1 = min(c0 + ept, vocab);

    // 1. maximum logit (Engine::sample :99)
    float mx = -INFINITY;
    for (int c = c0; c < c1; c += 8) {
        float f[8];
        bf16x8_to_f32(*reinterpret_cast<const uint4*>(row + c), f);
#pragma unroll
        for (int e = 0; e < 8; ++e) mx = fmaxf(mx, f[e]);
    }
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) mx = fmaxf(mx, __shfl_xor_sync(0xFFFFFFFFu, mx, o));
    if (lane == 0) sm.fred[warp] = mx;
    __syncthreads();
    mx = sm.fred[0];
    for (int w = 1; w < 32; ++w) mx = fmaxf(mx, sm.fred[w]);
    __syncthreads();
    // 2. sum of expf((l - max) / T) over the row (:101-106)
    float sum = 0.f;
    for (int c = c0; c < c1; c += 8) {
        float f[8];
        bf16x8_to_f32(*reinterpret_cast<const uint4*>(row + c), f);
#pragma unroll
        for (int e = 0; e < 8; ++e) sum += expf((f[e] - mx) / temperature);
    }
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) sum += __shfl_xor_sync(0xFFFFFFFFu, sum, o);
    if (lane == 0) sm.fred[warp] = sum;
    // 3. the k-th largest key: two 8-bit histogram passes (radix select)
    for (int i = tid; i < 256; i += kSampleThreads) sm.hist[i] = 0;
    __syncthreads();
    sum = 0.f;
    for (int w = 0; w < 32; ++w) sum += sm.fred[w];
    if (top_k <= 0) {
        // No filter (top_k_filter and top_p_filter return at once, :62-73): the entries stay
        // in index order; renormalise (:116-119) and take the first index whose running sum
        // exceeds r (:121-128), else the last index.  The running sum is a block-wide prefix
        // sum over the threads' index-ordered slices, each slice summed in order.
        __syncthreads();  // every thread has read sm.fred (the softmax denominator) above
        float s2 = 0.f;
        for (int c = c0; c < c1; c += 8) {
            float f[8];
            bf16x8_to_f32(*reinterpret_cast<const uint4*>(row + c), f);
#pragma unroll
            for (int e = 0; e < 8; ++e) s2 += expf((f[e] - mx) / temperature) / sum;
        }
        float tot;
        block_exclusive_scan_f(s2, sm.fred, &tot);  // tot = sum of the normalised entries
        const float s2all = tot;
        float part = 0.f;
        for (int c = c0; c < c1; c += 8) {
            float f[8];
            bf16x8_to_f32(*reinterpret_cast<const uint4*>(row + c), f);
#pragma unroll
            for (int e = 0; e < 8; ++e) part += expf((f[e] - mx) / temperature) / sum / s2all;
        }
        const float base = block_exclusive_scan_f(part, sm.fred, &tot);
        if (tid == 0) sm.found = vocab - 1;
        __syncthreads();
        const float r = uniforms[blockIdx.x];
        if (c0 < c1 && base <= r && r < base + part) {
            float cs = base;
            for (int c = c0; c < c1; ++c) {
                cs += expf((__bfloat162float(row[c]) - mx) / temperature) / sum / s2all;
                if (r < cs) {
                    atomicMin(&sm.found, c);
                    break;
                }
            }
        }
        __syncthreads();
        if (tid == 0) out[blockIdx.x] = sm.found;
        return;
    }
    for (int c = c0; c < c1; c += 8) {
        const uint4 v = *reinterpret_cast<const uint4*>(row + c);
        const uint32_t w4[4] = {v.x, v.y, v.z, v.w};
#pragma unroll
        for (int e = 0; e < 8; ++e)
            atomicAdd(&sm.hist[order_key((w4[e >> 1] >> (16 * (e & 1))) & 0xFFFFu) >> 8], 1);
    }
    __syncthreads();
    if (tid == 0) {
        int cum = 0, b = 255;
        for (; b > 0; --b) {
            if (cum + sm.hist[b] >= top_k) break;
            cum += sm.hist[b];
        }
        sm.b1 = b;
        sm.above1 = cum;
    }
    __syncthreads();
    const int b1 = sm.b1;
    for (int i = tid; i < 256; i += kSampleThreads) sm.hist[i] = 0;
    __syncthreads();
    for (int c = c0; c < c1; c += 8) {
        const uint4 v = *reinterpret_cast<const uint4*>(row + c);
        const uint32_t w4[4] = {v.x, v.y, v.z, v.w};
#pragma unroll
        for (int e = 0; e < 8; ++e) {
            const uint32_t key = order_key((w4[e >> 1] >> (16 * (e & 1))) & 0xFFFFu);
            if ((int)(key >> 8) == b1) atomicAdd(&sm.hist[key & 0xFF], 1);
        }
    }
    __syncthreads();
    if (tid == 0) {
        int cum = sm.above1, b = 255;
        for (; b > 0; --b) {
            if (cum + sm.hist[b] >= top_k) break;
            cum += sm.hist[b];
        }
        sm.kstar = (b1 << 8) | b;
        sm.c_gt = cum;
    }
    __syncthreads();
    // 4. gather the k candidates: every key above K*, and the lowest-index ties at K*
    const uint32_t kstar = (uint32_t)sm.kstar;
    const int c_gt = sm.c_gt, need = top_k - c_gt;
    int n_gt = 0, n_eq = 0;
    for (int c = c0; c < c1; c += 8) {
        const uint4 v = *reinterpret_cast<const uint4*>(row + c);
        const uint32_t w4[4] = {v.x, v.y, v.z, v.w};
#pragma unroll
        for (int e = 0; e < 8; ++e) {
            const uint32_t key = order_key((w4[e >> 1] >> (16 * (e & 1))) & 0xFFFFu);
            n_gt += key > kstar;
            n_eq += key == kstar;
        }
    }
    int tot;
    int slot_gt = block_exclusive_scan(n_gt, sm.warp_sums, &tot);
    int rank_eq = block_exclusive_scan(n_eq, sm.warp_sums, &tot);
    int P = 1;
    while (P < top_k) P <<= 1;
    for (int i = tid; i < P; i += kSampleThreads) sm.cand[i] = 0ull;
    __syncthreads();
    for (int c = c0; c < c1; c += 8) {
        const uint4 v = *reinterpret_cast<const uint4*>(row + c);
        const uint32_t w4[4] = {v.x, v.y, v.z, v.w};
#pragma unroll
        for (int e = 0; e < 8; ++e) {
            const uint32_t key = order_key((w4[e >> 1] >> (16 * (e & 1))) & 0xFFFFu);
            const unsigned long long ck =
                ((unsigned long long)key << 32) | (0xFFFFFFFFu - (uint32_t)(c + e));
            if (key > kstar) {
                sm.cand[slot_gt++] = ck;
            } else if (key == kstar) {
                if (rank_eq < need) sm.cand[c_gt + rank_eq] = ck;
                ++rank_eq;
            }
        }
    }
    __syncthreads();
    // 5. bitonic sort, descending: larger value first, equal values by ascending index
    for (int size = 2; size <= P; size <<= 1) {
        for (int stride = size >> 1; stride > 0; stride >>= 1) {
            for (int i = tid; i < P; i += kSampleThreads) {
                const int j = i ^ stride;
                if (j > i) {
                    const bool desc = (i & size) == 0;
                    const unsigned long long a = sm.cand[i], b = sm.cand[j];
                    if (desc ? (a < b) : (a > b)) {
                        sm.cand[i] = b;
                        sm.cand[j] = a;
                    }
                }
            }
            __syncthreads();
        }
    }
    // 6. the candidates' normalised probabilities (p = expf(scaled) / sum, :103-110), then
    // top-p, renormalisation and the draw with the reference's sequential fp32 sums
    for (int i = tid; i < top_k; i += kSampleThreads)
        sm.q[i] = expf((key_value((uint32_t)(sm.cand[i] >> 32)) - mx) / temperature) / sum;
    __syncthreads();
    if (tid == 0) {
        int n = top_k;
        if (top_p < 1.0f) {
            float cs = 0.f;
            for (int i = 0; i < n; ++i) {
                cs += sm.q[i];
                if (cs > top_p) {
                    n = i + 1;
                    break;
                }
            }
        }
        float s2 = 0.f;
        for (int i = 0; i < n; ++i) s2 += sm.q[i];
        const float r = uniforms[blockIdx.x];
        float cs = 0.f;
        int chosen = n - 1;
        for (int i = 0; i < n; ++i) {
            cs += sm.q[i] / s2;
            if (r < cs) {
                chosen = i;
                break;
            }
        }
        out[blockIdx.x] = (int)(0xFFFFFFFFu - (uint32_t)(sm.cand[chosen] & 0xFFFFFFFFull));
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

int nc_sample_rows(int* out, const void* logits, int rows, int vocab, float temperature,
                   int top_k, float top_p, const float* uniforms, cudaStream_t stream) {
    using namespace nc;
    if (rows < 0 || vocab < 8 || (vocab & 7) || !(temperature >= 0.f)) return NC_ERR_INVALID_ARG;
    if (rows == 0) return NC_OK;
    if (!out || !logits) return NC_ERR_INVALID_ARG;
    if (reinterpret_cast<uintptr_t>(logits) & 15) return NC_ERR_MISALIGNED;
    if (temperature == 0.f) return nc_argmax_rows(out, logits, rows, vocab, stream);
    if (!(top_p > 0.f) || !uniforms) return NC_ERR_INVALID_ARG;
    // top_k <= 0 or >= vocab: no top-k filter (top_p, if on, then cuts the whole row; its
    // per-key counters are 16-bit, which holds for vocab <= 65536).
    const bool no_topk = top_k <= 0 || top_k >= vocab;
    if (!no_topk && top_k > kSampleMaxK) return NC_ERR_INVALID_ARG;
    if (no_topk && top_p < 1.0f) {
        if (vocab > 65536) return NC_ERR_INVALID_ARG;
        int dev = 0;
        cudaError_t e = cudaGetDevice(&dev);
        if (e != cudaSuccess) return internal_cuda_fail(e);
        if (dev < 0 || dev >= kTopPMaxDev) return NC_ERR_INVALID_ARG;
        static bool attr_set[kTopPMaxDev] = {};
        if (!attr_set[dev]) {
            e = cudaFuncSetAttribute(sample_top_p_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                     (int)kTopPCountBytes);
            if (e != cudaSuccess) return internal_cuda_fail(e);
            attr_set[dev] = true;
        }
        sample_top_p_kernel<<<rows, kSampleThreads, kTopPCountBytes, stream>>>(
            out, static_cast<const bf16*>(logits), vocab, temperature, top_p, uniforms);
        e = cudaGetLastError();
        return e == cudaSuccess ? NC_OK : internal_cuda_fail(e);
    }
    if (no_topk) top_k = 0;
    sample_rows_kernel<<<rows, kSampleThreads, 0, stream>>>(
        out, static_cast<const bf16*>(logits), vocab, temperature, top_k, top_p, uniforms);
    cudaError_t e = cudaGetLastError();
    return e == cudaSuccess ? NC_OK : internal_cuda_fail(e);
}

}  // extern "C"

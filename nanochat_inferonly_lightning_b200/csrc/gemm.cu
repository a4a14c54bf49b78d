// Skinny bf16 GEMM for the decode step: out[M, N] = epilogue(x[M, K] . w[N, K]^T) with M <= 64
// (one row per sequence of a decode batch).  This is the reference's gemm_half /
// gemm_half_residual small-M branch (kernels/gemm.cu:62-166) together with the RMSNorm,
// ReLU^2 and tanh-cap passes around its decode call sites (src/model.cpp:110-177).
//
// At M <= 64 the work is streaming the weight: 2 bytes per weight element, 2*M flops.  The
// kernel is laid out for that:
//  * swap-AB: the weight tile is the MMA's A operand (M_mma = 128 output features per CTA) and
//    the activations the B operand (N_mma = M rounded up to 16, 32 or 64), so one
//    tcgen05.mma covers the whole batch and the accumulator is a 128 x N_mma fp32 tile in TMEM;
//  * the weight is streamed by TMA in 128 x 64 (16 KB, 128-byte swizzled) boxes through a
//    6-stage ring, marked L2 evict-first (read once per step; the activations, partials and
//    KV caches stay in L2);
//  * the K dimension is split across CTAs when N / 128 alone gives too few CTAs.  The S <= 12
//    splits of one output tile are launched as one thread-block cluster: each CTA leaves its
//    fp32 partial tile in its own shared memory, and after a cluster barrier CTA r sums rows
//    m = r, r + S, ... of the tile over all S CTAs' shared memory (distributed shared memory
//    loads, in split order, so results do not depend on timing) and runs the epilogue for
//    them.  No global workspace, no atomics;
//  * 6 stages of 16 + 2 KB leave room for two CTAs per SM, and the launch is a programmatic
//    dependent launch: the weight boxes of the first stages are requested before
//    griddepcontrol.wait (weights are never written by a preceding kernel), so a GEMM that
//    follows another kernel starts streaming while that kernel finishes;
//  * the epilogue applies the fused steps (RMSNorm row scale, residual, ReLU^2, tanh cap)
//    on the fp32 sum and rounds once to bf16.
//
// Warp roles (192 threads): warp 0 lane 0 issues TMA, warp 1 issues the MMAs (elected lane)
// and owns the TMEM allocation, warps 2-5 compute the RMSNorm scales, then read the
// accumulator (warp w reads TMEM lanes 32*(w%4)..+31, the quarter its SM sub-partition may
// access) and run the epilogue.  Every mbarrier wait is bounded (sm100_ptx.cuh).
#include <cooperative_groups.h>
#include <cuda.h>

#include <algorithm>
#include <cstdint>
#include <mutex>

#include "../../include/nanochat_attn.h"
#include "nc_common.cuh"
#include "sm100_ptx.cuh"

namespace nc {

namespace {

constexpr int kGemmThreads = 192;
constexpr int kTileN = 128;                      // output features per CTA (MMA M)
constexpr int kTileK = 64;                       // K per stage: one 128-byte swizzled row
constexpr int kStages = 6;
constexpr int kWBoxBytes = kTileN * kTileK * 2;  // 16 KB
constexpr int kMaxRows = 64;
// Cluster size limit (above 8 is non-portable).  Measured on the 2176 x 8704 down projection
// at M = 8: 9.4 us with 8 splits, 8.6 with 12, 12.7 with 16 (16-CTA clusters are harder to
// place next to the CTAs of the neighbouring kernels).
constexpr int kMaxSplits = 12;

struct GemmTail {
    uint64_t full[kStages];
    uint64_t empty[kStages];
    uint64_t accum;
    uint64_t drain;
    float rnorm[kMaxRows];
    uint32_t tmem;
    int abort;
};

// RMSNorm scales (reference kernels/rmsnorm.cu:17-48: fp32 sum of squares, rsqrt(sum / K +
// 1e-6)) of `count` rows of x, row i = mq + i * step, into rs_out[i * step], by one warp: four
// rows at a time, each lane summing the 16-byte pieces lane, lane + 32, ... of a row in order,
// then a butterfly sum.  The pieces of the four rows (up to nine per lane and row, K <= 2304 in
// one round) are all loaded before any is summed, so a group of rows costs one memory round
// trip.  Rows at or past M get the scale of an all-zero row.  Plain (coherent) loads: x may
// have been written by the kernel this one overlaps through programmatic dependent launch.
__device__ __forceinline__ void row_scales_warp(const bf16* x, int M, int K, int mq, int step,
                                                int count, int lane, float* rs_out) {
    constexpr int kPieces = 9;
    const int kp = K / 8;  // 16-byte pieces per row
    for (int r4 = 0; r4 < count; r4 += 4) {
        float ss[4] = {0.f, 0.f, 0.f, 0.f};
        for (int c0 = lane; c0 < kp; c0 += 32 * kPieces) {
            uint4 v[4][kPieces];
#pragma unroll
            for (int u = 0; u < 4; ++u) {
                const int mr = mq + (r4 + u) * step;
                const uint4* row = reinterpret_cast<const uint4*>(x + (size_t)(mr < M ? mr : 0) * K);
#pragma unroll
                for (int j = 0; j < kPieces; ++j) {
                    const int c = c0 + 32 * j;
                    v[u][j] = (mr < M && c < kp) ? row[c] : make_uint4(0u, 0u, 0u, 0u);
                }
            }
#pragma unroll
            for (int u = 0; u < 4; ++u) {
#pragma unroll
                for (int j = 0; j < kPieces; ++j) {
                    float f[8];
                    bf16x8_to_f32(v[u][j], f);
#pragma unroll
                    for (int e = 0; e < 8; ++e) ss[u] = __fmaf_rn(f[e], f[e], ss[u]);
                }
            }
        }
#pragma unroll
        for (int u = 0; u < 4; ++u) {
#pragma unroll
            for (int o = 16; o > 0; o >>= 1) ss[u] += __shfl_xor_sync(0xFFFFFFFFu, ss[u], o);
        }
        if (lane < 4 && r4 + lane < count) {
            const float t = lane == 0 ? ss[0] : lane == 1 ? ss[1] : lane == 2 ? ss[2] : ss[3];
            rs_out[(r4 + lane) * step] = rsqrtf(t / (float)K + kNormEps);
        }
    }
}

template <int MP>
constexpr int gemm_smem_bytes() {
    return kStages * (kWBoxBytes + MP * 128) + (int)sizeof(GemmTail) + 1024;
}

struct GemmParams {
    bf16* out;
    const bf16* x;
    const bf16* residual;
    int M, N, K;
    int kb_total;       // ceil(K / 64)
    int kb_per;         // K boxes per split
    int splits;         // CTAs per output tile = cluster size along y
    int flags;
    float cap;
    int seg_cols;
    int* status;
};

// Wait tags (ORed with kStatusTimeoutMbar into the status word).
constexpr int kTagEmpty = 0x41, kTagFull = 0x42, kTagAccum = 0x43, kTagDrainLoad = 0x44,
              kTagDrainMma = 0x45;

// Fused epilogue of one output element (row m, feature n) and its bf16 store.
__device__ __forceinline__ void finish(const GemmParams& p, const float* rnorm, int m, int n,
                                       float v) {
    if (p.flags & NC_GEMM_NORM_INPUT) v *= rnorm[m];
    if (p.flags & NC_GEMM_RESIDUAL) v += __bfloat162float(p.residual[(size_t)m * p.N + n]);
    if (p.flags & NC_GEMM_RELU2) {
        v = fmaxf(v, 0.f);
        v *= v;
    }
    if (p.flags & NC_GEMM_TANH_CAP) v = p.cap * tanhf(v / p.cap);
    const int seg = p.seg_cols;
    p.out[(size_t)(n / seg) * ((size_t)p.M * seg) + (size_t)m * seg + (n % seg)] =
        __float2bfloat16(v);
}

template <int MP>
__global__ void __launch_bounds__(kGemmThreads, 2)
    gemm_skinny_kernel(const __grid_constant__ CUtensorMap tmW,
                       const __grid_constant__ CUtensorMap tmX, const GemmParams p) {
    extern __shared__ uint8_t smem_raw[];
    // 128-byte swizzled TMA boxes want 1024-byte aligned destinations.
    const uint32_t raw = smem_u32(smem_raw);
    uint8_t* base = smem_raw + (((raw + 1023u) & ~1023u) - raw);
    uint8_t* sW = base;
    uint8_t* sX = base + kStages * kWBoxBytes;
    GemmTail* tail = reinterpret_cast<GemmTail*>(sX + kStages * MP * 128);
    constexpr uint32_t kXBoxBytes = MP * 128;
    constexpr uint32_t kTmemCols = MP < 32 ? 32 : MP;

    const int warp = threadIdx.x >> 5;
    const int lane = threadIdx.x & 31;
    const int tile = blockIdx.x;
    const int split = blockIdx.y;  // = rank in the cluster (cluster dims 1 x splits)
    const int n0 = tile * kTileN;
    const int kb0 = split * p.kb_per;
    const int nkb = min(p.kb_total, kb0 + p.kb_per) - kb0;  // >= 1 (host plans no empty split)

    if (threadIdx.x == 0) {
        for (int i = 0; i < kStages; ++i) {
            mbar_init(&tail->full[i], 1);
            mbar_init(&tail->empty[i], 1);
        }
        mbar_init(&tail->accum, 1);
        mbar_init(&tail->drain, 1);
        tail->abort = 0;
        fence_mbar_init();
    }
    if (warp == 0 && lane == 0) {
        prefetch_tmap(&tmW);
        prefetch_tmap(&tmX);
    }
    if (warp == 1) {
        tmem_alloc(&tail->tmem, kTmemCols);
        tmem_relinquish();
    }
    tc_fence_before();
    __syncthreads();
    tc_fence_after();
    const uint32_t tmem = tail->tmem;
    volatile int* abort_flag = &tail->abort;
    // Let a dependent launch (the next GEMM of the step) start now: its CTAs take the SM slots
    // this grid leaves free and stream their first weight boxes while this grid works; they
    // read nothing this grid writes before their griddepcontrol.wait.
    griddep_launch_dependents();

    if (warp == 0) {
        // ------------------------------------------------------------------ TMA producer
        if (lane == 0) {
            const uint64_t pol = l2_policy_evict_first();
            const int pre = min(nkb, kStages);
            // Weight boxes of the first stages: independent of earlier kernels.
            for (int i = 0; i < pre; ++i) {
                mbar_arrive_expect_tx(&tail->full[i], kWBoxBytes + kXBoxBytes);
                tma_load_2d_hint(sW + i * kWBoxBytes, &tmW, &tail->full[i], (kb0 + i) * kTileK,
                                 n0, pol);
            }
            griddep_wait();
            for (int i = 0; i < pre; ++i)
                tma_load_2d(sX + i * kXBoxBytes, &tmX, &tail->full[i], (kb0 + i) * kTileK, 0);
            int issued = pre;
            for (int i = pre; i < nkb; ++i) {
                const int st = i % kStages;
                if (!mbar_wait(&tail->empty[st], ((i / kStages) - 1) & 1, abort_flag, p.status,
                               kTagEmpty))
                    break;
                mbar_arrive_expect_tx(&tail->full[st], kWBoxBytes + kXBoxBytes);
                tma_load_2d_hint(sW + st * kWBoxBytes, &tmW, &tail->full[st],
                                 (kb0 + i) * kTileK, n0, pol);
                tma_load_2d(sX + st * kXBoxBytes, &tmX, &tail->full[st], (kb0 + i) * kTileK, 0);
                issued = i + 1;
            }
            if (*abort_flag) {
                // Leaving early: wait for the copies still in flight into this CTA's ring.
                for (int i = max(issued - kStages, 0); i < issued; ++i)
                    mbar_wait_drain(&tail->full[i % kStages], (i / kStages) & 1, p.status,
                                    kTagDrainLoad);
            }
        }
        __syncwarp();
    } else if (warp == 1) {
        // ------------------------------------------------------------------ MMA issuer
        const uint32_t idesc = idesc_bf16_f32(kTileN, MP, false);  // both operands K-major
        const uint64_t dW0 = smem_desc_sw128(smem_u32(sW), 16, 1024);
        const uint64_t dX0 = smem_desc_sw128(smem_u32(sX), 16, 1024);
        bool ok = true;
        for (int i = 0; i < nkb; ++i) {
            const int st = i % kStages;
            ok = __all_sync(0xFFFFFFFFu, mbar_wait(&tail->full[st], (i / kStages) & 1,
                                                   abort_flag, p.status, kTagFull));
            if (!ok) break;
            tc_fence_after();
            const uint64_t dW = dW0 + (uint64_t)(st * (kWBoxBytes >> 4));
            const uint64_t dX = dX0 + (uint64_t)(st * (kXBoxBytes >> 4));
#pragma unroll
            for (int kk = 0; kk < 4; ++kk)  // 16 K-elements = 32 bytes per MMA
                mma_ss_warp(tmem, dW + kk * 2, dX + kk * 2, idesc, (i | kk) ? 1u : 0u);
            mma_commit_warp(&tail->empty[st]);
        }
        if (ok) {
            mma_commit_warp(&tail->accum);
        } else {
            // Leaving early: wait for this warp's MMAs before TMEM is released.
            mma_commit_warp(&tail->drain);
            mbar_wait_drain(&tail->drain, 0, p.status, kTagDrainMma);
        }
        __syncwarp();
    } else {
        // ------------------------------------------------------------------ epilogue
        const int quarter = warp & 3;
        const int n = n0 + quarter * 32 + lane;
        griddep_wait();
        if (p.flags & NC_GEMM_NORM_INPUT) {
            // RMSNorm scale of each input row, rows m = warp - 2 (mod 4) in this warp.
            const int m0 = warp - 2;
            if (m0 < p.M)
                row_scales_warp(p.x, p.M, p.K, m0, 4, (p.M - m0 + 3) / 4, lane, tail->rnorm + m0);
        }
        float acc[MP];
#pragma unroll
        for (int m = 0; m < MP; ++m) acc[m] = 0.f;
        const bool ok = __all_sync(0xFFFFFFFFu, mbar_wait(&tail->accum, 0, abort_flag, p.status,
                                                          kTagAccum));
        tc_fence_after();
        if (ok) {
#pragma unroll
            for (int c = 0; c < MP / 16; ++c) {
                uint32_t r[16];
                tmem_ld16_sync(tmem + ((uint32_t)(quarter * 32) << 16) + c * 16, r);
#pragma unroll
                for (int j = 0; j < 16; ++j) acc[c * 16 + j] = __uint_as_float(r[j]);
            }
        }
        named_bar_sync(1, 128);  // RMSNorm scales visible to all epilogue threads
        if (p.splits == 1) {
            if (n < p.N) {
#pragma unroll
                for (int m = 0; m < MP; ++m)
                    if (m < p.M) finish(p, tail->rnorm, m, n, acc[m]);
            }
        } else if (ok) {
            // Partial tile into this CTA's (now idle) weight ring, [m][128] fp32.  Every copy
            // into the ring has landed: each was consumed by an MMA that the accumulator
            // barrier waited for.
            float* red = reinterpret_cast<float*>(sW);
            const int row = quarter * 32 + lane;  // the TMEM lane this thread read
#pragma unroll
            for (int m = 0; m < MP; ++m)
                if (m < p.M) red[m * kTileN + row] = acc[m];
        }
    }

    if (p.splits > 1) {
        // Cluster reduction: all threads of all CTAs of the tile take both barriers.
        namespace cg = cooperative_groups;
        cg::cluster_group cluster = cg::this_cluster();
        cluster.sync();  // release/acquire: every CTA's partial tile is visible
        if (warp >= 2 && !*abort_flag) {
            const int et = threadIdx.x - 64;
            const int n = n0 + et;
            const float* red = reinterpret_cast<const float*>(sW);
            const float* parts[kMaxSplits];
#pragma unroll
            for (int r = 0; r < kMaxSplits; ++r)
                parts[r] = r < p.splits ? cluster.map_shared_rank(red, r) : red;
            if (n < p.N) {
                for (int m = split; m < p.M; m += p.splits) {
                    float v[kMaxSplits];
#pragma unroll
                    for (int r = 0; r < kMaxSplits; ++r)
                        v[r] = r < p.splits ? parts[r][m * kTileN + et] : 0.f;
                    float sum = v[0];
#pragma unroll
                    for (int r = 1; r < kMaxSplits; ++r)
                        if (r < p.splits) sum += v[r];
                    finish(p, tail->rnorm, m, n, sum);
                }
            }
        }
        cluster.sync();  // no CTA leaves while another still reads its shared memory
    }

    tc_fence_before();
    __syncthreads();
    if (warp == 1) {
        tc_fence_after();
        tmem_dealloc(tmem, kTmemCols);
    }
}

// ---------------------------------------------------------------------------------------
// Prompt-pass GEMM on single CTAs (nc_gemm for M <= 128; larger M runs on the CTA pairs of
// gemm_pair_kernel below, which keeps these roles): persistent, one CTA per SM, 128 x 256
// output tiles (one tcgen05.mma of M = 128 rows of x, N = 256 output features,
// K = 16 per step), x and w boxes staged by TMA (no multicast) through a 4-stage ring of
// 48 KB stages, and two 256-column accumulators in TMEM so that the epilogue of one tile
// overlaps the MMAs of the next.  Tiles are numbered with the row block fastest, so the CTAs
// working at the same time share each weight tile through L2.
// Warp roles (192 threads): warp 0 lane 0 issues TMA, warp 1 the MMAs (elected lane) and owns
// TMEM, warps 2-5 the epilogue (warp w reads TMEM lanes 32*(w%4)..+31 = the tile's rows):
// while a tile's MMAs run they compute each row's RMSNorm scale from x (NC_GEMM_NORM_INPUT),
// then read the accumulator 32 columns at a time, hand it back once all 256 are read, apply
// the fused steps of finish() on the fp32 values and store 16-byte groups of 8 outputs.
// ---------------------------------------------------------------------------------------
constexpr int kTThreads = 192;
constexpr int kTBM = 128;
constexpr int kTBN = 256;
constexpr int kTStages = 4;
constexpr int kTABytes = kTBM * kTileK * 2;  // 16 KB
constexpr int kTBBytes = kTBN * kTileK * 2;  // 32 KB
constexpr uint32_t kTTmemCols = 512;

struct TileTail {
    uint64_t full[kTStages];
    uint64_t empty[kTStages];
    uint64_t acc_full[2];
    uint64_t acc_empty[2];
    uint64_t drain;
    float rs[kTBM];  // RMSNorm scale of each row of the current tile (its epilogue warp's rows)
    uint32_t tmem;
    int abort;
};
constexpr int kTSmemBytes = kTStages * (kTABytes + kTBBytes) + (int)sizeof(TileTail) + 1024;
static_assert(kTSmemBytes <= 227 * 1024, "shared memory budget");

struct TileParams {
    bf16* out;
    const bf16* x;
    const bf16* residual;
    int M, N, K;
    int kb_total;
    int m_tiles, n_tiles, tiles;
    int n_per;  // > 0: CTA c keeps row block c % m_tiles and takes its column tiles
                // c / m_tiles, + n_per, ...; 0: tiles t = c, c + grid, ... (row block fastest)
    int flags;
    float cap;
    int seg_cols;
    int* status;
};

// The tiles of one CTA, in order (every role walks the same sequence).
struct TileWalk {
    int mt, nt, t;
    __device__ __forceinline__ void start(const TileParams& p) {
        if (p.n_per) {
            mt = blockIdx.x % p.m_tiles;
            nt = blockIdx.x / p.m_tiles;
        } else {
            t = blockIdx.x;
            mt = t % p.m_tiles;
            nt = t / p.m_tiles;
        }
    }
    __device__ __forceinline__ bool valid(const TileParams& p) const {
        return p.n_per ? nt < p.n_tiles : t < p.tiles;
    }
    __device__ __forceinline__ void next(const TileParams& p) {
        if (p.n_per) {
            nt += p.n_per;
        } else {
            t += gridDim.x;
            mt = t % p.m_tiles;
            nt = t / p.m_tiles;
        }
    }
};

constexpr int kTagTEmpty = 0x51, kTagTFull = 0x52, kTagTAccFull = 0x53, kTagTAccEmpty = 0x54,
              kTagTDrainLoad = 0x55, kTagTDrainMma = 0x56;

__global__ void __launch_bounds__(kTThreads, 1)
    gemm_tile_kernel(const __grid_constant__ CUtensorMap tmX, const __grid_constant__ CUtensorMap tmW,
                     const TileParams p) {
    extern __shared__ uint8_t smem_raw[];
    const uint32_t raw = smem_u32(smem_raw);
    uint8_t* base = smem_raw + (((raw + 1023u) & ~1023u) - raw);
    uint8_t* sA = base;                          // stage i at sA + i * kTABytes
    uint8_t* sB = base + kTStages * kTABytes;    // stage i at sB + i * kTBBytes
    TileTail* tail = reinterpret_cast<TileTail*>(sB + kTStages * kTBBytes);
    const int warp = threadIdx.x >> 5;
    const int lane = threadIdx.x & 31;

    if (threadIdx.x == 0) {
        for (int i = 0; i < kTStages; ++i) {
            mbar_init(&tail->full[i], 1);
            mbar_init(&tail->empty[i], 1);
        }
        for (int i = 0; i < 2; ++i) {
            mbar_init(&tail->acc_full[i], 1);
            mbar_init(&tail->acc_empty[i], 128);
        }
        mbar_init(&tail->drain, 1);
        tail->abort = 0;
        fence_mbar_init();
    }
    if (warp == 0 && lane == 0) {
        prefetch_tmap(&tmX);
        prefetch_tmap(&tmW);
    }
    if (warp == 1) {
        tmem_alloc(&tail->tmem, kTTmemCols);
        tmem_relinquish();
    }
    tc_fence_before();
    __syncthreads();
    tc_fence_after();
    const uint32_t tmem = tail->tmem;
    volatile int* abort_flag = &tail->abort;
    // Programmatic dependent launch: the setup above may overlap the previous kernel's tail;
    // nothing in global memory is read or written before this wait, which returns once that
    // kernel has completed and its writes are visible.
    griddep_launch_dependents();
    griddep_wait();

    if (warp == 0) {
        // ------------------------------------------------------------------ TMA producer
        if (lane == 0) {
            int it = 0;  // running k-block count of this CTA: stage it % kTStages
            bool ok = true;
            TileWalk tw;
            for (tw.start(p); ok && tw.valid(p); tw.next(p)) {
                const int m0 = tw.mt * kTBM;
                const int n0 = tw.nt * kTBN;
                for (int kb = 0; kb < p.kb_total; ++kb, ++it) {
                    const int st = it % kTStages;
                    if (it >= kTStages &&
                        !(ok = mbar_wait(&tail->empty[st], ((it / kTStages) - 1) & 1, abort_flag,
                                         p.status, kTagTEmpty)))
                        break;
                    mbar_arrive_expect_tx(&tail->full[st], kTABytes + kTBBytes);
                    tma_load_2d(sA + st * kTABytes, &tmX, &tail->full[st], kb * kTileK, m0);
                    tma_load_2d(sB + st * kTBBytes, &tmW, &tail->full[st], kb * kTileK, n0);
                }
            }
            if (!ok) {
                // Leaving early: wait for the copies still in flight into this CTA's ring.
                for (int i = max(it - kTStages, 0); i < it; ++i)
                    mbar_wait_drain(&tail->full[i % kTStages], (i / kTStages) & 1, p.status,
                                    kTagTDrainLoad);
            }
        }
        __syncwarp();
    } else if (warp == 1) {
        // ------------------------------------------------------------------ MMA issuer
        const uint32_t idesc = idesc_bf16_f32(kTBM, kTBN, false);  // both operands K-major
        const uint64_t dA0 = smem_desc_sw128(smem_u32(sA), 16, 1024);
        const uint64_t dB0 = smem_desc_sw128(smem_u32(sB), 16, 1024);
        bool ok = true;
        int it = 0, lt = 0;
        TileWalk tw;
        for (tw.start(p); ok && tw.valid(p); tw.next(p), ++lt) {
            const int buf = lt & 1;
            // The accumulator buffer is free once the epilogue read the tile before last.
            if (lt >= 2 && !(ok = __all_sync(0xFFFFFFFFu,
                                             mbar_wait(&tail->acc_empty[buf], ((lt >> 1) - 1) & 1,
                                                       abort_flag, p.status, kTagTAccEmpty))))
                break;
            tc_fence_after();
            const uint32_t acc = tmem + buf * kTBN;
            for (int kb = 0; kb < p.kb_total; ++kb, ++it) {
                const int st = it % kTStages;
                if (!(ok = __all_sync(0xFFFFFFFFu, mbar_wait(&tail->full[st], (it / kTStages) & 1,
                                                             abort_flag, p.status, kTagTFull))))
                    break;
                tc_fence_after();
                const uint64_t dA = dA0 + (uint64_t)(st * (kTABytes >> 4));
                const uint64_t dB = dB0 + (uint64_t)(st * (kTBBytes >> 4));
#pragma unroll
                for (int kk = 0; kk < 4; ++kk)  // 16 K-elements = 32 bytes per MMA
                    mma_ss_warp(acc, dA + kk * 2, dB + kk * 2, idesc, (kb | kk) ? 1u : 0u);
                mma_commit_warp(&tail->empty[st]);
            }
            if (ok) mma_commit_warp(&tail->acc_full[buf]);
        }
        // Leave only once every MMA issued above has completed: TMEM is released below.
        mma_commit_warp(&tail->drain);
        mbar_wait_drain(&tail->drain, 0, p.status, kTagTDrainMma);
        __syncwarp();
    } else {
        // ------------------------------------------------------------------ epilogue
        const int quarter = warp & 3;
        const int r = quarter * 32 + lane;  // the tile row (TMEM lane) this thread owns
        const uint32_t lane_base = static_cast<uint32_t>(quarter * 32) << 16;
        int lt = 0;
        float rs = 1.f;
        TileWalk tw;
        for (tw.start(p); tw.valid(p); tw.next(p), ++lt) {
            const int buf = lt & 1;
            const int m = tw.mt * kTBM + r;
            const int n0 = tw.nt * kTBN;
            // RMSNorm scale of the warp's 32 rows, while the tile's MMAs run.  A CTA that keeps
            // one row block computes them once.
            if ((p.flags & NC_GEMM_NORM_INPUT) && (lt == 0 || !p.n_per)) {
                row_scales_warp(p.x, p.M, p.K, tw.mt * kTBM + quarter * 32, 1, 32, lane,
                                tail->rs + quarter * 32);
                __syncwarp();
                rs = tail->rs[quarter * 32 + lane];
                __syncwarp();  // read before the next tile's scales overwrite it
            }
            if (!__all_sync(0xFFFFFFFFu, mbar_wait(&tail->acc_full[buf], (lt >> 1) & 1, abort_flag,
                                                   p.status, kTagTAccFull)))
                break;
            tc_fence_after();
            // The residual of the first chunk, then each next chunk's ahead of this one's work:
            // its loads are in flight while this chunk is read from TMEM and stored.
            uint4 rnext[4];
            auto load_res = [&](int c, uint4 (&r)[4]) {
#pragma unroll
                for (int g8 = 0; g8 < 4; ++g8) {
                    const int n = n0 + 32 * c + 8 * g8;
                    r[g8] = ((p.flags & NC_GEMM_RESIDUAL) && m < p.M && n < p.N)
                                ? *reinterpret_cast<const uint4*>(p.residual + (size_t)m * p.N + n)
                                : make_uint4(0u, 0u, 0u, 0u);
                }
            };
            load_res(0, rnext);
            for (int c = 0; c < kTBN / 32; ++c) {
                uint4 rcur[4];
#pragma unroll
                for (int g8 = 0; g8 < 4; ++g8) rcur[g8] = rnext[g8];
                if (c + 1 < kTBN / 32) load_res(c + 1, rnext);
                uint32_t v[32];
                tmem_ld32_sync(tmem + buf * kTBN + 32 * c + lane_base, v);
                if (c == kTBN / 32 - 1) {
                    // Every column of this accumulator has been read: the tile after next may
                    // accumulate into it.
                    tc_fence_before();
                    mbar_arrive(&tail->acc_empty[buf]);
                }
                if (m >= p.M) continue;
#pragma unroll
                for (int g8 = 0; g8 < 4; ++g8) {
                    const int n = n0 + 32 * c + 8 * g8;
                    if (n >= p.N) break;
                    float f[8];
#pragma unroll
                    for (int e = 0; e < 8; ++e) f[e] = __uint_as_float(v[8 * g8 + e]);
                    if (p.flags & NC_GEMM_NORM_INPUT) {
#pragma unroll
                        for (int e = 0; e < 8; ++e) f[e] *= rs;
                    }
                    if (p.flags & NC_GEMM_RESIDUAL) {
                        float rr[8];
                        bf16x8_to_f32(rcur[g8], rr);
#pragma unroll
                        for (int e = 0; e < 8; ++e) f[e] += rr[e];
                    }
                    if (p.flags & NC_GEMM_RELU2) {
#pragma unroll
                        for (int e = 0; e < 8; ++e) {
                            const float y = fmaxf(f[e], 0.f);
                            f[e] = y * y;
                        }
                    }
                    if (p.flags & NC_GEMM_TANH_CAP) {
#pragma unroll
                        for (int e = 0; e < 8; ++e) f[e] = p.cap * tanhf(f[e] / p.cap);
                    }
                    const int seg = p.seg_cols;
                    bf16* dst = p.out + (size_t)(n / seg) * ((size_t)p.M * seg) + (size_t)m * seg +
                                (n % seg);
                    *reinterpret_cast<uint4*>(dst) = f32_to_bf16x8(f);
                }
            }
        }
    }

    tc_fence_before();
    __syncthreads();
    if (warp == 1) {
        tc_fence_after();
        tmem_dealloc(tmem, kTTmemCols);
    }
}

// ---------------------------------------------------------------------------------------
// nc_gemm on CTA pairs (cta_group::2).  The two CTAs of a cluster share 256 x 256 output
// tiles: each CTA stages its own 128 rows of x and 128 of the tile's 256 weight rows (16 KB
// each per 64-deep K block, no multicast), the even CTA issues one M = 256, N = 256 MMA per 16
// K-elements that reads both CTAs' halves, and each CTA's tensor memory receives its own 128
// rows of the accumulator.  Per SM that is 32 KB staged from L2 per 512 cycles of MMAs,
// against 48 KB for a CTA alone on 128 x 256 tiles.
//   warp 0      TMA producer of each CTA; the loads of both CTAs count on the even CTA's full
//               barrier (which expects both halves); each CTA waits on its own empty barrier.
//   warp 1      the even CTA's MMA issuer: commits every stage's release, and each
//               accumulator's completion, to the barriers of both CTAs.
//   warps 2-5   epilogue of each CTA on its own 128 rows (as in gemm_tile_kernel); each warp
//               releases an accumulator buffer with one arrival on the even CTA's barrier.
// ---------------------------------------------------------------------------------------
constexpr int kPStages = 6;
constexpr int kPABytes = kTBM * kTileK * 2;        // 16 KB: this CTA's 128 rows of x
constexpr int kPBBytes = (kTBN / 2) * kTileK * 2;  // 16 KB: this CTA's 128 rows of w

struct PairTail {
    uint64_t full[kPStages];   // even CTA: both CTAs' copies of a stage landed (64 KB)
    uint64_t empty[kPStages];  // each CTA: the MMAs reading its copy of the stage are done
    uint64_t acc_full[2];      // each CTA: accumulator buffer complete
    uint64_t acc_empty[2];     // even CTA: all eight epilogue warps read the buffer
    uint64_t drain;
    float rs[kTBM];
    uint32_t tmem;
    int abort;
};
constexpr int kPSmemBytes = kPStages * (kPABytes + kPBBytes) + (int)sizeof(PairTail) + 1024;
static_assert(kPSmemBytes <= 227 * 1024, "shared memory budget");

// The tiles of one CTA pair, in order; m_tiles counts 256-row blocks.
struct PairWalk {
    int mt, nt, t;
    __device__ __forceinline__ void start(const TileParams& p) {
        const int pid = blockIdx.x >> 1;
        if (p.n_per) {
            mt = pid % p.m_tiles;
            nt = pid / p.m_tiles;
        } else {
            t = pid;
            mt = t % p.m_tiles;
            nt = t / p.m_tiles;
        }
    }
    __device__ __forceinline__ bool valid(const TileParams& p) const {
        return p.n_per ? nt < p.n_tiles : t < p.tiles;
    }
    __device__ __forceinline__ void next(const TileParams& p) {
        if (p.n_per) {
            nt += p.n_per;
        } else {
            t += gridDim.x >> 1;
            mt = t % p.m_tiles;
            nt = t / p.m_tiles;
        }
    }
};

constexpr int kTagPEmpty = 0x61, kTagPFull = 0x62, kTagPAccFull = 0x63, kTagPAccEmpty = 0x64,
              kTagPDrainLoad = 0x65, kTagPDrainMma = 0x66;

// KF >= 0: the fused steps fixed at compile time (the prompt pass's combinations); -1: read
// from flags.
template <int KF>
__global__ void __launch_bounds__(kTThreads, 1)
    gemm_pair_kernel(const __grid_constant__ CUtensorMap tmX, const __grid_constant__ CUtensorMap tmW,
                     const TileParams p) {
    extern __shared__ uint8_t smem_raw[];
    const uint32_t raw = smem_u32(smem_raw);
    uint8_t* base = smem_raw + (((raw + 1023u) & ~1023u) - raw);
    uint8_t* sA = base;                          // stage i at sA + i * kPABytes
    uint8_t* sB = base + kPStages * kPABytes;    // stage i at sB + i * kPBBytes
    PairTail* tail = reinterpret_cast<PairTail*>(sB + kPStages * kPBBytes);
    const int warp = threadIdx.x >> 5;
    const int lane = threadIdx.x & 31;
    const int flags = KF >= 0 ? KF : p.flags;
    const uint32_t rank = cluster_ctarank() & 1u;  // cluster = one pair
    const bool leader = rank == 0;

    if (threadIdx.x == 0) {
        for (int i = 0; i < kPStages; ++i) {
            mbar_init(&tail->full[i], 1);
            mbar_init(&tail->empty[i], 1);
        }
        for (int i = 0; i < 2; ++i) {
            mbar_init(&tail->acc_full[i], 1);
            mbar_init(&tail->acc_empty[i], 8);
        }
        mbar_init(&tail->drain, 1);
        tail->abort = 0;
        fence_mbar_init();
    }
    if (warp == 0 && lane == 0) {
        prefetch_tmap(&tmX);
        prefetch_tmap(&tmW);
    }
    if (warp == 1) {
        tmem_alloc_pair(&tail->tmem, kTTmemCols);
        tmem_relinquish_pair();
    }
    tc_fence_before();
    __syncthreads();
    // Both CTAs' barriers are initialised before either signals the other's.
    cluster_arrive();
    cluster_wait();
    tc_fence_after();
    const uint32_t tmem = tail->tmem;
    volatile int* abort_flag = &tail->abort;
    // Programmatic dependent launch, as in gemm_tile_kernel.
    griddep_launch_dependents();
    griddep_wait();

    if (warp == 0) {
        // ------------------------------------------------------------------ TMA producer
        if (lane == 0) {
            int it = 0;  // running k-block count of this pair: stage it % kPStages
            bool ok = true;
            PairWalk tw;
            for (tw.start(p); ok && tw.valid(p); tw.next(p)) {
                const int m0 = tw.mt * (2 * kTBM) + (int)rank * kTBM;
                const int n0 = tw.nt * kTBN + (int)rank * (kTBN / 2);
                for (int kb = 0; kb < p.kb_total; ++kb, ++it) {
                    const int st = it % kPStages;
                    if (it >= kPStages &&
                        !(ok = mbar_wait_cl(&tail->empty[st], ((it / kPStages) - 1) & 1,
                                            abort_flag, p.status, kTagPEmpty)))
                        break;
                    const uint32_t full0 = map_shared_rank_u32(smem_u32(&tail->full[st]), 0);
                    if (leader) mbar_arrive_expect_tx(&tail->full[st], 2 * (kPABytes + kPBBytes));
                    tma_load_2d_pair(sA + st * kPABytes, &tmX, full0, kb * kTileK, m0);
                    tma_load_2d_pair(sB + st * kPBBytes, &tmW, full0, kb * kTileK, n0);
                }
            }
            // The even CTA's full barriers count both CTAs' copies: before the pair leaves,
            // the last stages' copies must have landed (on the normal path the MMAs already
            // waited for them and these waits return at once).
            if (leader)
                for (int i = max(it - kPStages, 0); i < it; ++i)
                    mbar_wait_drain(&tail->full[i % kPStages], (i / kPStages) & 1, p.status,
                                    kTagPDrainLoad);
        }
        __syncwarp();
    } else if (warp == 1) {
        // ------------------------------------------------------------------ MMA issuer
        if (leader) {
            const uint32_t idesc = idesc_bf16_f32(2 * kTBM, kTBN, false);  // both K-major
            const uint64_t dA0 = smem_desc_sw128(smem_u32(sA), 16, 1024);
            const uint64_t dB0 = smem_desc_sw128(smem_u32(sB), 16, 1024);
            bool ok = true;
            int it = 0, lt = 0;
            PairWalk tw;
            for (tw.start(p); ok && tw.valid(p); tw.next(p), ++lt) {
                const int buf = lt & 1;
                // Free once all eight epilogue warps read the tile before last.
                if (lt >= 2 &&
                    !(ok = __all_sync(0xFFFFFFFFu,
                                      mbar_wait_cl(&tail->acc_empty[buf], ((lt >> 1) - 1) & 1,
                                                   abort_flag, p.status, kTagPAccEmpty))))
                    break;
                tc_fence_after();
                const uint32_t acc = tmem + buf * kTBN;
                for (int kb = 0; kb < p.kb_total; ++kb, ++it) {
                    const int st = it % kPStages;
                    if (!(ok = __all_sync(0xFFFFFFFFu,
                                          mbar_wait(&tail->full[st], (it / kPStages) & 1,
                                                    abort_flag, p.status, kTagPFull))))
                        break;
                    tc_fence_after();
                    const uint64_t dA = dA0 + (uint64_t)(st * (kPABytes >> 4));
                    const uint64_t dB = dB0 + (uint64_t)(st * (kPBBytes >> 4));
#pragma unroll
                    for (int kk = 0; kk < 4; ++kk)  // 16 K-elements = 32 bytes per MMA
                        mma_pair_ss_warp(acc, dA + kk * 2, dB + kk * 2, idesc, (kb | kk) ? 1u : 0u);
                    const uint32_t e = smem_u32(&tail->empty[st]);
                    mma_pair_commit_warp(map_shared_rank_u32(e, 0));
                    mma_pair_commit_warp(map_shared_rank_u32(e, 1));
                }
                if (ok) {
                    const uint32_t a = smem_u32(&tail->acc_full[buf]);
                    mma_pair_commit_warp(map_shared_rank_u32(a, 0));
                    mma_pair_commit_warp(map_shared_rank_u32(a, 1));
                }
            }
            // Leave only once every MMA issued above has completed: the TMEM of both CTAs is
            // released after the closing cluster barrier.
            mma_pair_commit_warp(map_shared_rank_u32(smem_u32(&tail->drain), 0));
            mbar_wait_drain(&tail->drain, 0, p.status, kTagPDrainMma);
        }
        __syncwarp();
    } else {
        // ------------------------------------------------------------------ epilogue
        const int quarter = warp & 3;
        const int r = quarter * 32 + lane;  // the CTA-tile row (TMEM lane) this thread owns
        const uint32_t lane_base = static_cast<uint32_t>(quarter * 32) << 16;
        int lt = 0;
        float rs = 1.f;
        PairWalk tw;
        for (tw.start(p); tw.valid(p); tw.next(p), ++lt) {
            const int buf = lt & 1;
            const int mrow0 = tw.mt * (2 * kTBM) + (int)rank * kTBM;  // this CTA's first row
            const int m = mrow0 + r;
            const int n0 = tw.nt * kTBN;
            // RMSNorm scale of the warp's 32 rows, while the tile's MMAs run; a pair that keeps
            // one row block computes them once.
            if ((flags & NC_GEMM_NORM_INPUT) && (lt == 0 || !p.n_per)) {
                row_scales_warp(p.x, p.M, p.K, mrow0 + quarter * 32, 1, 32, lane,
                                tail->rs + quarter * 32);
                __syncwarp();
                rs = tail->rs[quarter * 32 + lane];
                __syncwarp();
            }
            auto load_res = [&](int c, uint4 (&r)[4]) {
#pragma unroll
                for (int g8 = 0; g8 < 4; ++g8) {
                    const int n = n0 + 32 * c + 8 * g8;
                    r[g8] = ((flags & NC_GEMM_RESIDUAL) && m < p.M && n < p.N)
                                ? *reinterpret_cast<const uint4*>(p.residual + (size_t)m * p.N + n)
                                : make_uint4(0u, 0u, 0u, 0u);
                }
            };
            // With a residual known at compile time, this thread's whole residual row segment
            // (8 chunks x 32 columns, 128 registers) is loaded before the accumulator wait, so
            // its latency hides behind the tile's MMAs.  The residual is an input of the kernel
            // (read after griddepcontrol.wait) and each element is read and then written by the
            // one thread that owns it, so the early loads are safe when out == residual.
            constexpr bool kPreload = KF >= 0 && (KF & NC_GEMM_RESIDUAL) != 0;
            uint4 rall[kPreload ? kTBN / 32 : 1][4];
            if constexpr (kPreload) {
#pragma unroll
                for (int c = 0; c < kTBN / 32; ++c) load_res(c, rall[c]);
            }
            if (!__all_sync(0xFFFFFFFFu, mbar_wait_cl(&tail->acc_full[buf], (lt >> 1) & 1,
                                                      abort_flag, p.status, kTagPAccFull)))
                break;
            tc_fence_after();
            // One 32-column chunk: read it from TMEM (the last chunk also frees the buffer),
            // apply the fused steps and store.
            auto do_chunk = [&](int c, const uint4 (&rcur)[4]) {
                uint32_t v[32];
                tmem_ld32_sync(tmem + buf * kTBN + 32 * c + lane_base, v);
                if (c == kTBN / 32 - 1) {
                    // This warp has read every column of the buffer: one arrival on the even
                    // CTA's barrier, which frees the buffer once all eight warps have arrived.
                    tc_fence_before();
                    __syncwarp();
                    if (lane == 0)
                        mbar_arrive_cluster(map_shared_rank_u32(smem_u32(&tail->acc_empty[buf]), 0));
                }
                if (m >= p.M) return;
#pragma unroll
                for (int g8 = 0; g8 < 4; ++g8) {
                    const int n = n0 + 32 * c + 8 * g8;
                    if (n >= p.N) break;
                    float f[8];
#pragma unroll
                    for (int e = 0; e < 8; ++e) f[e] = __uint_as_float(v[8 * g8 + e]);
                    if (flags & NC_GEMM_NORM_INPUT) {
#pragma unroll
                        for (int e = 0; e < 8; ++e) f[e] *= rs;
                    }
                    if (flags & NC_GEMM_RESIDUAL) {
                        float rr[8];
                        bf16x8_to_f32(rcur[g8], rr);
#pragma unroll
                        for (int e = 0; e < 8; ++e) f[e] += rr[e];
                    }
                    if (flags & NC_GEMM_RELU2) {
#pragma unroll
                        for (int e = 0; e < 8; ++e) {
                            const float y = fmaxf(f[e], 0.f);
                            f[e] = y * y;
                        }
                    }
                    if (flags & NC_GEMM_TANH_CAP) {
#pragma unroll
                        for (int e = 0; e < 8; ++e) f[e] = p.cap * tanhf(f[e] / p.cap);
                    }
                    const int seg = p.seg_cols;
                    bf16* dst = p.out + (size_t)(n / seg) * ((size_t)p.M * seg) + (size_t)m * seg +
                                (n % seg);
                    *reinterpret_cast<uint4*>(dst) = f32_to_bf16x8(f);
                }
            };
            if constexpr (kPreload) {
#pragma unroll
                for (int c = 0; c < kTBN / 32; ++c) do_chunk(c, rall[c]);
            } else {
                // The residual of the first chunk, then each next chunk's ahead of this one's
                // work: its loads are in flight while this chunk is read from TMEM and stored.
                uint4 rnext[4];
                load_res(0, rnext);
                for (int c = 0; c < kTBN / 32; ++c) {
                    uint4 rcur[4];
#pragma unroll
                    for (int g8 = 0; g8 < 4; ++g8) rcur[g8] = rnext[g8];
                    if (c + 1 < kTBN / 32) load_res(c + 1, rnext);
                    do_chunk(c, rcur);
                }
            }
        }
    }

    tc_fence_before();
    __syncthreads();
    // Neither CTA releases its tensor memory or leaves while the pair may still signal it.
    cluster_arrive();
    cluster_wait();
    if (warp == 1) {
        tc_fence_after();
        tmem_dealloc_pair(tmem, kTTmemCols);
    }
}

// ---------------------------------------------------------------------------------------
// host side
// ---------------------------------------------------------------------------------------
using EncodeTiledFn = CUresult (*)(CUtensorMap*, CUtensorMapDataType, cuuint32_t, void*,
                                   const cuuint64_t*, const cuuint64_t*, const cuuint32_t*,
                                   const cuuint32_t*, CUtensorMapInterleave, CUtensorMapSwizzle,
                                   CUtensorMapL2promotion, CUtensorMapFloatOOBfill);

EncodeTiledFn encode_fn() {
    static EncodeTiledFn fn = [] {
        void* f = nullptr;
        cudaDriverEntryPointQueryResult q{};
        if (cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &f, cudaEnableDefault, &q) !=
                cudaSuccess ||
            q != cudaDriverEntryPointSuccess)
            return static_cast<EncodeTiledFn>(nullptr);
        return reinterpret_cast<EncodeTiledFn>(f);
    }();
    return fn;
}

// Row-major [rows][cols] bf16 matrix, box of 64 columns x box_rows rows, 128-byte swizzle;
// rows and columns beyond the matrix read as zero.
struct Map2DKey {
    const void* base;
    int rows, cols, box_rows, dev;
    bool operator==(const Map2DKey& o) const {
        return base == o.base && rows == o.rows && cols == o.cols && box_rows == o.box_rows &&
               dev == o.dev;
    }
};
struct Map2DEntry {
    Map2DKey key;
    CUtensorMap map;
    bool used;
};
std::mutex g_map2d_mutex;
Map2DEntry g_map2d[512];

bool map_2d(CUtensorMap* m, const void* base, int rows, int cols, int box_rows, int dev) {
    const Map2DKey key{base, rows, cols, box_rows, dev};
    size_t h = reinterpret_cast<uintptr_t>(base) >> 8;
    h ^= (size_t)rows * 0x9E3779B1u ^ (size_t)cols * 0x85EBCA6Bu ^
         (size_t)box_rows * 0xC2B2AE35u ^ (size_t)dev * 0x27D4EB2Fu;
    h ^= h >> 13;
    Map2DEntry& e = g_map2d[h & 511];
    {
        std::lock_guard<std::mutex> lk(g_map2d_mutex);
        if (e.used && e.key == key) {
            *m = e.map;
            return true;
        }
    }
    EncodeTiledFn enc = encode_fn();
    if (!enc) return false;
    const cuuint64_t dims[2] = {(cuuint64_t)cols, (cuuint64_t)rows};
    const cuuint64_t strides[1] = {(cuuint64_t)cols * 2};
    const cuuint32_t box[2] = {(cuuint32_t)kTileK, (cuuint32_t)box_rows};
    const cuuint32_t estr[2] = {1, 1};
    if (enc(m, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 2, const_cast<void*>(base), dims, strides, box,
            estr, CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B,
            CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
            CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE) != CUDA_SUCCESS)
        return false;
    std::lock_guard<std::mutex> lk(g_map2d_mutex);
    e.key = key;
    e.map = *m;
    e.used = true;
    return true;
}

constexpr int kMaxDev = 64;

struct GemmPlan {
    int n_tiles, kb_total, kb_per, splits;
};

// Split count: aim for about two CTAs per SM of a B200 (148 SMs) over the whole grid (each SM
// then keeps two CTAs' rings, 192 KB of weight, in flight), at most kMaxSplits (one cluster
// per output tile); `req` > 0 sets it instead (clamped the same way).
constexpr int kPlanSMs = 148;
GemmPlan plan_gemm(int N, int K, int req) {
    GemmPlan g;
    g.n_tiles = (N + kTileN - 1) / kTileN;
    g.kb_total = (K + kTileK - 1) / kTileK;
    int s = req > 0 ? req : std::max(1, (2 * kPlanSMs) / g.n_tiles);
    s = std::min(std::min(s, kMaxSplits), g.kb_total);
    g.kb_per = (g.kb_total + s - 1) / s;
    g.splits = (g.kb_total + g.kb_per - 1) / g.kb_per;  // no empty split
    return g;
}

template <int MP>
cudaError_t launch_mp(const CUtensorMap& mw, const CUtensorMap& mx, const GemmParams& p,
                      const GemmPlan& g, int dev, cudaStream_t stream) {
    static bool attr_set[kMaxDev] = {};
    if (!attr_set[dev]) {
        cudaError_t e = cudaFuncSetAttribute(gemm_skinny_kernel<MP>,
                                             cudaFuncAttributeMaxDynamicSharedMemorySize,
                                             gemm_smem_bytes<MP>());
        if (e == cudaSuccess)  // clusters above 8 CTAs (the portable limit)
            e = cudaFuncSetAttribute(gemm_skinny_kernel<MP>,
                                     cudaFuncAttributeNonPortableClusterSizeAllowed, 1);
        if (e != cudaSuccess) return e;
        attr_set[dev] = true;
    }
    cudaLaunchConfig_t cfg = {};
    cfg.gridDim = dim3((unsigned)g.n_tiles, (unsigned)g.splits);
    cfg.blockDim = dim3(kGemmThreads);
    cfg.dynamicSmemBytes = gemm_smem_bytes<MP>();
    cfg.stream = stream;
    cudaLaunchAttribute attr[2];
    attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
    attr[0].val.programmaticStreamSerializationAllowed = 1;
    attr[1].id = cudaLaunchAttributeClusterDimension;
    attr[1].val.clusterDim.x = 1;
    attr[1].val.clusterDim.y = (unsigned)g.splits;
    attr[1].val.clusterDim.z = 1;
    cfg.attrs = attr;
    cfg.numAttrs = 2;
    return cudaLaunchKernelEx(&cfg, gemm_skinny_kernel<MP>, mw, mx, p);
}

bool overlaps(const void* a, size_t an, const void* b, size_t bn) {
    const uintptr_t x = reinterpret_cast<uintptr_t>(a), y = reinterpret_cast<uintptr_t>(b);
    return x < y + bn && y < x + an;
}

cudaError_t set_pair_smem() {
    cudaError_t e = cudaSuccess;
    const void* fns[4] = {(const void*)gemm_pair_kernel<-1>,
                          (const void*)gemm_pair_kernel<NC_GEMM_NORM_INPUT>,
                          (const void*)gemm_pair_kernel<NC_GEMM_RESIDUAL>,
                          (const void*)gemm_pair_kernel<NC_GEMM_NORM_INPUT | NC_GEMM_RELU2>};
    for (const void* f : fns)
        if (e == cudaSuccess)
            e = cudaFuncSetAttribute(f, cudaFuncAttributeMaxDynamicSharedMemorySize, kPSmemBytes);
    return e;
}

}  // namespace

}  // namespace nc

extern "C" {

int nc_gemm_skinny(void* out, const void* x, const void* w, const void* residual, int M, int N,
                   int K, int flags, float cap, int seg_cols, int splits, cudaStream_t stream) {
    using namespace nc;
    if (M < 1 || M > kMaxRows || N < 1 || K < 8 || (K & 7) || splits < 0) return NC_ERR_INVALID_ARG;
    if (flags & ~(NC_GEMM_NORM_INPUT | NC_GEMM_RESIDUAL | NC_GEMM_RELU2 | NC_GEMM_TANH_CAP))
        return NC_ERR_INVALID_ARG;
    if (!out || !x || !w || ((flags & NC_GEMM_RESIDUAL) && !residual)) return NC_ERR_INVALID_ARG;
    if ((flags & NC_GEMM_TANH_CAP) && !(cap > 0.f)) return NC_ERR_INVALID_ARG;
    if (seg_cols == 0) seg_cols = N;
    if (seg_cols < 1 || N % seg_cols) return NC_ERR_INVALID_ARG;
    if ((reinterpret_cast<uintptr_t>(x) & 15) || (reinterpret_cast<uintptr_t>(w) & 15) ||
        (reinterpret_cast<uintptr_t>(out) & 1) || (reinterpret_cast<uintptr_t>(residual) & 1))
        return NC_ERR_MISALIGNED;
    if (overlaps(out, (size_t)M * N * 2, x, (size_t)M * K * 2)) return NC_ERR_INVALID_ARG;
    if ((flags & NC_GEMM_RESIDUAL) && residual != out &&
        overlaps(out, (size_t)M * N * 2, residual, (size_t)M * N * 2))
        return NC_ERR_INVALID_ARG;
    int dev = 0;
    cudaError_t e = cudaGetDevice(&dev);
    if (e != cudaSuccess) return internal_cuda_fail(e);
    if (dev < 0 || dev >= kMaxDev) return NC_ERR_INVALID_ARG;
    int* status = nullptr;
    int st = internal_status_word(&status);
    if (st) return st;

    const GemmPlan g = plan_gemm(N, K, splits);
    const int mp = M <= 16 ? 16 : (M <= 32 ? 32 : 64);
    CUtensorMap mw, mx;
    if (!map_2d(&mw, w, N, K, kTileN, dev) || !map_2d(&mx, x, M, K, mp, dev))
        return NC_ERR_INVALID_ARG;
    GemmParams p;
    p.out = static_cast<bf16*>(out);
    p.x = static_cast<const bf16*>(x);
    p.residual = static_cast<const bf16*>(residual);
    p.M = M;
    p.N = N;
    p.K = K;
    p.kb_total = g.kb_total;
    p.kb_per = g.kb_per;
    p.splits = g.splits;
    p.flags = flags;
    p.cap = cap;
    p.seg_cols = seg_cols;
    p.status = status;
    if (mp == 16) e = launch_mp<16>(mw, mx, p, g, dev, stream);
    else if (mp == 32) e = launch_mp<32>(mw, mx, p, g, dev, stream);
    else e = launch_mp<64>(mw, mx, p, g, dev, stream);
    return e == cudaSuccess ? NC_OK : internal_cuda_fail(e);
}

int nc_gemm(void* out, const void* x, const void* w, const void* residual, int M, int N, int K,
            int flags, float cap, int seg_cols, cudaStream_t stream) {
    using namespace nc;
    if (M < 1 || N < 8 || (N & 7) || K < 8 || (K & 7)) return NC_ERR_INVALID_ARG;
    if (flags & ~(NC_GEMM_NORM_INPUT | NC_GEMM_RESIDUAL | NC_GEMM_RELU2 | NC_GEMM_TANH_CAP))
        return NC_ERR_INVALID_ARG;
    if (!out || !x || !w || ((flags & NC_GEMM_RESIDUAL) && !residual)) return NC_ERR_INVALID_ARG;
    if ((flags & NC_GEMM_TANH_CAP) && !(cap > 0.f)) return NC_ERR_INVALID_ARG;
    if (seg_cols == 0) seg_cols = N;
    if (seg_cols < 8 || (seg_cols & 7) || N % seg_cols) return NC_ERR_INVALID_ARG;
    if ((reinterpret_cast<uintptr_t>(x) & 15) || (reinterpret_cast<uintptr_t>(w) & 15) ||
        (reinterpret_cast<uintptr_t>(out) & 15) || (reinterpret_cast<uintptr_t>(residual) & 15))
        return NC_ERR_MISALIGNED;
    if (overlaps(out, (size_t)M * N * 2, x, (size_t)M * K * 2)) return NC_ERR_INVALID_ARG;
    if ((flags & NC_GEMM_RESIDUAL) && residual != out &&
        overlaps(out, (size_t)M * N * 2, residual, (size_t)M * N * 2))
        return NC_ERR_INVALID_ARG;
    int dev = 0;
    cudaError_t e = cudaGetDevice(&dev);
    if (e != cudaSuccess) return internal_cuda_fail(e);
    if (dev < 0 || dev >= kMaxDev) return NC_ERR_INVALID_ARG;
    int* status = nullptr;
    int st = internal_status_word(&status);
    if (st) return st;
    static bool attr_set[kMaxDev] = {};
    static int sms[kMaxDev] = {};
    static int pairs_max[kMaxDev] = {};
    cudaLaunchAttribute attr[2];
    attr[0].id = cudaLaunchAttributeClusterDimension;
    attr[0].val.clusterDim.x = 2;
    attr[0].val.clusterDim.y = 1;
    attr[0].val.clusterDim.z = 1;
    cudaLaunchConfig_t cfg = {};
    cfg.blockDim = dim3(kTThreads);
    cfg.dynamicSmemBytes = kPSmemBytes;
    cfg.stream = stream;
    cfg.attrs = attr;
    cfg.numAttrs = 1;
    if (!attr_set[dev]) {
        e = cudaFuncSetAttribute(gemm_tile_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                 kTSmemBytes);
        if (e == cudaSuccess)
            e = set_pair_smem();
        if (e == cudaSuccess)
            e = cudaDeviceGetAttribute(&sms[dev], cudaDevAttrMultiProcessorCount, dev);
        // Pairs that can be resident at once: a pair needs two SMs of one GPC, so an odd SM
        // count per GPC leaves SMs that no pair can use.  More pairs than this would make a
        // second wave.
        if (e == cudaSuccess) {
            cfg.gridDim = dim3(2);
            e = cudaOccupancyMaxActiveClusters(&pairs_max[dev], gemm_pair_kernel<-1>, &cfg);
        }
        if (e != cudaSuccess) return internal_cuda_fail(e);
        attr_set[dev] = true;
    }
    // More than one 128-row block: CTA pairs on 256 x 256 tiles.
    const bool pair = M > kTBM;
    const int bm = pair ? 2 * kTBM : kTBM;
    CUtensorMap mx, mw;
    if (!map_2d(&mx, x, M, K, kTBM, dev) || !map_2d(&mw, w, N, K, pair ? kTBN / 2 : kTBN, dev))
        return NC_ERR_INVALID_ARG;
    TileParams p;
    p.out = static_cast<bf16*>(out);
    p.x = static_cast<const bf16*>(x);
    p.residual = static_cast<const bf16*>(residual);
    p.M = M;
    p.N = N;
    p.K = K;
    p.kb_total = (K + kTileK - 1) / kTileK;
    p.m_tiles = (M + bm - 1) / bm;
    p.n_tiles = (N + kTBN - 1) / kTBN;
    p.tiles = p.m_tiles * p.n_tiles;
    // With at most one row block per worker (a CTA, or a pair), each worker keeps a row block
    // (its RMSNorm scales are computed once) and the workers are a whole number per row block.
    const int workers = pair ? std::max(1, std::min(sms[dev] / 2, pairs_max[dev])) : sms[dev];
    p.n_per = p.m_tiles <= workers ? std::min(p.n_tiles, workers / p.m_tiles) : 0;
    p.flags = flags;
    p.cap = cap;
    p.seg_cols = seg_cols;
    p.status = status;
    const unsigned used =
        (unsigned)(p.n_per ? p.m_tiles * p.n_per : std::min(p.tiles, workers));
    // Both kernels are launched as programmatic dependents of the previous kernel in the stream.
    attr[1].id = cudaLaunchAttributeProgrammaticStreamSerialization;
    attr[1].val.programmaticStreamSerializationAllowed = 1;
    if (!pair) {
        cudaLaunchConfig_t tcfg = {};
        tcfg.gridDim = dim3(used);
        tcfg.blockDim = dim3(kTThreads);
        tcfg.dynamicSmemBytes = kTSmemBytes;
        tcfg.stream = stream;
        tcfg.attrs = &attr[1];
        tcfg.numAttrs = 1;
        e = cudaLaunchKernelEx(&tcfg, gemm_tile_kernel, mx, mw, p);
        return e == cudaSuccess ? NC_OK : internal_cuda_fail(e);
    }
    cfg.numAttrs = 2;
    cfg.gridDim = dim3(2 * used);
    switch (flags) {
        case NC_GEMM_NORM_INPUT:
            e = cudaLaunchKernelEx(&cfg, gemm_pair_kernel<NC_GEMM_NORM_INPUT>, mx, mw, p);
            break;
        case NC_GEMM_RESIDUAL:
            e = cudaLaunchKernelEx(&cfg, gemm_pair_kernel<NC_GEMM_RESIDUAL>, mx, mw, p);
            break;
        case NC_GEMM_NORM_INPUT | NC_GEMM_RELU2:
            e = cudaLaunchKernelEx(&cfg, gemm_pair_kernel<NC_GEMM_NORM_INPUT | NC_GEMM_RELU2>, mx,
                                   mw, p);
            break;
        default:
            e = cudaLaunchKernelEx(&cfg, gemm_pair_kernel<-1>, mx, mw, p);
    }
    return e == cudaSuccess ? NC_OK : internal_cuda_fail(e);
}

}  // extern "C"

// Causal prefill attention on the 5th-generation tensor cores (tcgen05 + tensor memory),
// with Q/K/V tiles staged in shared memory by TMA.
//
// Replaces the seq_q > 1 use of reference kernels/flash_attention.cu:19-171, which runs one
// 128-thread CTA per (query, head) on CUDA cores and walks every key up to kv_len.
//
// Work unit ("tile"): 128 query rows x one head x one sequence.  Keys are consumed in blocks
// of 128; only blocks that hold a visible key are visited (causal rule
// key <= query + kv_offset and key < kv_len, reference flash_attention.cu:37, :74).
// Persistent schedule: one CTA per SM walks a fixed list of tiles.  Tiles are ranked longest
// first and dealt out in a zigzag (CTA c takes ranks c, 2G-1-c, 2G+c, ...), which evens out
// the per-CTA sum of key blocks.  A running block counter drives every ring across tile
// boundaries, and the Q tile is double-buffered, so the next tile's loads and first QK MMAs
// overlap the current tile's last blocks and epilogue.
//
// Roles (320 threads, one CTA per SM):
//   warp 0      TMA producers: lane 0 K(j) into a two-stage ring, lane 1 V(j) into a
//               two-stage ring, lane 2 each tile's Q (two buffers).
//   warp 1      allocates all 512 TMEM columns; one lane issues every tcgen05.mma.
//   warps 2..9  softmax / epilogue, two warps per TMEM lane quarter (warp w owns query rows
//               32 * (w % 4) .. + 31 = its TMEM lanes): warps 2..5 take keys [0, 64) of every
//               block ("half A"), warps 6..9 keys [64, 128) ("half B").  Each half keeps its own
//               running max, row sum and output accumulator, so the two warps of a quarter never
//               wait for each other inside a tile; they merge once, in the tile's epilogue.
//               Two softmax warps per SMSP hide each other's latencies.
// Tensor memory (512 columns): S0 [0,128) and S1 [128,256) hold Q.K^T of consecutive key
// blocks (fp32); O_A [256,384) and O_B [384,512) accumulate P.V of the two key halves (fp32).
// Once a half has read its 64 S columns it writes its bf16 probabilities (two per column) over
// the first 32 of them, where the P.V MMA reads them straight from TMEM.
// Pipeline: the MMA warp keeps QK two blocks ahead of the softmax, so while the softmax of
// block j+1 runs, the tensor pipe executes PV(j) and QK(j+2); the softmax warps go from one
// block to the next without waiting for the tensor pipe.
//
// Softmax: fp32, base-2 exponentials of scale*log2(e)-scaled scores, with a lazily updated
// reference max: O and the row sum are rescaled only when a block's max exceeds the
// reference by more than 8 (log2 units).  The reference starts at the bound on the scores of
// RMS-normalised q and k, so a tile's first block needs no max pass either.  Rows without any visible key produce NaN, as the
// reference's 0/0 does.
#include <cuda.h>

#include <algorithm>
#include <mutex>

#include "nc_common.cuh"
#include "sm100_ptx.cuh"

namespace nc {

namespace {

constexpr int kBM = 128;             // query rows per CTA
constexpr int kBN = 128;             // keys per block
constexpr int kThreads = 320;      // producer warp, MMA warp, eight softmax warps
constexpr uint32_t kBoxBytes = 64 * 128 * 2;    // one 64-dim x 128-row box, 128B swizzle
constexpr uint32_t kTileBytes = 2 * kBoxBytes;  // 128 x 128 bf16
constexpr uint32_t kTmemCols = 512;
constexpr uint32_t kColS = 0;        // S0 at 0, S1 at 128; half h's P over [64h, 64h + 32) of S
constexpr uint32_t kColOA = 256;     // O of key half A
constexpr uint32_t kColOB = 384;     // O of key half B
constexpr float kRescaleThreshold = 8.0f;
// A tile's first block is accepted on the optimistic path only if its row sum is at least this
// (below it the starting reference was far above the real max; the exact path resets it).
constexpr float kMinFirstSum = 5.421010862427522e-20f;  // 2^-64
constexpr float kNegInf = -__builtin_huge_valf();

enum Bar : int {
    kBarQ = 0,   // [2] Q buffer full
    kBarQFree = kBarQ + 2,  // [2] every QK of the tile that used the Q buffer is done
    kBarKFull = kBarQFree + 2,   // [2]
    kBarVFull = kBarKFull + 2,   // [2]
    kBarS = kBarVFull + 2,       // [2] QK(g) done: S(g & 1) full and K stage g & 1 free
    kBarP = kBarS + 2,           // [2] both halves wrote P(g) (256 arrivals)
    kBarPV = kBarP + 2,          // [2] PV(g) done: V stage free, P(g & 1) free
    kBarOFinal = kBarPV + 2,
    kBarXch = kBarOFinal + 1,    // [4] per lane quarter: both halves posted (max, sum) (64)
    kBarXrd = kBarXch + 4,       // [4] per lane quarter: both halves read the other's (64)
    kBarDrain = kBarXrd + 4,     // the MMA warp's last commit: every MMA it issued is done
    kNumBars
};

struct __align__(8) SmemTail {
    uint64_t bars[kNumBars];
    float2 xch[4][2][32];  // per lane quarter and key half: each row's (max, sum) at the epilogue
    uint32_t tmem_base;
    int abort;
};

// Two Q buffers + two K stages + two V stages + the output staging tile.
constexpr uint32_t kStageOutBytes = 128 * 128 * 2;  // 4 warps x (32 rows x 256 B)
// No alignment slack: the dynamic shared memory window starts 1024-byte aligned (checked at
// kernel entry), which the 128B-swizzled tiles need.
constexpr size_t kSmemBytes = 6 * kTileBytes + kStageOutBytes + sizeof(SmemTail);
static_assert(kSmemBytes <= 227 * 1024, "shared memory budget");

struct PrefillKParams {
    bf16* out;
    const int* kv_offset_dev;
    int kv_offset;
    int kv_len;
    int kv_len_from_offset;  // batched mode: kv_len_b = kv_offset_b + seq_q
    int batch;
    int seq_q;
    int heads;
    int n_qtiles;
    int total_tiles;
    float scale_log2;
    int* status;
    const int* page_table;  // paged K/V (see PrefillArgs); null: per-sequence caches
    int page_rows, pages_per_seq, num_pages;
};

// One tile of work: its coordinates and how many key blocks it visits.
struct Tile {
    int h, b, q0, off, kv_len, nb;
};

__device__ __forceinline__ Tile make_tile(const PrefillKParams& p, int rank) {
    const int groups = p.heads * p.batch;
    const int r = rank / groups;
    const int g = rank - r * groups;
    Tile t;
    t.h = g % p.heads;
    t.b = g / p.heads;
    t.q0 = (p.n_qtiles - 1 - r) * kBM;  // rank 0 = last (longest) query tile
    t.off = p.kv_offset_dev ? p.kv_offset_dev[t.b] : p.kv_offset;
    t.kv_len = p.kv_len_from_offset ? t.off + p.seq_q : p.kv_len;
    const int q_last = min(t.q0 + kBM - 1, p.seq_q - 1);
    const int kv_end = min(t.kv_len, q_last + t.off + 1);  // keys [0, kv_end) may be visible
    t.nb = kv_end > 0 ? (kv_end + kBN - 1) / kBN : 0;
    return t;
}

// Rank of the k-th tile of CTA c out of G: c, 2G-1-c, 2G+c, 4G-1-c, ...
__device__ __forceinline__ int tile_rank(int k, int c, int G) {
    const int base = (k >> 1) * 2 * G;
    return (k & 1) ? base + 2 * G - 1 - c : base + c;
}

// Walks the key blocks of this CTA's non-empty tiles in order (used two blocks ahead by the
// MMA issuer for its QK lookahead).
struct BlockCursor {
    int k, j, qi;  // tile index in the CTA's list, block in the tile, non-empty-tile counter
    Tile t;
    bool valid;
};

__device__ __forceinline__ void cursor_seek(BlockCursor& c, const PrefillKParams& p) {
    // from tile index c.k (block 0), skip empty tiles
    for (;; ++c.k) {
        const int rank = tile_rank(c.k, blockIdx.x, gridDim.x);
        if (rank >= p.total_tiles) {
            c.valid = false;
            return;
        }
        c.t = make_tile(p, rank);
        if (c.t.nb > 0) {
            c.j = 0;
            c.valid = true;
            return;
        }
    }
}

__device__ __forceinline__ void cursor_next(BlockCursor& c, const PrefillKParams& p) {
    if (++c.j < c.t.nb) return;
    ++c.k;
    ++c.qi;
    cursor_seek(c, p);
}

__device__ __forceinline__ void tma_load_3d(void* smem_dst, const CUtensorMap* tmap, uint64_t* bar,
                                            int x, int y, int z) {
    asm volatile(
        "cp.async.bulk.tensor.3d.shared::cluster.global.mbarrier::complete_tx::bytes"
        " [%0], [%1, {%3, %4, %5}], [%2];" ::"r"(smem_u32(smem_dst)),
        "l"(reinterpret_cast<uint64_t>(tmap)), "r"(smem_u32(bar)), "r"(x), "r"(y), "r"(z)
        : "memory");
}

__device__ __forceinline__ void tma_store_3d(const CUtensorMap* tmap, const void* smem_src, int x,
                                             int y, int z) {
    asm volatile(
        "cp.async.bulk.tensor.3d.global.shared::cta.bulk_group [%0, {%2, %3, %4}], [%1];" ::"l"(
            reinterpret_cast<uint64_t>(tmap)),
        "r"(smem_u32(smem_src)), "r"(x), "r"(y), "r"(z)
        : "memory");
}
__device__ __forceinline__ void bulk_commit() { asm volatile("cp.async.bulk.commit_group;" ::: "memory"); }
__device__ __forceinline__ void bulk_wait_read_all() {
    asm volatile("cp.async.bulk.wait_group.read 0;" ::: "memory");
}
__device__ __forceinline__ void bulk_wait_all() { asm volatile("cp.async.bulk.wait_group 0;" ::: "memory"); }

__global__ void __launch_bounds__(kThreads, 1)
    prefill_kernel(const __grid_constant__ CUtensorMap tmQ, const __grid_constant__ CUtensorMap tmK,
                   const __grid_constant__ CUtensorMap tmV, const __grid_constant__ CUtensorMap tmO,
                   const PrefillKParams p) {
    extern __shared__ __align__(1024) uint8_t smem_raw[];
    // The budget has no room to realign: a window that is not 1024-byte aligned is reported
    // and the kernel does nothing (uniform across the CTA, before any barrier or TMEM use).
    if (smem_u32(smem_raw) & 1023u) {
        if (threadIdx.x == 0) atomicOr(p.status, kStatusBounds);
        return;
    }
    uint8_t* smem = smem_raw;
    uint8_t* sQ = smem;                    // buffers at sQ, sQ + kTileBytes
    uint8_t* sK = smem + 2 * kTileBytes;   // stages at sK, sK + kTileBytes
    uint8_t* sV = smem + 4 * kTileBytes;   // stages at sV, sV + kTileBytes
    uint8_t* sO = smem + 6 * kTileBytes;   // output staging, 4 KB per softmax warp
    SmemTail* tail = reinterpret_cast<SmemTail*>(smem + 6 * kTileBytes + kStageOutBytes);
    uint64_t* bars = tail->bars;
    volatile int* abort_flag = &tail->abort;

    const int warp = threadIdx.x >> 5;
    const int lane = threadIdx.x & 31;

    if (threadIdx.x == 0) {
        for (int i = 0; i < kNumBars; ++i)
            mbar_init(&bars[i], (i == kBarP || i == kBarP + 1)         ? 256u
                                : (i >= kBarXch && i < kBarXrd + 4) ? 64u
                                                                    : 1u);
        tail->abort = 0;
        fence_mbar_init();
    }
    if (warp == 1) {
        tmem_alloc(&tail->tmem_base, kTmemCols);
        tmem_relinquish();
    }
    if (warp == 0 && lane == 0) {
        prefetch_tmap(&tmQ);
        prefetch_tmap(&tmK);
        prefetch_tmap(&tmV);
        prefetch_tmap(&tmO);
    }
    tc_fence_before();
    __syncthreads();
    tc_fence_after();
    const uint32_t tmem = tail->tmem_base;
    // The kernel is launched with programmatic stream serialization: everything above (barrier
    // init, TMEM allocation, tensor-map prefetch) may overlap the tail of the previous kernel
    // in the stream, typically the RoPE/append pass that writes Q, K and V.  No global memory
    // is read or written before this wait, which returns once that kernel has completed and
    // its writes are visible.
    asm volatile("griddepcontrol.wait;" ::: "memory");

    // Ring positions are driven by g, the running count of key blocks this CTA has visited
    // (stage g & 1, parity (g >> 1) & 1), and by qi, the running count of non-empty tiles
    // (Q buffer qi & 1, parity (qi >> 1) & 1).
    if (warp == 0) {
        // ------------------------------------------------------------------ producers
        // Lane 0 loads K, lane 1 loads V and lane 2 loads Q, each waiting only on the barrier
        // that frees its own ring: K(g+2) streams in as soon as QK(g) is done, V(g+2) once
        // PV(g) is, and a tile's Q as soon as its buffer's previous tile has finished its QKs
        // (up to two tiles ahead), so the next tile's first QK never waits behind K loads.
        if (lane < 3) {
            const bool kq = lane == 0;
            const bool qload = lane == 2;
            int g = 0, qi = 0;
            bool ok = true;
            for (int k = 0; ok; ++k) {
                const int rank = tile_rank(k, blockIdx.x, gridDim.x);
                if (rank >= p.total_tiles) break;
                const Tile t = make_tile(p, rank);
                if (t.nb == 0) continue;
                const int x0 = t.h * 128;
                if (qload) {
                    const int qb = qi & 1;
                    if (qi >= 2 && !(ok = mbar_wait(&bars[kBarQFree + qb], ((qi >> 1) - 1) & 1,
                                                    abort_flag, p.status, 1)))
                        break;
                    uint8_t* dq = sQ + qb * kTileBytes;
                    mbar_arrive_expect_tx(&bars[kBarQ + qb], kTileBytes);
                    tma_load_3d(dq, &tmQ, &bars[kBarQ + qb], x0, t.q0, t.b);
                    tma_load_3d(dq + kBoxBytes, &tmQ, &bars[kBarQ + qb], x0 + 64, t.q0, t.b);
                    ++qi;
                    continue;
                }
                for (int j = 0; j < t.nb; ++j, ++g) {
                    const int st = g & 1;
                    const uint32_t ph = ((g >> 1) - 1) & 1;  // previous use of stage st
                    // Key block j: rows [j*128, j*128 + 128) of sequence t.b, or, paged, of its
                    // page (a page holds a multiple of 128 rows).  The page id is read before
                    // the ring wait below so that its latency overlaps the wait.  A block past
                    // the sequence's pages or a page id outside the pool is flagged and loaded
                    // from an out-of-range row (TMA fills it with zeros).
                    int ky = j * kBN, kz = t.b;
                    if (p.page_table) {
                        const int pidx = (j * kBN) / p.page_rows;
                        const int page = pidx < p.pages_per_seq
                                             ? p.page_table[t.b * p.pages_per_seq + pidx]
                                             : -1;
                        kz = 0;
                        if (page < 0 || page >= p.num_pages) {
                            atomicOr(p.status, kStatusBounds);
                            ky = -kBN;
                        } else {
                            ky = page * p.page_rows + (j * kBN) % p.page_rows;
                        }
                    }
                    // K stage st is free once QK(g-2) completed (kBarS), V stage once PV(g-2) did.
                    if (g >= 2 && !(ok = mbar_wait(&bars[(kq ? kBarS : kBarPV) + st], ph, abort_flag,
                                                   p.status, kq ? 2 : 3)))
                        break;
                    uint8_t* dst = (kq ? sK : sV) + st * kTileBytes;
                    uint64_t* full = &bars[(kq ? kBarKFull : kBarVFull) + st];
                    const CUtensorMap* map = kq ? &tmK : &tmV;
                    mbar_arrive_expect_tx(full, kTileBytes);
                    tma_load_3d(dst, map, full, x0, ky, kz);
                    tma_load_3d(dst + kBoxBytes, map, full, x0 + 64, ky, kz);
                }
                ++qi;
            }
            // Do not leave with loads still landing in shared memory.  On the normal path the
            // last loads of each ring are consumed by MMAs whose completion arrives on kBarS (K)
            // / kBarPV (V), and every Q load is waited for before that tile's first QK.  After
            // an abort, the last load issued into each stage or buffer must still land: its
            // full barrier completes then (on the normal path these waits return at once).
            if (!qload)
                for (int x = max(g - 2, 0); x < g; ++x)
                    mbar_wait(&bars[(kq ? kBarS : kBarPV) + (x & 1)], (x >> 1) & 1, abort_flag,
                              p.status, 3);
            const int issued = qload ? qi : g;
            const int full = qload ? kBarQ : (kq ? kBarKFull : kBarVFull);
            for (int x = max(issued - 2, 0); x < issued; ++x)
                mbar_wait_drain(&bars[full + (x & 1)], (x >> 1) & 1, p.status, 12);
        }
        __syncwarp();
    } else if (warp == 1) {
        // ------------------------------------------------------------------ MMA issuer
        // The whole warp runs this loop, converged, so the descriptors and the loop state
        // stay in uniform registers; every MMA and commit is issued by one elected lane
        // (the same lane each time).  Each wait is taken by all lanes and combined with a
        // vote so that control flow stays uniform.
        const uint32_t idesc_qk = idesc_bf16_f32(kBM, kBN, false);  // B = K tile, K-major
        const uint32_t idesc_pv = idesc_bf16_f32(kBM, 128, true);   // B = V tile, MN-major
        // Descriptors are built once; a k-step only adds a constant to the start-address
        // field (16-byte units): +2 per 32 bytes along K inside a 128-byte swizzled row,
        // +1024 to move to the second 64-column box, +128 per 16 V rows (2048 bytes).
        const uint64_t dQ0 = smem_desc_sw128(smem_u32(sQ), 16, 1024);
        const uint64_t dK0 = smem_desc_sw128(smem_u32(sK), 16, 1024);
        const uint64_t dV0 = smem_desc_sw128(smem_u32(sV), kBoxBytes, 1024);
        constexpr uint64_t kStageStep = kTileBytes >> 4;
        auto wait_all = [&](int bar, uint32_t parity, int tag) -> bool {
            return __all_sync(0xFFFFFFFFu,
                              mbar_wait(&bars[bar], parity, abort_flag, p.status, tag));
        };
        bool ok = true;
        // Per block: wait for V(g) and P(g); issue the 8 P.V MMAs; wait for the operands of
        // QK(g+2); issue its 8 Q.K^T MMAs and commit kBarS (frees the K stage and hands S to
        // the softmax); then commit kBarPV (frees V stage g & 1 and P(g & 1)).  QK stays two
        // blocks ahead of PV.
        BlockCursor ahead;  // the block whose QK is next to issue
        ahead.k = 0;
        ahead.qi = 0;
        cursor_seek(ahead, p);
        int ahead_g = 0;
        auto wait_qk_operands = [&]() -> bool {
            if (ahead.j == 0 && !wait_all(kBarQ + (ahead.qi & 1), (ahead.qi >> 1) & 1, 4))
                return false;
            return wait_all(kBarKFull + (ahead_g & 1), (ahead_g >> 1) & 1, 5);
        };
        auto issue_qk = [&]() {
            const uint64_t dQ = dQ0 + (ahead.qi & 1) * kStageStep;
            const uint64_t dK = dK0 + (ahead_g & 1) * kStageStep;
            const uint32_t ts = tmem + kColS + (ahead_g & 1) * 128;
#pragma unroll
            for (int kk = 0; kk < 8; ++kk) {
                const uint64_t ko = (kk >> 2) * 1024 + (kk & 3) * 2;
                mma_ss_warp(ts, dQ + ko, dK + ko, idesc_qk, kk > 0 ? 1u : 0u);
            }
            mma_commit_warp(&bars[kBarS + (ahead_g & 1)]);
            if (ahead.j + 1 == ahead.t.nb) mma_commit_warp(&bars[kBarQFree + (ahead.qi & 1)]);
            cursor_next(ahead, p);
            ++ahead_g;
        };
        // Prologue: QK of the first two blocks.
        for (int i = 0; i < 2 && ok && ahead.valid; ++i) {
            if (!(ok = wait_qk_operands())) break;
            tc_fence_after();
            issue_qk();
        }
        int g = 0;
        for (int k = 0; ok; ++k) {
            const int rank = tile_rank(k, blockIdx.x, gridDim.x);
            if (rank >= p.total_tiles) break;
            const int nb = make_tile(p, rank).nb;
            for (int j = 0; ok && j < nb; ++j, ++g) {
                const int st = g & 1;
                const uint32_t ph = (g >> 1) & 1;
                if (!(ok = wait_all(kBarVFull + st, ph, 7))) break;
                if (!(ok = wait_all(kBarP + st, ph, 6))) break;
                tc_fence_after();
                const uint64_t dV = dV0 + st * kStageStep;
                const uint32_t tp = tmem + kColS + st * 128;  // P(g) lives in S slot g & 1
                const uint32_t acc0 = j > 0 ? 1u : 0u;  // first block of a tile starts O_A, O_B
#pragma unroll
                for (int x = 0; x < 2; ++x) {
#pragma unroll
                    for (int kk = 0; kk < 4; ++kk) {
                        // Key half x, 16 keys per step: P columns [64x + 8kk, +8) (bf16 pairs),
                        // V rows [64x + 16kk, +16) = two 8-row swizzle groups, into O_x.
                        mma_ts_warp(tmem + (x ? kColOB : kColOA), tp + 64 * x + 8 * kk,
                                    dV + (4 * x + kk) * 128, idesc_pv, kk > 0 ? 1u : acc0);
                    }
                }
                // The tile's output is complete once its last P.V is: the epilogue does not
                // wait behind the next tile's QK.
                if (j + 1 == nb) mma_commit_warp(&bars[kBarOFinal]);
                // softmax(g) has read S(g & 1) and written P(g) over part of it; QK(g+2) refills
                // the slot.  The tensor pipe executes one thread's MMAs in issue order, so
                // QK(g+2) overwrites P(g) only after the P.V MMAs above have read it.
                if (ahead.valid) {
                    if (!(ok = wait_qk_operands())) break;
                    tc_fence_after();
                    issue_qk();
                }
                // Committed after QK(g+2): completes once PV(g) and QK(g+2) are done.  Freeing
                // V stage g & 1 this late keeps the V reload off the tensor pipe's critical
                // stretch (measured: committing right after the P.V MMAs made the next QK
                // batch ~4x slower).
                mma_commit_warp(&bars[kBarPV + st]);
            }
        }
        // Leave only once every MMA issued above has completed, aborted or not: TMEM is
        // released after the block barrier below, and no MMA may still read shared memory or
        // write TMEM then.
        mma_commit_warp(&bars[kBarDrain]);
        mbar_wait_drain(&bars[kBarDrain], 0, p.status, 13);
    } else {
        // ------------------------------------------------------------------ softmax / epilogue
        // Warp w: lane quarter w % 4 (query rows = TMEM lanes), key half hx of every block.
        const int quarter = warp & 3;
        const int hx = (warp - 2) >> 2;  // 0: keys [0, 64) of each block, 1: keys [64, 128)
        const int r = quarter * 32 + lane;
        const uint32_t lane_base = static_cast<uint32_t>(quarter * 32) << 16;
        const uint32_t tOA = tmem + kColOA + lane_base;
        const uint32_t tOB = tmem + kColOB + lane_base;
        const uint32_t tOx = hx ? tOB : tOA;  // this half's accumulator
        const float sl2 = p.scale_log2;
        // Starting reference max: 128 |scale * log2(e)| bounds every score when q and k are
        // RMS-normalised over 128 dims (|q.k| <= 128), as the fused RoPE + QK-norm pass leaves
        // them.  A tile's first block then takes the optimistic path too.  For other inputs
        // the optimistic checks fall back to the exact path: a block sum above 2^8 (scores
        // above the bound), or on the first block one below 2^-64 (the bound far above them).
        const float m_init = 128.f * fabsf(sl2);
        int g = 0, qi = 0, xi = 0;
        bool ok = true;
        // Epilogue of a tile: O = (O_A 2^(mA-M) + O_B 2^(mB-M)) / (lA 2^(mA-M) + lB 2^(mB-M))
        // -> bf16 -> out[b, q, h, :]; this warp writes dims [64hx, 64hx + 64).  Run between
        // the next tile's first P store and its arrive (or after the last tile): the next
        // tile's first PV, which overwrites O_A and O_B, waits for that arrive, and the wait for
        // this tile's last PV overlaps the next tile's first softmax block.
        auto finish_tile = [&](const Tile& t, float m_ref, float l) -> bool {
            // Exchange (max, sum) with the other half's warp of this lane quarter: wait until it
            // has read the previous tile's values, post ours, wait for its, read them, say so.
            if (xi > 0 && !__all_sync(0xFFFFFFFFu, mbar_wait(&bars[kBarXrd + quarter], (xi - 1) & 1,
                                                             abort_flag, p.status, 15))) {
                return false;
            }
            tail->xch[quarter][hx][lane] = make_float2(m_ref, l);
            mbar_arrive(&bars[kBarXch + quarter]);
            if (!__all_sync(0xFFFFFFFFu, mbar_wait(&bars[kBarXch + quarter], xi & 1, abort_flag,
                                                   p.status, 16))) {
                return false;
            }
            const float2 other = tail->xch[quarter][hx ^ 1][lane];
            mbar_arrive(&bars[kBarXrd + quarter]);
            ++xi;
            if (!__all_sync(0xFFFFFFFFu, mbar_wait(&bars[kBarOFinal], qi & 1, abort_flag, p.status, 10))) {
                return false;
            }
            ++qi;
            tc_fence_after();
            const float mA = hx ? other.x : m_ref, lA = hx ? other.y : l;
            const float mB = hx ? m_ref : other.x, lB = hx ? l : other.y;
            const float M = fmaxf(mA, mB);
            const float muM = (M == kNegInf) ? 0.f : M;
            const float wA = fast_exp2(mA - muM), wB = fast_exp2(mB - muM);  // 0 for -inf
            const float inv = 1.0f / (lA * wA + lB * wB);  // no visible key: 0 * inf = NaN
            const float fa = wA * inv, fb = wB * inv;
            // The warp stages its 32 rows x 64 dims in shared memory in the 128B-swizzled
            // layout of a (64 dims x 32 rows) box and lane 0 writes them with one TMA store:
            // whole lines reach L2 instead of 32 scattered 16-byte pieces per store
            // instruction.  The staging area is reused only after the previous store from it
            // has finished reading it.  Rows at or past seq_q are clipped by the tensor map.
            uint8_t* stg = sO + (quarter * 2 + hx) * 4096;
            if (lane == 0) bulk_wait_read_all();
            __syncwarp();
    #pragma unroll
            for (int c = 0; c < 2; ++c) {
                uint32_t ra[32], rb[32];
                tmem_ld32_sync(tOA + 64 * hx + 32 * c, ra);
                tmem_ld32_sync(tOB + 64 * hx + 32 * c, rb);
    #pragma unroll
                for (int i = 0; i < 4; ++i) {
                    float o[8];
    #pragma unroll
                    for (int e = 0; e < 8; ++e)
                        o[e] = __fmaf_rn(__uint_as_float(ra[8 * i + e]), fa,
                                         __uint_as_float(rb[8 * i + e]) * fb);
                    const int d = 32 * c + 8 * i;           // first of the 8 dims (0..63)
                    const int granule = (d >> 3) ^ (lane & 7);  // 16-byte unit, swizzled
                    *reinterpret_cast<uint4*>(stg + lane * 128 + granule * 16) = f32_to_bf16x8(o);
                }
            }
            fence_proxy_async_smem();
            __syncwarp();
            const int y0 = t.q0 + quarter * 32;
            if (lane == 0 && y0 < p.seq_q) {
                tma_store_3d(&tmO, stg, t.h * 128 + 64 * hx, y0, t.b);
                bulk_commit();
            }
            tc_fence_before();
            return true;
        };
        bool pend = false;  // a finished tile whose epilogue has not run yet: pt, pm, pl
        Tile pt{};
        float pm = 0.f, pl = 0.f;
        for (int k = 0; ok; ++k) {
            const int rank = tile_rank(k, blockIdx.x, gridDim.x);
            if (rank >= p.total_tiles) break;
            const Tile t = make_tile(p, rank);
            const int q = t.q0 + r;
            const int qlim = q + t.off;  // last visible key for this row
            if (t.nb == 0) {
                // No visible key for any row of the tile: NaN, like the reference's 0/0.
                if (pend) {
                    if (!(ok = finish_tile(pt, pm, pl))) break;
                    pend = false;
                }
                if (q < p.seq_q) {
                    bf16* orow = p.out + (((size_t)t.b * p.seq_q + q) * p.heads + t.h) * kHeadDim + 64 * hx;
                    const uint4 nan4 = make_uint4(0x7FC07FC0u, 0x7FC07FC0u, 0x7FC07FC0u, 0x7FC07FC0u);
#pragma unroll
                    for (int i = 0; i < 8; ++i) reinterpret_cast<uint4*>(orow)[i] = nan4;
                }
                continue;
            }
            float m_ref = m_init, l = 0.f;  // this half's running reference max and row sum
            for (int j = 0; j < t.nb; ++j, ++g) {
                const int st = g & 1;
                // Warp-uniform outcome: the TMEM accesses below are warp-collective.
                if (!__all_sync(0xFFFFFFFFu, mbar_wait(&bars[kBarS + st], (g >> 1) & 1,
                                                       abort_flag, p.status, 9))) {
                    ok = false;
                    break;
                }
                tc_fence_after();
                // This half's 64 scores: S slot st, columns [64hx, 64hx + 64) = keys
                // key0 + 64hx + c.
                const uint32_t sbase = tmem + kColS + st * 128 + 64 * hx + lane_base;
                const int key0 = j * kBN + 64 * hx;
                // Two ways through a block.  Exact: the half-row max first, then the reference
                // max is renewed (this half's O and row sum rescaled) if the block max exceeds it
                // by more than the threshold, then P.  Optimistic: once every row of the warp has
                // a finite reference, P is computed against it straight away; no renewal was
                // needed exactly when no P exceeds 2^threshold, which the half-block's row sum
                // bounds (each P <= the sum), so a sum <= 2^threshold accepts the block and
                // anything else (or NaN) redoes it the exact way.
                const uint64_t sl2x2 = f2_pack(sl2, sl2);
                uint64_t acc2[2];
                uint32_t pk[32];
                bool exact = __any_sync(0xFFFFFFFFu, m_ref == kNegInf);
                for (;;) {
                    // S is (re)loaded from TMEM on each way through: it stays there until this
                    // warp writes P over it, and reloading is cheaper than keeping 64 scores live
                    // across a possible second pass.
                    uint32_t sraw[64];
                    tmem_ld64_sync(sbase, sraw);
                    float s_[64];
#pragma unroll
                    for (int c = 0; c < 64; ++c) s_[c] = __uint_as_float(sraw[c]);
                    if (key0 + 63 > t.q0 + t.off || key0 + 64 > t.kv_len) {  // CTA-uniform
                        const int lim = min(qlim + 1, t.kv_len) - key0;  // columns >= lim masked
#pragma unroll
                        for (int c = 0; c < 64; ++c) s_[c] = c < lim ? s_[c] : kNegInf;
                    }
                    if (exact) {
                        // Half-row max: 3-input max over pairs, eight independent chains.
                        float pm[8];
#pragma unroll
                        for (int i = 0; i < 8; ++i) pm[i] = fmaxf(s_[2 * i], s_[2 * i + 1]);
#pragma unroll
                        for (int c = 16; c < 64; c += 2)
                            pm[(c >> 1) & 7] = fmax3(pm[(c >> 1) & 7], s_[c], s_[c + 1]);
                        const float bm = fmax3(fmax3(pm[0], pm[1], pm[2]), fmax3(pm[3], pm[4], pm[5]),
                                               fmaxf(pm[6], pm[7]));
                        const float bm2 = bm * sl2;
                        // On a tile's first block the reference is only the starting bound: it is
                        // replaced by the block max (nothing has been accumulated yet).
                        const bool renew = j == 0 || (bm2 > m_ref + kRescaleThreshold) ||
                                           (m_ref == kNegInf && bm2 != kNegInf);
                        float alpha = 1.f;
                        if (renew) {
                            alpha = (m_ref == kNegInf || j == 0) ? 0.f : fast_exp2(m_ref - bm2);
                            m_ref = bm2;
                        }
                        l *= alpha;
                        // Rescale this half's O for rows that renewed; it must first hold
                        // PV(g-1) complete.
                        if (j > 0 && __any_sync(0xFFFFFFFFu, renew && alpha != 1.f)) {
                            const int sp = (g - 1) & 1;
                            if (!__all_sync(0xFFFFFFFFu,
                                            mbar_wait(&bars[kBarPV + sp], ((g - 1) >> 1) & 1,
                                                      abort_flag, p.status, 11))) {
                                ok = false;
                                break;
                            }
                            tc_fence_after();
#pragma unroll
                            for (int c = 0; c < 4; ++c) {
                                uint32_t raw[32];
                                tmem_ld32_sync(tOx + 32 * c, raw);
#pragma unroll
                                for (int i = 0; i < 32; ++i)
                                    raw[i] = __float_as_uint(__uint_as_float(raw[i]) * alpha);
                                tmem_st32_sync(tOx + 32 * c, raw);
                            }
                        }
                    }
                    const float mu = (m_ref == kNegInf) ? 0.f : m_ref;
                    // P = exp2(s * scale * log2e - mu), packed to bf16 pairs.  The scaling and
                    // the row sum run on packed f32x2 pairs; one pair in eight takes the FMA-pipe
                    // polynomial (input clamped to 127 so that it stays monotone) instead of
                    // MUFU.  Masked scores are -inf and give exactly 0.
                    const uint64_t nmu2 = f2_pack(-mu, -mu);
                    acc2[0] = f2_pack(0.f, 0.f);
                    acc2[1] = f2_pack(0.f, 0.f);
#pragma unroll
                    for (int i = 0; i < 32; ++i) {
                        float x0, x1, p0, p1;
                        f2_unpack(f2_fma(f2_pack(s_[2 * i], s_[2 * i + 1]), sl2x2, nmu2), x0, x1);
                        if ((i & 7) == 7) {
                            exp2_poly2(fminf(x0, 127.f), fminf(x1, 127.f), p0, p1);
                        } else {
                            p0 = fast_exp2(x0);
                            p1 = fast_exp2(x1);
                        }
                        acc2[i & 1] = f2_add(acc2[i & 1], f2_pack(p0, p1));
                        pk[i] = pack_bf16x2(p0, p1);
                    }
                    if (exact) break;
                    float c0, c1, d0, d1;
                    f2_unpack(acc2[0], c0, c1);
                    f2_unpack(acc2[1], d0, d1);
                    const float bsum = (c0 + c1) + (d0 + d1);
                    constexpr float kRenewSum = 256.0f;  // 2^kRescaleThreshold
                    exact = __any_sync(0xFFFFFFFFu, !(bsum <= kRenewSum) ||
                                                        (j == 0 && !(bsum >= kMinFirstSum)));
                    if (!exact) break;
                }
                if (!ok) break;
                float a0, a1, b0, b1;
                f2_unpack(acc2[0], a0, a1);
                f2_unpack(acc2[1], b0, b1);
                // P(g) goes over the first 32 of this half's S columns, which this warp has
                // finished reading (every load above waited).  Their previous reader as P was
                // PV(g-2); the MMA thread issued QK(g) after it and committed kBarS(g) after
                // both, so the kBarS(g) wait above covers it.
                tmem_st32_sync(sbase, pk);
                l += (a0 + a1) + (b0 + b1);
                if (j == 0 && pend) {
                    if (!(ok = finish_tile(pt, pm, pl))) break;
                    pend = false;
                }
                tc_fence_before();
                mbar_arrive(&bars[kBarP + st]);
            }
            if (!ok) break;
            pend = true;
            pt = t;
            pm = m_ref;
            pl = l;
        }
        if (ok && pend) ok = finish_tile(pt, pm, pl);
        // Output stores still reading the staging tile must finish before the CTA exits.
        if (lane == 0) bulk_wait_all();
        __syncwarp();
    }

    tc_fence_before();
    __syncthreads();
    if (warp == 1) {
        tc_fence_after();
        tmem_dealloc(tmem, kTmemCols);
    }
}

// ---------------------------------------------------------------------------------------
// host side: tensor maps
// ---------------------------------------------------------------------------------------
using EncodeTiledFn = CUresult (*)(CUtensorMap*, CUtensorMapDataType, cuuint32_t, void*,
                                   const cuuint64_t*, const cuuint64_t*, const cuuint32_t*,
                                   const cuuint32_t*, CUtensorMapInterleave, CUtensorMapSwizzle,
                                   CUtensorMapL2promotion, CUtensorMapFloatOOBfill);

EncodeTiledFn get_encode_fn() {
    static EncodeTiledFn fn = [] {
        void* p = nullptr;
        cudaDriverEntryPointQueryResult q{};
        if (cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &p, cudaEnableDefault, &q) !=
                cudaSuccess ||
            q != cudaDriverEntryPointSuccess)
            return static_cast<EncodeTiledFn>(nullptr);
        return reinterpret_cast<EncodeTiledFn>(p);
    }();
    return fn;
}

// 3-D map over [batch][rows][heads*128] bf16 with a (64 dims, box_rows rows, 1) box, 128B
// swizzle.
bool make_map(CUtensorMap* m, const void* base, int heads, int rows, int batch,
              long long batch_stride_elems, int box_rows) {
    EncodeTiledFn enc = get_encode_fn();
    if (!enc) return false;
    const cuuint64_t dims[3] = {(cuuint64_t)heads * 128, (cuuint64_t)rows, (cuuint64_t)batch};
    const cuuint64_t strides[2] = {(cuuint64_t)heads * 128 * 2,
                                   (cuuint64_t)(batch > 1 ? batch_stride_elems * 2
                                                          : (long long)rows * heads * 128 * 2)};
    const cuuint32_t box[3] = {64, (cuuint32_t)box_rows, 1};
    const cuuint32_t estr[3] = {1, 1, 1};
    return enc(m, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 3, const_cast<void*>(base), dims, strides,
               box, estr, CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B,
               CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE) ==
           CUDA_SUCCESS;
}

// Encoded tensor maps are cached per device (keyed by every encoding parameter), so repeated
// calls on the same buffers, e.g. one per layer and decode step of an engine, skip the host
// encoding work.  Small direct-mapped table; a collision just re-encodes.
struct MapKey {
    const void* base;
    int heads, rows, batch, dev, box_rows;
    long long stride;
    bool operator==(const MapKey& o) const {
        return base == o.base && heads == o.heads && rows == o.rows && batch == o.batch &&
               dev == o.dev && box_rows == o.box_rows && stride == o.stride;
    }
};
struct MapEntry {
    MapKey key;
    CUtensorMap map;
    bool used;
};
std::mutex g_map_mutex;
MapEntry g_maps[256];

bool cached_map(CUtensorMap* m, const void* base, int heads, int rows, int batch,
                long long batch_stride_elems, int dev, int box_rows) {
    const MapKey key{base, heads, rows, batch, dev, box_rows, batch_stride_elems};
    size_t h = reinterpret_cast<uintptr_t>(base) >> 8;
    h ^= (size_t)rows * 0x9E3779B1u ^ (size_t)heads * 0x85EBCA6Bu ^ (size_t)batch * 0xC2B2AE35u ^
         (size_t)dev * 0x27D4EB2Fu ^ (size_t)batch_stride_elems ^ (size_t)box_rows * 0x165667B1u;
    MapEntry& e = g_maps[h & 255];
    {
        std::lock_guard<std::mutex> lk(g_map_mutex);
        if (e.used && e.key == key) {
            *m = e.map;
            return true;
        }
    }
    if (!make_map(m, base, heads, rows, batch, batch_stride_elems, box_rows)) return false;
    std::lock_guard<std::mutex> lk(g_map_mutex);
    e.key = key;
    e.map = *m;
    e.used = true;
    return true;
}

}  // namespace

cudaError_t launch_prefill(const PrefillArgs& a, cudaStream_t stream) {
    if (a.batch <= 0 || a.seq_q <= 0) return cudaSuccess;
    // The shared-memory opt-in is per device context; remember it per device.
    static bool attr_set[64] = {};
    int dev = 0;
    cudaError_t e0 = cudaGetDevice(&dev);
    if (e0 != cudaSuccess) return e0;
    if (dev < 0 || dev >= 64) return cudaErrorInvalidDevice;
    if (!attr_set[dev]) {
        cudaError_t e = cudaFuncSetAttribute(prefill_kernel,
                                             cudaFuncAttributeMaxDynamicSharedMemorySize,
                                             (int)kSmemBytes);
        if (e != cudaSuccess) return e;
        attr_set[dev] = true;
    }
    CUtensorMap mq, mk, mv, mo;
    const int kv_rows = a.kv_rows;
    const long long qo_stride = (long long)a.seq_q * a.heads * 128;
    // Q/K/V loads move (64 dims x 128 rows) boxes; the output is stored by each softmax warp
    // in (64 dims x 32 rows) boxes.
    // Paged K/V: one map over the whole pool (batch extent 1); the producer turns (sequence,
    // key block) into a pool row through the page table.
    const bool paged = a.page_table != nullptr;
    const int kv_map_rows = paged ? a.num_pages * a.page_rows : kv_rows;
    const int kv_map_batch = paged ? 1 : a.batch;
    const long long kv_map_stride = paged ? 0 : a.kv_batch_stride;
    if (!cached_map(&mq, a.q, a.heads, a.seq_q, a.batch, qo_stride, dev, 128) ||
        !cached_map(&mk, a.k, a.heads, kv_map_rows, kv_map_batch, kv_map_stride, dev, 128) ||
        !cached_map(&mv, a.v, a.heads, kv_map_rows, kv_map_batch, kv_map_stride, dev, 128) ||
        !cached_map(&mo, a.out, a.heads, a.seq_q, a.batch, qo_stride, dev, 32))
        return cudaErrorInvalidValue;
    PrefillKParams kp;
    kp.out = a.out;
    kp.kv_offset_dev = a.kv_offset_dev;
    kp.kv_offset = a.kv_offset;
    kp.kv_len = a.kv_len;
    kp.kv_len_from_offset = a.kv_offset_dev != nullptr;
    kp.batch = a.batch;
    kp.seq_q = a.seq_q;
    kp.heads = a.heads;
    kp.n_qtiles = (a.seq_q + kBM - 1) / kBM;
    static int sm_count[64] = {};
    if (!sm_count[dev]) {
        cudaError_t e = cudaDeviceGetAttribute(&sm_count[dev], cudaDevAttrMultiProcessorCount, dev);
        if (e != cudaSuccess) return e;
    }
    kp.total_tiles = kp.n_qtiles * a.heads * a.batch;
    kp.scale_log2 = a.scale * kLog2e;
    kp.status = a.status;
    kp.page_table = a.page_table;
    kp.page_rows = a.page_rows;
    kp.pages_per_seq = a.pages_per_seq;
    kp.num_pages = a.num_pages;
    // Persistent: one CTA per SM (or fewer when there are fewer tiles).
    const unsigned grid = (unsigned)std::min<long long>(kp.total_tiles, sm_count[dev]);
    cudaLaunchConfig_t cfg = {};
    cfg.gridDim = dim3(grid);
    cfg.blockDim = dim3(kThreads);
    cfg.dynamicSmemBytes = kSmemBytes;
    cfg.stream = stream;
    cudaLaunchAttribute attr[1];
    attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
    attr[0].val.programmaticStreamSerializationAllowed = 1;
    cfg.attrs = attr;
    cfg.numAttrs = 1;
    return cudaLaunchKernelEx(&cfg, prefill_kernel, mq, mk, mv, mo, kp);
}

}  // namespace nc

// Host side of the library: argument checking, per-device state (RoPE table, decode
// workspace for the single-sequence entry point), the extern "C" ABI declared in
// include/nanochat_attn.h, the reference-compatible nanochat:: entry points declared in
// include/nanochat_attn_dropin.hpp, and the KV-cache object.
#include <algorithm>
#include <cstdint>
#include <cstdio>
#include <mutex>
#include <vector>

#include "../../include/nanochat_attn.h"
#include "../../include/nanochat_attn_dropin.hpp"
#include "nc_common.cuh"
#include "sm100_ptx.cuh"

namespace nc {

namespace {

// Kernel status word (per device); bounded waits that give up OR a code into it.
__device__ int g_nc_status = 0;

thread_local int t_last_cuda = 0;
thread_local int t_last_status = 0;

constexpr int kMaxDevices = 64;
std::mutex g_dev_mutex;
struct DeviceState {
    const float2* rope_cs = nullptr;  // set once the table is on this device
    int* status = nullptr;            // device address of g_nc_status
};
DeviceState g_dev[kMaxDevices];

// Decode workspaces of the single-sequence entry point (flash_attention with seq_q == 1), one
// per (device, stream handle): calls on different streams never share split counters or
// partial results.
struct StreamWorkspace {
    int dev;
    cudaStream_t stream;
    void* ws;
    size_t bytes;
};
std::vector<StreamWorkspace> g_stream_ws;

int cuda_fail(cudaError_t e) {
    t_last_cuda = (int)e;
    return NC_ERR_CUDA;
}

bool aligned16(const void* p) { return (reinterpret_cast<uintptr_t>(p) & 15u) == 0; }

int current_device(int* dev) {
    cudaError_t e = cudaGetDevice(dev);
    if (e != cudaSuccess) return cuda_fail(e);
    if (*dev < 0 || *dev >= kMaxDevices) return NC_ERR_INVALID_ARG;
    return NC_OK;
}

// Uploads the RoPE table to the current device on first use; returns its address.
int ensure_rope(const float2** table) {
    int dev;
    int st = current_device(&dev);
    if (st) return st;
    std::lock_guard<std::mutex> lk(g_dev_mutex);
    if (!g_dev[dev].rope_cs) {
        const float2* p = nullptr;
        cudaError_t e = upload_rope_table(&p);
        if (e != cudaSuccess) return cuda_fail(e);
        g_dev[dev].rope_cs = p;
    }
    *table = g_dev[dev].rope_cs;
    return NC_OK;
}

int status_word(int** out) {
    int dev;
    int st = current_device(&dev);
    if (st) return st;
    std::lock_guard<std::mutex> lk(g_dev_mutex);
    if (!g_dev[dev].status) {
        void* p = nullptr;
        cudaError_t e = cudaGetSymbolAddress(&p, g_nc_status);
        if (e != cudaSuccess) return cuda_fail(e);
        g_dev[dev].status = static_cast<int*>(p);
    }
    *out = g_dev[dev].status;
    return NC_OK;
}

// Keys per split-KV chunk for the streaming layout.  The persistent grid (one CTA per SM)
// takes its (split, sequence) items from a queue, so a call costs about items / SMs rounds
// plus, on average, half a round of tail, each round one item of T keys: T keys of streaming
// and a fixed part (the stage ring's ramp, the partial's write, the combine) worth about 40
// keys.  The host knows only the longest length, so the item count assumes an average of half
// of it and one partial split per two sequences.  T is the multiple of 16 from 64 (up to
// 1024) with the lowest estimated cost, at most 32 splits per sequence (the last split of a
// head combines all of them).  Measured on cfg3's lengths: 64 sequences 99 us at the chosen
// 160 keys against 110 us at the former rule (four items per CTA), the two 32-sequence halves
// 55.4 / 74.5 us at the chosen 128 against 58.3 / 77.0.
int auto_split_len(int batch, int max_kv_len) {
    // Small calls use the per-head layout (decode.cu), which takes 64 keys per split.
    if (decode_use_head_layout(batch, max_kv_len, 0)) return kDecodeHeadSplit;
    constexpr int kSms = 148;
    constexpr int kItemCostKeys = 40;
    const long long est_keys = batch > 1 ? (long long)batch * max_kv_len / 2 : max_kv_len;
    int best_t = 0;
    long long best_cost = 0;
    for (int t = 64; t <= 1024; t += 16) {
        if ((max_kv_len + t - 1) / t > 32) continue;
        const long long items = (est_keys + t - 1) / t + (batch + 1) / 2;
        const long long cost = (2 * items + kSms) * (t + kItemCostKeys);  // x 2 * kSms
        if (best_t == 0 || cost < best_cost) {
            best_t = t;
            best_cost = cost;
        }
    }
    long long t = best_t;
    // A batch of at most 8 that is too long for the per-head layout: longer splits, fewer
    // partials to combine (measured: 8 sequences x 1024 keys, 23.7 us with 80-key splits, 26.8
    // with 32).
    if (batch <= 8) t = std::max<long long>(t, 80);
    t = (t + 15) / 16 * 16;
    return (int)std::min<long long>(std::max<long long>(t, 16), 1024);
}

int check_heads(int heads) { return (heads >= 1 && heads <= 32) ? NC_OK : NC_ERR_INVALID_ARG; }

struct WsLayout {
    float* part_o;
    float2* part_ml;
    unsigned* counters;
};

// Workspace layout: the split counters come first, at a fixed offset, so calls with a
// different number of splits find them where the previous call left them (at zero).
WsLayout carve_ws(void* ws, int batch, int max_splits, int heads) {
    const size_t n = (size_t)batch * max_splits * heads;
    uint8_t* p = static_cast<uint8_t*>(ws);
    WsLayout w;
    w.counters = reinterpret_cast<unsigned*>(p);
    size_t off = (decode_counter_words(batch, heads) * sizeof(unsigned) + 255) & ~(size_t)255;
    w.part_ml = reinterpret_cast<float2*>(p + off);
    off = (off + n * sizeof(float2) + 255) & ~(size_t)255;
    w.part_o = reinterpret_cast<float*>(p + off);
    return w;
}

int rope_common(RopeMode mode, void* x, const void* k, const void* v, void* kc, void* vc,
                int seq_len, int heads, int start_pos, cudaStream_t stream) {
    if (seq_len < 0 || start_pos < 0 || check_heads(heads)) return NC_ERR_INVALID_ARG;
    if (seq_len == 0) return NC_OK;
    if (!x || (mode == kRopeNormAppend && (!k || !v || !kc || !vc))) return NC_ERR_INVALID_ARG;
    if (!aligned16(x) || !aligned16(k) || !aligned16(v) || !aligned16(kc) || !aligned16(vc))
        return NC_ERR_MISALIGNED;
    if ((long long)start_pos + seq_len > kRopeMaxSeq) return NC_ERR_RANGE;
    RopeArgs a{};
    int st = ensure_rope(&a.rope_cs);
    if (st) return st;
    a.q = static_cast<bf16*>(x);
    a.k = static_cast<const bf16*>(k);
    a.v = static_cast<const bf16*>(v);
    const size_t row0 = (size_t)start_pos * heads * kHeadDim;
    a.k_dst = kc ? static_cast<bf16*>(kc) + row0 : nullptr;
    a.v_dst = vc ? static_cast<bf16*>(vc) + row0 : nullptr;
    a.seq_len = seq_len;
    a.heads = heads;
    a.start_pos = start_pos;
    cudaError_t e = launch_rope(mode, a, stream);
    return e == cudaSuccess ? NC_OK : cuda_fail(e);
}

// Paged cache of nc_decode_attention_paged (see DecodeArgs).
struct PagedKV {
    void* k_pool;
    void* v_pool;
    const int* page_table;
    int num_pages, page_rows, pages_per_seq;
};

int decode_common(void* out, const void* q, const void* k_new, const void* v_new,
                  void* const* k_caches, void* const* v_caches, void* k_single, void* v_single,
                  const int* kv_len, int n_visible_single, int batch, int heads, float scale,
                  int max_kv_len, int split_len, void* ws, size_t ws_bytes,
                  cudaStream_t stream, int overlap = 0, const PagedKV* pg = nullptr) {
    // The decode kernel runs one warp per head plus a producer warp (<= 1024 threads).
    if (batch < 0 || heads < 1 || heads > 31 || max_kv_len < 0) return NC_ERR_INVALID_ARG;
    if (batch == 0) return NC_OK;
    if (!out || !q) return NC_ERR_INVALID_ARG;
    if ((k_new == nullptr) != (v_new == nullptr)) return NC_ERR_INVALID_ARG;
    if (!aligned16(out) || !aligned16(q) || !aligned16(k_new) || !aligned16(v_new) ||
        !aligned16(k_single) || !aligned16(v_single))
        return NC_ERR_MISALIGNED;
    if (split_len < 0 || (split_len % 16) != 0) return NC_ERR_INVALID_ARG;
    if (k_new && max_kv_len > kRopeMaxSeq) return NC_ERR_RANGE;
    if (pg) {
        if (!pg->k_pool || !pg->v_pool || !pg->page_table || !kv_len) return NC_ERR_INVALID_ARG;
        if (pg->page_rows < 16 || pg->page_rows % 16 || pg->num_pages < 1 ||
            pg->pages_per_seq < 1 || (long long)pg->pages_per_seq * pg->page_rows < max_kv_len)
            return NC_ERR_INVALID_ARG;
        if (!aligned16(pg->k_pool) || !aligned16(pg->v_pool)) return NC_ERR_MISALIGNED;
    }
    const int T = split_len ? split_len : auto_split_len(batch, std::max(max_kv_len, 1));
    const int max_splits = std::max(1, (max_kv_len + T - 1) / T);
    if (max_splits > 65535) return NC_ERR_INVALID_ARG;
    const size_t need = decode_workspace_bytes(batch, max_splits, heads);
    const bool head_layout = decode_use_head_layout(batch, max_kv_len, split_len);
    // Splits combined through a global workspace: all but the per-head layout's cluster case.
    const bool uses_ws =
        max_splits > 1 && !(head_layout && decode_head_cluster(max_splits, batch, overlap != 0));
    if (uses_ws && (!ws || ws_bytes < need)) return NC_ERR_WORKSPACE;
    DecodeArgs a{};
    if (k_new) {
        int st = ensure_rope(&a.rope_cs);
        if (st) return st;
    }
    a.out = static_cast<bf16*>(out);
    a.q = static_cast<const bf16*>(q);
    a.k_new = static_cast<const bf16*>(k_new);
    a.v_new = static_cast<const bf16*>(v_new);
    a.k_cache = reinterpret_cast<bf16* const*>(k_caches);
    a.v_cache = reinterpret_cast<bf16* const*>(v_caches);
    a.k_single = static_cast<bf16*>(k_single);
    a.v_single = static_cast<bf16*>(v_single);
    a.kv_len = kv_len;
    a.n_visible_single = n_visible_single;
    a.max_kv_len = max_kv_len;
    a.batch = batch;
    a.heads = heads;
    a.q_raw = k_new != nullptr;
    if (pg) {
        a.k_pool = static_cast<bf16*>(pg->k_pool);
        a.v_pool = static_cast<bf16*>(pg->v_pool);
        a.page_table = pg->page_table;
        a.page_rows = pg->page_rows;
        a.pages_per_seq = pg->pages_per_seq;
        a.num_pages = pg->num_pages;
    }
    a.head_layout = head_layout ? 1 : 0;
    a.overlap = overlap && a.head_layout ? 1 : 0;
    a.scale_log2 = scale * kLog2e;
    a.split_len = T;
    a.max_splits = max_splits;
    if (ws && uses_ws) {
        WsLayout w = carve_ws(ws, batch, max_splits, heads);
        a.part_o = w.part_o;
        a.part_ml = w.part_ml;
        a.counters = w.counters;
    }
    int st = status_word(&a.status);
    if (st) return st;
    cudaError_t e = launch_decode(a, stream);
    return e == cudaSuccess ? NC_OK : cuda_fail(e);
}

// Library-owned workspace for the single-sequence entry point, one per (device, stream).
// First use on a stream allocates it (cudaMalloc, so not under stream capture) and zeroes it
// on that stream; growing it waits for that stream's earlier work, which may still use it.
int single_ws(int heads, int n_visible, cudaStream_t stream, void** ws, size_t* bytes) {
    const int T = auto_split_len(1, std::max(n_visible, 1));
    const int splits = std::max(1, (n_visible + T - 1) / T);
    const size_t need = decode_workspace_bytes(1, splits, heads);
    int dev;
    int st = current_device(&dev);
    if (st) return st;
    std::lock_guard<std::mutex> lk(g_dev_mutex);
    StreamWorkspace* w = nullptr;
    for (StreamWorkspace& x : g_stream_ws)
        if (x.dev == dev && x.stream == stream) w = &x;
    if (!w) {
        g_stream_ws.push_back(StreamWorkspace{dev, stream, nullptr, 0});
        w = &g_stream_ws.back();
    }
    if (w->bytes < need) {
        if (w->ws) {
            cudaError_t e = cudaStreamSynchronize(stream);
            if (e != cudaSuccess) return cuda_fail(e);
            cudaFree(w->ws);
            w->ws = nullptr;
            w->bytes = 0;
        }
        const size_t alloc = std::max(need, (size_t)1 << 20);
        void* p = nullptr;
        cudaError_t e = cudaMalloc(&p, alloc);
        if (e != cudaSuccess) return cuda_fail(e);
        e = cudaMemsetAsync(p, 0, alloc, stream);
        if (e != cudaSuccess) {
            cudaFree(p);
            return cuda_fail(e);
        }
        w->ws = p;
        w->bytes = alloc;
    }
    *ws = w->ws;
    *bytes = w->bytes;
    return NC_OK;
}

int prefill_common(void* out, const void* q, const void* k, const void* v, long long stride,
                   int rows, const int* kv_offset_dev, int kv_offset, int kv_len, int batch,
                   int seq_q, int heads, float scale, cudaStream_t stream) {
    PrefillArgs a{};
    a.out = static_cast<bf16*>(out);
    a.q = static_cast<const bf16*>(q);
    a.k = static_cast<const bf16*>(k);
    a.v = static_cast<const bf16*>(v);
    a.kv_batch_stride = stride;
    a.kv_rows = std::max(rows, 1);
    a.kv_offset_dev = kv_offset_dev;
    a.kv_offset = kv_offset;
    a.kv_len = kv_len;
    a.batch = batch;
    a.seq_q = seq_q;
    a.heads = heads;
    a.scale = scale;
    int st = status_word(&a.status);
    if (st) return st;
    cudaError_t e = launch_prefill(a, stream);
    return e == cudaSuccess ? NC_OK : cuda_fail(e);
}

int flash_attention_impl(void* out, const void* Q, const void* K, const void* V, int seq_q,
                         int kv_len, int heads, float scale, int kv_offset,
                         cudaStream_t stream) {
    if (seq_q < 0 || kv_len < 0 || check_heads(heads)) return NC_ERR_INVALID_ARG;
    if (seq_q == 0) return NC_OK;
    if (!out || !Q || !K || !V) return NC_ERR_INVALID_ARG;
    if (!aligned16(out) || !aligned16(Q) || !aligned16(K) || !aligned16(V))
        return NC_ERR_MISALIGNED;
    if (seq_q == 1) {
        const int n_visible = std::min(kv_len, kv_offset + 1);
        void* ws = nullptr;
        size_t wsb = 0;
        // Up to 16 splits of the per-head layout combine in a thread-block cluster and need no
        // workspace; longer calls use this stream's library-owned workspace.
        const int T = auto_split_len(1, std::max(n_visible, 1));
        const int splits = std::max(1, (std::max(n_visible, 0) + T - 1) / T);
        if (splits > 1 && !(decode_use_head_layout(1, std::max(n_visible, 0), 0) &&
                            decode_head_cluster(splits, 1, false))) {
            int st = single_ws(heads, std::max(n_visible, 0), stream, &ws, &wsb);
            if (st) return st;
        }
        return decode_common(out, Q, nullptr, nullptr, nullptr, nullptr, const_cast<void*>(K),
                             const_cast<void*>(V), nullptr, n_visible, 1, heads, scale,
                             std::max(n_visible, 0), 0, ws, wsb, stream);
    }
    return prefill_common(out, Q, K, V, 0, kv_len, nullptr, kv_offset, kv_len, 1, seq_q, heads,
                          scale, stream);
}

}  // namespace

int internal_rope_table(const float2** table) { return ensure_rope(table); }
int internal_status_word(int** status) { return status_word(status); }
int internal_cuda_fail(cudaError_t e) { return cuda_fail(e); }
int internal_auto_split_len(int batch, int max_kv_len) { return auto_split_len(batch, max_kv_len); }

}  // namespace nc

using namespace nc;

// =========================================================================================
// extern "C" ABI
// =========================================================================================
extern "C" {

const char* nc_status_string(int status) {
    switch (status) {
        case NC_OK: return "ok";
        case NC_ERR_INVALID_ARG: return "invalid argument";
        case NC_ERR_MISALIGNED: return "pointer not 16-byte aligned";
        case NC_ERR_CUDA: return "CUDA runtime error";
        case NC_ERR_WORKSPACE: return "workspace missing or too small";
        case NC_ERR_RANGE: return "position beyond the RoPE table";
        case NC_ERR_DEVICE_TIMEOUT: return "kernel wait timed out";
        case NC_ERR_TOO_LARGE: return "request exceeds the fixed scratch of the allocation-free entry point";
        default: return "unknown status";
    }
}

int nc_last_cuda_error(void) { return t_last_cuda; }
int nc_last_status(void) { return t_last_status; }

int nc_device_status(int reset) {
    int v = 0;
    cudaError_t e = cudaMemcpyFromSymbol(&v, g_nc_status, sizeof(int));
    if (e != cudaSuccess) {
        t_last_cuda = (int)e;
        return -1;
    }
    if (reset) {
        const int z = 0;
        e = cudaMemcpyToSymbol(g_nc_status, &z, sizeof(int));
        if (e != cudaSuccess) t_last_cuda = (int)e;
    }
    return v;
}

int nc_init_rope_tables(void) {
    int dev;
    int st = current_device(&dev);
    if (st) return st;
    std::lock_guard<std::mutex> lk(g_dev_mutex);
    const float2* p = nullptr;
    cudaError_t e = upload_rope_table(&p);
    if (e != cudaSuccess) return cuda_fail(e);
    g_dev[dev].rope_cs = p;
    return NC_OK;
}

int nc_apply_rope(void* x, int seq_len, int n_heads, int start_pos, cudaStream_t stream) {
    return rope_common(kRopeOnly, x, nullptr, nullptr, nullptr, nullptr, seq_len, n_heads,
                       start_pos, stream);
}

int nc_apply_rope_rmsnorm(void* x, int seq_len, int n_heads, int start_pos,
                          cudaStream_t stream) {
    return rope_common(kRopeNorm, x, nullptr, nullptr, nullptr, nullptr, seq_len, n_heads,
                       start_pos, stream);
}

int nc_rope_qknorm_append(void* q, const void* k, const void* v, void* k_cache, void* v_cache,
                          int seq_len, int heads, int start_pos, cudaStream_t stream) {
    return rope_common(kRopeNormAppend, q, k, v, k_cache, v_cache, seq_len, heads, start_pos,
                       stream);
}

int nc_flash_attention(void* out, const void* Q, const void* K, const void* V, int seq_q,
                       int kv_len, int heads, float scale, int kv_offset, cudaStream_t stream) {
    return flash_attention_impl(out, Q, K, V, seq_q, kv_len, heads, scale, kv_offset, stream);
}

size_t nc_decode_workspace_bytes(int batch, int max_kv_len, int heads, int split_len) {
    if (batch <= 0 || heads <= 0 || max_kv_len < 0 || split_len < 0) return 0;
    const int T = split_len ? split_len : auto_split_len(batch, std::max(max_kv_len, 1));
    const int max_splits = std::max(1, (max_kv_len + T - 1) / T);
    return decode_workspace_bytes(batch, max_splits, heads);
}

int nc_decode_attention(void* out, const void* q, const void* k_new, const void* v_new,
                        void* const* k_caches, void* const* v_caches, const int* kv_len,
                        int batch, int heads, float scale, int max_kv_len, int split_len,
                        void* workspace, size_t workspace_bytes, cudaStream_t stream) {
    if (batch > 0 && (!k_caches || !v_caches || !kv_len)) return NC_ERR_INVALID_ARG;
    return decode_common(out, q, k_new, v_new, k_caches, v_caches, nullptr, nullptr, kv_len, 0,
                         batch, heads, scale, max_kv_len, split_len, workspace,
                         workspace_bytes, stream);
}

int nc_decode_attention_paged(void* out, const void* q, const void* k_new, const void* v_new,
                              void* k_pool, void* v_pool, int num_pages, int page_rows,
                              const int* page_table, int pages_per_seq, const int* kv_len,
                              int batch, int heads, float scale, int max_kv_len, int split_len,
                              void* workspace, size_t workspace_bytes, cudaStream_t stream) {
    const PagedKV pg{k_pool, v_pool, page_table, num_pages, page_rows, pages_per_seq};
    return decode_common(out, q, k_new, v_new, nullptr, nullptr, nullptr, nullptr, kv_len, 0,
                         batch, heads, scale, max_kv_len, split_len, workspace,
                         workspace_bytes, stream, 0, &pg);
}

int nc_decode_attention_overlap(void* out, const void* q, const void* k_new, const void* v_new,
                                void* const* k_caches, void* const* v_caches, const int* kv_len,
                                int batch, int heads, float scale, int max_kv_len, int split_len,
                                void* workspace, size_t workspace_bytes, cudaStream_t stream) {
    if (batch > 0 && (!k_caches || !v_caches || !kv_len)) return NC_ERR_INVALID_ARG;
    return decode_common(out, q, k_new, v_new, k_caches, v_caches, nullptr, nullptr, kv_len, 0,
                         batch, heads, scale, max_kv_len, split_len, workspace,
                         workspace_bytes, stream, 1);
}

int nc_prefill_attention_paged(void* out, const void* q, const void* k_pool, const void* v_pool,
                               int num_pages, int page_rows, const int* page_table,
                               int pages_per_seq, const int* kv_offset, int batch, int seq_q,
                               int heads, float scale, cudaStream_t stream) {
    if (batch < 0 || seq_q < 0 || check_heads(heads)) return NC_ERR_INVALID_ARG;
    if (batch == 0 || seq_q == 0) return NC_OK;
    if (!out || !q || !k_pool || !v_pool || !page_table || !kv_offset) return NC_ERR_INVALID_ARG;
    if (page_rows < 128 || page_rows % 128 || num_pages < 1 || pages_per_seq < 1 ||
        (long long)num_pages * page_rows > INT32_MAX / 2)
        return NC_ERR_INVALID_ARG;
    if (!aligned16(out) || !aligned16(q) || !aligned16(k_pool) || !aligned16(v_pool))
        return NC_ERR_MISALIGNED;
    PrefillArgs a{};
    a.out = static_cast<bf16*>(out);
    a.q = static_cast<const bf16*>(q);
    a.k = static_cast<const bf16*>(k_pool);
    a.v = static_cast<const bf16*>(v_pool);
    a.kv_rows = num_pages * page_rows;
    a.kv_offset_dev = kv_offset;
    a.batch = batch;
    a.seq_q = seq_q;
    a.heads = heads;
    a.scale = scale;
    a.page_table = page_table;
    a.page_rows = page_rows;
    a.pages_per_seq = pages_per_seq;
    a.num_pages = num_pages;
    int st = status_word(&a.status);
    if (st) return st;
    cudaError_t e = launch_prefill(a, stream);
    return e == cudaSuccess ? NC_OK : cuda_fail(e);
}

int nc_rope_qknorm_append_paged(void* q, const void* k, const void* v, void* k_pool,
                                void* v_pool, int num_pages, int page_rows, const int* pages,
                                int n_pages, int seq_len, int heads, int start_pos,
                                cudaStream_t stream) {
    if (seq_len < 0 || start_pos < 0 || check_heads(heads)) return NC_ERR_INVALID_ARG;
    if (seq_len == 0) return NC_OK;
    if (!q || !k || !v || !k_pool || !v_pool || !pages || page_rows < 1 || num_pages < 1)
        return NC_ERR_INVALID_ARG;
    if (!aligned16(q) || !aligned16(k) || !aligned16(v) || !aligned16(k_pool) ||
        !aligned16(v_pool))
        return NC_ERR_MISALIGNED;
    if ((long long)start_pos + seq_len > kRopeMaxSeq) return NC_ERR_RANGE;
    if ((long long)(start_pos + seq_len - 1) / page_rows >= n_pages) return NC_ERR_INVALID_ARG;
    for (int j = start_pos / page_rows; j <= (start_pos + seq_len - 1) / page_rows; ++j)
        if (pages[j] < 0 || pages[j] >= num_pages) return NC_ERR_INVALID_ARG;
    RopeArgs a{};
    int st = ensure_rope(&a.rope_cs);
    if (st) return st;
    const size_t rowstride = (size_t)heads * kHeadDim;
    // One launch per page the chunk touches; each page is contiguous in the pool.
    for (int p0 = start_pos; p0 < start_pos + seq_len;) {
        const int j = p0 / page_rows;
        const int p1 = std::min(start_pos + seq_len, (j + 1) * page_rows);
        const size_t src = (size_t)(p0 - start_pos) * rowstride;
        const size_t dst = ((size_t)pages[j] * page_rows + (p0 - j * page_rows)) * rowstride;
        a.q = static_cast<bf16*>(q) + src;
        a.k = static_cast<const bf16*>(k) + src;
        a.v = static_cast<const bf16*>(v) + src;
        a.k_dst = static_cast<bf16*>(k_pool) + dst;
        a.v_dst = static_cast<bf16*>(v_pool) + dst;
        a.seq_len = p1 - p0;
        a.heads = heads;
        a.start_pos = p0;
        cudaError_t e = launch_rope(kRopeNormAppend, a, stream);
        if (e != cudaSuccess) return cuda_fail(e);
        p0 = p1;
    }
    return NC_OK;
}

int nc_rope_qknorm_append_batched(void* q, const void* k, const void* v, void* k_slab,
                                  void* v_slab, long long seq_stride, int batch, int seq_len,
                                  int heads, int start_pos, cudaStream_t stream) {
    if (batch < 0 || seq_len < 0 || start_pos < 0 || check_heads(heads)) return NC_ERR_INVALID_ARG;
    if (batch == 0 || seq_len == 0) return NC_OK;
    if (!q || !k || !v || !k_slab || !v_slab) return NC_ERR_INVALID_ARG;
    if (seq_stride % 8 || (batch > 1 && seq_stride < (long long)(start_pos + seq_len) * heads * kHeadDim))
        return NC_ERR_INVALID_ARG;
    if ((long long)batch * seq_len * heads > INT32_MAX / 2) return NC_ERR_INVALID_ARG;
    if (!aligned16(q) || !aligned16(k) || !aligned16(v) || !aligned16(k_slab) || !aligned16(v_slab))
        return NC_ERR_MISALIGNED;
    if ((long long)start_pos + seq_len > kRopeMaxSeq) return NC_ERR_RANGE;
    RopeArgs a{};
    int st = ensure_rope(&a.rope_cs);
    if (st) return st;
    const size_t row0 = (size_t)start_pos * heads * kHeadDim;
    a.q = static_cast<bf16*>(q);
    a.k = static_cast<const bf16*>(k);
    a.v = static_cast<const bf16*>(v);
    a.k_dst = static_cast<bf16*>(k_slab) + row0;
    a.v_dst = static_cast<bf16*>(v_slab) + row0;
    a.seq_len = seq_len;
    a.heads = heads;
    a.start_pos = start_pos;
    a.batch = batch;
    a.dst_stride = seq_stride;
    cudaError_t e = launch_rope(kRopeNormAppend, a, stream);
    return e == cudaSuccess ? NC_OK : cuda_fail(e);
}

int nc_rope_qknorm_append_paged_batched(void* q, const void* k, const void* v, void* k_pool,
                                        void* v_pool, int num_pages, int page_rows,
                                        const int* page_table, int pages_per_seq, int batch,
                                        int seq_len, int heads, int start_pos,
                                        cudaStream_t stream) {
    if (batch < 0 || seq_len < 0 || start_pos < 0 || check_heads(heads)) return NC_ERR_INVALID_ARG;
    if (batch == 0 || seq_len == 0) return NC_OK;
    if (!q || !k || !v || !k_pool || !v_pool || !page_table || page_rows < 1 || num_pages < 1)
        return NC_ERR_INVALID_ARG;
    if ((long long)(start_pos + seq_len - 1) / page_rows >= pages_per_seq) return NC_ERR_INVALID_ARG;
    if ((long long)batch * seq_len * heads > INT32_MAX / 2) return NC_ERR_INVALID_ARG;
    if (!aligned16(q) || !aligned16(k) || !aligned16(v) || !aligned16(k_pool) ||
        !aligned16(v_pool))
        return NC_ERR_MISALIGNED;
    if ((long long)start_pos + seq_len > kRopeMaxSeq) return NC_ERR_RANGE;
    RopeArgs a{};
    int st = ensure_rope(&a.rope_cs);
    if (st) return st;
    st = status_word(&a.status);
    if (st) return st;
    a.q = static_cast<bf16*>(q);
    a.k = static_cast<const bf16*>(k);
    a.v = static_cast<const bf16*>(v);
    a.k_dst = static_cast<bf16*>(k_pool);
    a.v_dst = static_cast<bf16*>(v_pool);
    a.seq_len = seq_len;
    a.heads = heads;
    a.start_pos = start_pos;
    a.batch = batch;
    a.page_table = page_table;
    a.pages_per_seq = pages_per_seq;
    a.page_rows = page_rows;
    a.num_pages = num_pages;
    cudaError_t e = launch_rope(kRopeNormAppend, a, stream);
    return e == cudaSuccess ? NC_OK : cuda_fail(e);
}

int nc_prefill_attention_batched(void* out, const void* q, const void* k_slab,
                                 const void* v_slab, long long seq_stride, int rows_per_seq,
                                 const int* kv_offset, int batch, int seq_q, int heads,
                                 float scale, cudaStream_t stream) {
    if (batch < 0 || seq_q < 0 || rows_per_seq < 1 || check_heads(heads)) return NC_ERR_INVALID_ARG;
    if (batch == 0 || seq_q == 0) return NC_OK;
    if (!out || !q || !k_slab || !v_slab || !kv_offset) return NC_ERR_INVALID_ARG;
    if (seq_stride < (long long)rows_per_seq * heads * kHeadDim || (seq_stride % 8) != 0)
        return NC_ERR_INVALID_ARG;
    if (!aligned16(out) || !aligned16(q) || !aligned16(k_slab) || !aligned16(v_slab))
        return NC_ERR_MISALIGNED;
    return prefill_common(out, q, k_slab, v_slab, seq_stride, rows_per_seq, kv_offset, 0, 0,
                          batch, seq_q, heads, scale, stream);
}

}  // extern "C"

// =========================================================================================
// Reference-compatible C++ entry points (namespace nanochat, C++ linkage).
// =========================================================================================
namespace nanochat {

void apply_rope(nv_bfloat16* x, int seq_len, int n_heads, int start_pos, cudaStream_t stream) {
    t_last_status = nc_apply_rope(x, seq_len, n_heads, start_pos, stream);
}

void apply_rope_rmsnorm(nv_bfloat16* x, int seq_len, int n_heads, int start_pos,
                        cudaStream_t stream) {
    t_last_status = nc_apply_rope_rmsnorm(x, seq_len, n_heads, start_pos, stream);
}

void init_rope_tables() { t_last_status = nc_init_rope_tables(); }

void flash_attention(nv_bfloat16* out, const nv_bfloat16* Q, const nv_bfloat16* K,
                     const nv_bfloat16* V, int seq_q, int kv_len, int heads, float scale,
                     int kv_offset, cudaStream_t stream) {
    t_last_status =
        nc_flash_attention(out, Q, K, V, seq_q, kv_len, heads, scale, kv_offset, stream);
}

}  // namespace nanochat

// =========================================================================================
// KV cache
// =========================================================================================
struct nc_kv_cache {
    int n_layers = 0, n_seqs = 0, max_len = 0, heads = 0, device = 0;
    long long seq_stride = 0;               // elements between sequences in a slab
    std::vector<bf16*> k_slab, v_slab;      // per layer, [n_seqs][max_len][heads][128]
    void** d_tables = nullptr;              // device [n_layers][2][n_seqs]
    std::vector<int> lens;                  // [n_layers][n_seqs]
    int* d_lens = nullptr;                  // device [n_layers][n_seqs], decode staging
    void* ws = nullptr;                     // decode workspace for n_seqs x max_len
    size_t ws_bytes = 0;
};

namespace {

void kv_free(nc_kv_cache* c) {
    for (bf16* p : c->k_slab) cudaFree(p);
    for (bf16* p : c->v_slab) cudaFree(p);
    if (c->d_tables) cudaFree(c->d_tables);
    if (c->d_lens) cudaFree(c->d_lens);
    if (c->ws) cudaFree(c->ws);
    delete c;
}

bool kv_ok(const nc_kv_cache* c, int layer, int seq) {
    return c && layer >= 0 && layer < c->n_layers && seq >= 0 && seq < c->n_seqs;
}

}  // namespace

extern "C" {

int nc_kv_cache_create(nc_kv_cache** out, int n_layers, int n_seqs, int max_len, int heads) {
    if (!out || n_layers < 1 || n_seqs < 1 || max_len < 1 || check_heads(heads))
        return NC_ERR_INVALID_ARG;
    if (max_len > kRopeMaxSeq) return NC_ERR_RANGE;
    *out = nullptr;
    nc_kv_cache* c = new nc_kv_cache();
    c->n_layers = n_layers;
    c->n_seqs = n_seqs;
    c->max_len = max_len;
    c->heads = heads;
    cudaError_t e = cudaGetDevice(&c->device);
    if (e != cudaSuccess) {
        delete c;
        return cuda_fail(e);
    }
    c->seq_stride = (long long)max_len * heads * kHeadDim;
    const size_t slab = (size_t)n_seqs * c->seq_stride * sizeof(bf16);
    c->lens.assign((size_t)n_layers * n_seqs, 0);
    std::vector<void*> tables((size_t)n_layers * 2 * n_seqs);
    for (int l = 0; l < n_layers; ++l) {
        bf16 *k = nullptr, *v = nullptr;
        if ((e = cudaMalloc(&k, slab)) != cudaSuccess) break;
        c->k_slab.push_back(k);
        if ((e = cudaMalloc(&v, slab)) != cudaSuccess) break;
        c->v_slab.push_back(v);
        if ((e = cudaMemset(k, 0, slab)) != cudaSuccess) break;
        if ((e = cudaMemset(v, 0, slab)) != cudaSuccess) break;
        for (int s = 0; s < n_seqs; ++s) {
            tables[((size_t)l * 2 + 0) * n_seqs + s] = k + (size_t)s * c->seq_stride;
            tables[((size_t)l * 2 + 1) * n_seqs + s] = v + (size_t)s * c->seq_stride;
        }
    }
    if (e == cudaSuccess) e = cudaMalloc(&c->d_tables, tables.size() * sizeof(void*));
    if (e == cudaSuccess)
        e = cudaMemcpy(c->d_tables, tables.data(), tables.size() * sizeof(void*),
                       cudaMemcpyHostToDevice);
    if (e == cudaSuccess) e = cudaMalloc(&c->d_lens, c->lens.size() * sizeof(int));
    if (e == cudaSuccess) e = cudaMemset(c->d_lens, 0, c->lens.size() * sizeof(int));
    if (e == cudaSuccess) {
        c->ws_bytes = nc_decode_workspace_bytes(n_seqs, max_len, heads, 0);
        e = cudaMalloc(&c->ws, c->ws_bytes);
        if (e == cudaSuccess) e = cudaMemset(c->ws, 0, c->ws_bytes);
    }
    if (e != cudaSuccess) {
        kv_free(c);
        return cuda_fail(e);
    }
    *out = c;
    return NC_OK;
}

int nc_kv_cache_destroy(nc_kv_cache* cache) {
    if (!cache) return NC_ERR_INVALID_ARG;
    cudaError_t e = cudaDeviceSynchronize();
    kv_free(cache);
    return e == cudaSuccess ? NC_OK : cuda_fail(e);
}

void* nc_kv_cache_k(nc_kv_cache* c, int layer, int seq) {
    return kv_ok(c, layer, seq) ? c->k_slab[layer] + (size_t)seq * c->seq_stride : nullptr;
}
void* nc_kv_cache_v(nc_kv_cache* c, int layer, int seq) {
    return kv_ok(c, layer, seq) ? c->v_slab[layer] + (size_t)seq * c->seq_stride : nullptr;
}
void* const* nc_kv_cache_k_table(nc_kv_cache* c, int layer) {
    return kv_ok(c, layer, 0) ? c->d_tables + (size_t)layer * 2 * c->n_seqs : nullptr;
}
void* const* nc_kv_cache_v_table(nc_kv_cache* c, int layer) {
    return kv_ok(c, layer, 0) ? c->d_tables + ((size_t)layer * 2 + 1) * c->n_seqs : nullptr;
}
long long nc_kv_cache_seq_stride(const nc_kv_cache* c) { return c ? c->seq_stride : 0; }
int nc_kv_cache_max_len(const nc_kv_cache* c) { return c ? c->max_len : 0; }

int nc_kv_cache_len(const nc_kv_cache* c, int layer, int seq) {
    return kv_ok(c, layer, seq) ? c->lens[(size_t)layer * c->n_seqs + seq] : -1;
}

int nc_kv_cache_set_len(nc_kv_cache* c, int layer, int seq, int len) {
    if (!kv_ok(c, layer, seq) || len < 0 || len > c->max_len) return NC_ERR_INVALID_ARG;
    c->lens[(size_t)layer * c->n_seqs + seq] = len;
    return NC_OK;
}

int nc_kv_cache_clear(nc_kv_cache* c, int seq) {
    if (!c || seq >= c->n_seqs) return NC_ERR_INVALID_ARG;
    for (int l = 0; l < c->n_layers; ++l)
        for (int s = 0; s < c->n_seqs; ++s)
            if (seq < 0 || s == seq) c->lens[(size_t)l * c->n_seqs + s] = 0;
    return NC_OK;
}

int nc_kv_cache_prefill(nc_kv_cache* c, int layer, int seq, void* out, void* q, const void* k,
                        const void* v, int seq_len, float scale, cudaStream_t stream) {
    if (!kv_ok(c, layer, seq) || seq_len < 0) return NC_ERR_INVALID_ARG;
    if (seq_len == 0) return NC_OK;
    int& len = c->lens[(size_t)layer * c->n_seqs + seq];
    const int start = len;
    if ((long long)start + seq_len > c->max_len) return NC_ERR_RANGE;
    void* kc = nc_kv_cache_k(c, layer, seq);
    void* vc = nc_kv_cache_v(c, layer, seq);
    int st = nc_rope_qknorm_append(q, k, v, kc, vc, seq_len, c->heads, start, stream);
    if (st) return st;
    st = nc_flash_attention(out, q, kc, vc, seq_len, start + seq_len, c->heads, scale, start,
                            stream);
    if (st) return st;
    len = start + seq_len;
    return NC_OK;
}

int nc_kv_cache_decode(nc_kv_cache* c, int layer, void* out, const void* q, const void* k_new,
                       const void* v_new, float scale, cudaStream_t stream) {
    if (!kv_ok(c, layer, 0) || !k_new || !v_new) return NC_ERR_INVALID_ARG;
    int* lens = &c->lens[(size_t)layer * c->n_seqs];
    std::vector<int> next(c->n_seqs);
    for (int s = 0; s < c->n_seqs; ++s) {
        next[s] = lens[s] + 1;
        if (next[s] > c->max_len) return NC_ERR_RANGE;
    }
    int* d = c->d_lens + (size_t)layer * c->n_seqs;
    // Pageable source: the runtime stages it before returning, so `next` may go away.
    cudaError_t e = cudaMemcpyAsync(d, next.data(), c->n_seqs * sizeof(int),
                                    cudaMemcpyHostToDevice, stream);
    if (e != cudaSuccess) return cuda_fail(e);
    int st = nc_decode_attention(out, q, k_new, v_new, nc_kv_cache_k_table(c, layer),
                                 nc_kv_cache_v_table(c, layer), d, c->n_seqs, c->heads, scale,
                                 c->max_len, 0, c->ws, c->ws_bytes, stream);
    if (st) return st;
    for (int s = 0; s < c->n_seqs; ++s) lens[s] = next[s];
    return NC_OK;
}

}  // extern "C"

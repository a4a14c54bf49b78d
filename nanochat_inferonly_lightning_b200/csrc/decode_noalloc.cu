// Batched decode attention that allocates no device memory.
//
// The split-KV decode kernel keeps per-split partial results (running max, row sum and 128
// fp32 accumulators per head) plus one split counter per sequence in global scratch memory.
// nc_decode_attention takes that scratch from the caller; this entry point instead uses a
// fixed array compiled into the library, for callers that cannot hand out device memory:
// an engine whose device memory is fully planned by an outside allocator, a host binding
// (cgo, JNI, ctypes) with no device allocator of its own to pass a workspace, or a
// latency-critical serving loop where cudaMalloc, which can synchronize the whole device,
// is not acceptable.  Nothing here calls cudaMalloc, cudaFree or an allocating library
// routine.
//
// Costs and rules of the shared array:
//   * every GPU that loads the library holds kNoAllocScratchBytes (8 MiB) until exit;
//   * all calls on a device share the one array and it keeps the last call's contents, so
//     calls whose kernels overlap on the GPU (different streams, or different host threads
//     without ordering) race on it; order them on one stream;
//   * the first call on a device does the set-up (it resolves the array's device address,
//     and the fused path uploads the RoPE table); make that first call before any stream
//     capture;
//   * every call clears the split counters it will use (a memset on the caller's stream)
//     before the decode kernel runs.  The kernel returns its counters to zero when it
//     completes, but a launch whose bounded wait gave up leaves them set, and a caller of this
//     entry point has no workspace of its own to re-zero.
#include <algorithm>
#include <mutex>

#include "../../include/nanochat_attn.h"
#include "nc_common.cuh"

namespace nc {

namespace {

constexpr size_t kNoAllocScratchBytes = 8u << 20;
constexpr int kNoAllocMaxBatch = 256;
// Work-queue words and per-(sequence, head) split tickets for batch 256 x 32 heads (32.8 KB),
// at a fixed offset 0.
constexpr size_t kCounterBytes = 64u << 10;
constexpr int kMaxDevices = 64;

// Split counters at [0, 64 KiB), then the partial maxima/sums and the partial accumulators.
// Every call clears the counter words it uses before its kernel runs.
static __device__ __align__(256) unsigned char g_noalloc_scratch[kNoAllocScratchBytes];

std::mutex g_setup_mutex;
unsigned char* g_scratch_addr[kMaxDevices] = {};

// Per-device set-up, once, with that device current.  In host code g_noalloc_scratch names
// a host-side stand-in, not device memory: a kernel must get the address resolved here.
int scratch_address(unsigned char** out) {
    int dev = 0;
    cudaError_t e = cudaGetDevice(&dev);
    if (e != cudaSuccess) return internal_cuda_fail(e);
    if (dev < 0 || dev >= kMaxDevices) return NC_ERR_INVALID_ARG;
    std::lock_guard<std::mutex> lk(g_setup_mutex);
    if (!g_scratch_addr[dev]) {
        void* p = nullptr;
        e = cudaGetSymbolAddress(&p, g_noalloc_scratch);
        if (e != cudaSuccess) return internal_cuda_fail(e);
        if (!p) return internal_cuda_fail(cudaErrorInvalidSymbol);
        g_scratch_addr[dev] = static_cast<unsigned char*>(p);
    }
    *out = g_scratch_addr[dev];
    return NC_OK;
}

size_t round256(size_t n) { return (n + 255) & ~(size_t)255; }

// Partial-result bytes for this batch, split count and head count.
size_t partial_bytes(int batch, int splits, int heads) {
    const size_t n = (size_t)batch * splits * heads;
    return round256(n * sizeof(float2)) + n * kHeadDim * sizeof(float);
}

bool aligned16(const void* p) { return (reinterpret_cast<uintptr_t>(p) & 15u) == 0; }

}  // namespace

}  // namespace nc

using namespace nc;

extern "C" int nc_decode_attention_noalloc(void* out, const void* q, const void* k_new,
                                           const void* v_new, void* const* k_caches,
                                           void* const* v_caches, const int* kv_len, int batch,
                                           int heads, float scale, int max_kv_len,
                                           cudaStream_t stream) {
    if (batch < 0 || heads < 1 || heads > 31 || max_kv_len < 0) return NC_ERR_INVALID_ARG;
    if (batch == 0) return NC_OK;
    if (!out || !q || !k_caches || !v_caches || !kv_len) return NC_ERR_INVALID_ARG;
    if ((k_new == nullptr) != (v_new == nullptr)) return NC_ERR_INVALID_ARG;
    if (!aligned16(out) || !aligned16(q) || !aligned16(k_new) || !aligned16(v_new))
        return NC_ERR_MISALIGNED;
    if (batch > kNoAllocMaxBatch || max_kv_len > kRopeMaxSeq) return NC_ERR_TOO_LARGE;

    // Split plan: the one nc_decode_attention makes for these sizes (same split length, same
    // layout), with the split length doubled only while the partial results would not fit in
    // the array (a single split needs no partials at all).  The per-head layout's calls
    // (<= 16 sequences, <= 16384 keys in all, 64-key splits) always fit: at most 256
    // (sequence, split) pairs x 31 heads x 520 bytes.
    const int L = std::max(max_kv_len, 1);
    const int T_auto = internal_auto_split_len(batch, L);
    long long T = T_auto;
    const size_t room = kNoAllocScratchBytes - kCounterBytes;
    int splits = (int)((L + T - 1) / T);
    while (splits > 1 && partial_bytes(batch, splits, heads) > room) {
        T *= 2;
        splits = (int)((L + T - 1) / T);
    }
    if (splits > 1 && partial_bytes(batch, splits, heads) > room) return NC_ERR_TOO_LARGE;
    const size_t counter_bytes = decode_counter_words(batch, heads) * sizeof(unsigned);
    if (counter_bytes > kCounterBytes) return NC_ERR_TOO_LARGE;

    unsigned char* base = nullptr;
    int st = scratch_address(&base);
    if (st) return st;
    DecodeArgs a{};
    if (k_new) {
        st = internal_rope_table(&a.rope_cs);
        if (st) return st;
    }
    st = internal_status_word(&a.status);
    if (st) return st;
    a.out = static_cast<bf16*>(out);
    a.q = static_cast<const bf16*>(q);
    a.k_new = static_cast<const bf16*>(k_new);
    a.v_new = static_cast<const bf16*>(v_new);
    a.k_cache = reinterpret_cast<bf16* const*>(k_caches);
    a.v_cache = reinterpret_cast<bf16* const*>(v_caches);
    a.kv_len = kv_len;
    a.max_kv_len = max_kv_len;
    a.batch = batch;
    a.heads = heads;
    a.q_raw = k_new != nullptr;
    a.scale_log2 = scale * kLog2e;
    a.split_len = (int)T;
    a.max_splits = splits;
    a.head_layout = decode_use_head_layout(batch, max_kv_len, T == T_auto ? 0 : (int)T) ? 1 : 0;
    a.counters = reinterpret_cast<unsigned*>(base);
    a.part_ml = reinterpret_cast<float2*>(base + kCounterBytes);
    a.part_o = reinterpret_cast<float*>(
        base + kCounterBytes + round256((size_t)batch * splits * heads * sizeof(float2)));
    // Counters start at zero for this call whatever an earlier call left behind.
    cudaError_t e = cudaMemsetAsync(base, 0, counter_bytes, stream);
    if (e != cudaSuccess) return internal_cuda_fail(e);
    e = launch_decode(a, stream);
    return e == cudaSuccess ? NC_OK : internal_cuda_fail(e);
}

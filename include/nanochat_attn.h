/*
 * nanochat_attn.h - C ABI of the B200 (sm_100a) attention hot path for the nanochat
 * inference engine: RoPE / fused RoPE + QK-RMSNorm, KV-cache append, causal prefill
 * attention on tcgen05 tensor cores, and split-KV decode attention.
 *
 * Library: libnanochat_attn_sm100.so.  Every function returns an nc_status (0 = success)
 * and is asynchronous on the given stream unless stated otherwise.  All device pointers must
 * be 16-byte aligned (cudaMalloc gives 256).  Tensors are bf16 (passed as void*), row-major:
 *   Q, K, V, caches : [rows, heads, 128]      (head_dim is fixed at 128)
 *   attention out   : [rows, heads * 128]
 * The same library also exports the reference engine's own C++ entry points
 * (namespace nanochat, see nanochat_attn_dropin.hpp), so it links in place of the
 * reference's kernels/flash_attention.cu and kernels/rope.cu.
 */
#ifndef NANOCHAT_ATTN_H
#define NANOCHAT_ATTN_H

#include <stddef.h>
#include <cuda_runtime_api.h>

#ifdef __cplusplus
extern "C" {
#endif

typedef enum nc_status {
    NC_OK = 0,
    NC_ERR_INVALID_ARG = 1,     /* bad size, null pointer, heads outside [1, 32] ([1, 31]
                                   for the decode entry points) ...                        */
    NC_ERR_MISALIGNED = 2,      /* a pointer is not 16-byte aligned                        */
    NC_ERR_CUDA = 3,            /* a CUDA runtime call failed (see nc_last_cuda_error)     */
    NC_ERR_WORKSPACE = 4,       /* workspace missing or smaller than required              */
    NC_ERR_RANGE = 5,           /* a position is beyond the RoPE table (20480 positions)   */
    NC_ERR_DEVICE_TIMEOUT = 6,  /* a kernel's bounded wait gave up (nc_device_status)      */
    NC_ERR_TOO_LARGE = 7        /* beyond the fixed scratch of nc_decode_attention_noalloc */
} nc_status;

/* Human-readable name of a status code. */
const char* nc_status_string(int status);
/* The last cudaError_t seen by this thread (0 if none). */
int nc_last_cuda_error(void);
/* Status of the most recent call made through the void-returning nanochat:: entry points
 * on this thread (those cannot return it). */
int nc_last_status(void);
/* Reads (and, if reset != 0, clears) the current device's kernel status word.  Non-zero
 * means a kernel's bounded wait gave up; bits 0x100 | tag identify the wait.  Synchronous. */
int nc_device_status(int reset);

/* Builds the fp32 cos/sin table (positions 0..20479, base 10000, 64 frequencies) on the
 * host with the reference's expression order and uploads it to the current device.
 * Synchronous.  Other entry points upload it on first use per device, so calling this is
 * optional; call it before any stream capture.
 * Replaces: kernels/rope.cu:14-30 (init_rope_tables), declared src/model.h:16. */
int nc_init_rope_tables(void);

/* In place: half-split RoPE at positions start_pos.. with one bf16 rounding.
 * Replaces: kernels/rope.cu:34-68 (apply_rope), declared src/model.h:14. */
int nc_apply_rope(void* x, int seq_len, int n_heads, int start_pos, cudaStream_t stream);

/* In place: RoPE then parameter-free RMSNorm per head (eps 1e-6), one bf16 rounding.
 * Replaces: kernels/rope.cu:74-158 (apply_rope_rmsnorm), declared src/model.h:15. */
int nc_apply_rope_rmsnorm(void* x, int seq_len, int n_heads, int start_pos,
                          cudaStream_t stream);

/* Fused prologue of one attention layer: q gets RoPE + QK-norm in place; k gets RoPE +
 * QK-norm and is written to k_cache rows [start_pos, start_pos + seq_len); v is copied to the
 * same rows of v_cache.  k and v are not modified.
 * Replaces: the two apply_rope_rmsnorm calls and the two cache-append cudaMemcpyAsync
 * calls of Model::attention, src/model.cpp:119-131. */
int nc_rope_qknorm_append(void* q, const void* k, const void* v, void* k_cache, void* v_cache,
                          int seq_len, int heads, int start_pos, cudaStream_t stream);

/* out[s, h, :] = softmax(scale * Q[s,h] . K[j,h]^T) V[j,h] over keys j < kv_len with
 * j <= s + kv_offset; fp32 softmax, bf16 output.  seq_q > 1 runs the tcgen05 prefill
 * kernel; seq_q == 1 runs the split-KV decode kernel (its partial results live in a
 * per-device workspace the library allocates on first use and grows as needed; see the
 * drop-in notes below for what that implies).  A row with
 * no visible key gets NaN, as the reference's 0/0 does.
 * Replaces: kernels/flash_attention.cu:159-171 (flash_attention), declared src/model.h:26-27;
 * called from src/model.cpp:134-136. */
int nc_flash_attention(void* out, const void* Q, const void* K, const void* V, int seq_q,
                       int kv_len, int heads, float scale, int kv_offset, cudaStream_t stream);

/* Bytes of workspace nc_decode_attention needs for this batch and bound on kv_len. */
size_t nc_decode_workspace_bytes(int batch, int max_kv_len, int heads, int split_len);

/* Batched decode step for `batch` independent sequences, one query token each.
 *   q       [batch, heads, 128]: the new tokens' queries.  If k_new/v_new are non-null, q
 *           is taken before RoPE and gets RoPE + QK-norm inside the kernel (q is not
 *           written); the new key gets RoPE + QK-norm and, with the value, is appended at
 *           row kv_len[b]-1 of sequence b's cache.  If k_new/v_new are null, q is used as
 *           given and the caches must already hold rows [0, kv_len[b]).
 *   k_caches, v_caches  device arrays [batch] of per-sequence cache bases ([rows,heads,128])
 *   kv_len  device array [batch]: keys visible to sequence b (its query sits at position
 *           kv_len[b]-1), 1 <= kv_len[b] <= max_kv_len.
 *   split_len  keys per split-KV chunk (multiple of 16) or 0 for automatic.
 *   workspace  >= nc_decode_workspace_bytes(...) bytes, zero-filled before first use and
 *           again before a call with a larger batch than any earlier call on it; it starts
 *           with (2 + batch*heads) 32-bit counters (a work queue, an exit count and one split
 *           ticket per sequence and head) that each call leaves at zero, so a call can be
 *           captured in a CUDA graph and replayed.  Calls sharing one workspace must not
 *           overlap on the GPU.  A launch whose bounded wait gave up (nc_device_status
 *           bit 0x100) can leave counters set: zero the workspace again before reusing it.
 * Replaces: the seq_len == 1 path of Model::attention (src/model.cpp:119-136): two
 * apply_rope_rmsnorm launches, two append copies and flash_attention, for one sequence. */
int nc_decode_attention(void* out, const void* q, const void* k_new, const void* v_new,
                        void* const* k_caches, void* const* v_caches, const int* kv_len,
                        int batch, int heads, float scale, int max_kv_len, int split_len,
                        void* workspace, size_t workspace_bytes, cudaStream_t stream);

/* nc_decode_attention over a paged cache.  K and V live in two pools of num_pages pages, each
 * [page_rows][heads][128] bf16 (page_rows a multiple of 16); row r of sequence b is row
 * r % page_rows of page page_table[b * pages_per_seq + r / page_rows] (page_table: device
 * int32 [batch][pages_per_seq], pages_per_seq * page_rows >= max_kv_len).  The new key and
 * value are appended at row kv_len[b] - 1 through the same table, so the caller maps a page
 * for that row before the call.  A page id outside [0, num_pages) is not dereferenced: the
 * access is skipped and bit 0x400 of the device status word is set.  Otherwise as
 * nc_decode_attention, with the same workspace rules.
 * Replaces: the contiguous per-layer KVCache buffers (src/model.h:65-73) for decode, so that a
 * sequence holds only the pages it uses.  No counterpart in the reference. */
int nc_decode_attention_paged(void* out, const void* q, const void* k_new, const void* v_new,
                              void* k_pool, void* v_pool, int num_pages, int page_rows,
                              const int* page_table, int pages_per_seq, const int* kv_len,
                              int batch, int heads, float scale, int max_kv_len, int split_len,
                              void* workspace, size_t workspace_bytes, cudaStream_t stream);

/* nc_decode_attention for a call that directly follows, on the same stream, a kernel that
 * writes none of the caches, kv_len or the two pointer arrays (typically the Q/K/V projection
 * of nc_gemm_skinny).  Small batches (the per-head layout) then launch as a programmatic
 * dependent launch: the call's CTAs start while that kernel is still running and load their
 * cache rows, lengths and cache bases before waiting for it; q, k_new, v_new and every write
 * come after the wait.  Results are those of nc_decode_attention.  Not for a call right after
 * a kernel that appends to the same caches (nc_rope_qknorm_append, another decode call): its
 * rows could be read before they are written.  No counterpart in the reference. */
int nc_decode_attention_overlap(void* out, const void* q, const void* k_new, const void* v_new,
                                void* const* k_caches, void* const* v_caches, const int* kv_len,
                                int batch, int heads, float scale, int max_kv_len, int split_len,
                                void* workspace, size_t workspace_bytes, cudaStream_t stream);

/* nc_decode_attention without the workspace argument, for callers that cannot allocate
 * device memory (an engine whose device memory is planned by an outside allocator, a host
 * binding with no device allocator to pass a workspace, or a latency-critical loop where
 * cudaMalloc's device synchronization is not acceptable).  No counterpart in the reference:
 * it is an addition of this library.  The split-KV partial results live in one fixed 8 MiB
 * device array inside the library (held by every GPU that loads it until exit), so:
 * batch <= 256 and max_kv_len <= 20480, else NC_ERR_TOO_LARGE; the split length grows as
 * needed to fit.  All calls on a device share the array and it keeps the last call's
 * contents: calls that overlap on the GPU race, so order them on one stream.  Each call first
 * clears the array's split counters with a memset on `stream`, so a call never inherits
 * counters left set by an earlier launch whose bounded wait gave up.  The first call on a
 * device sets the array up (and, with k_new, uploads the RoPE table); make it before any
 * stream capture.  Allocates nothing: no cudaMalloc, cudaFree or allocating library call. */
int nc_decode_attention_noalloc(void* out, const void* q, const void* k_new, const void* v_new,
                                void* const* k_caches, void* const* v_caches, const int* kv_len,
                                int batch, int heads, float scale, int max_kv_len,
                                cudaStream_t stream);

/* nc_rope_qknorm_append for `batch` sequences in one launch: q, k, v are [batch, seq_len,
 * heads, 128] (sequence b's chunk at rows b*seq_len..), all at positions start_pos ..
 * start_pos + seq_len - 1; sequence b's cache starts at k_slab / v_slab + b * seq_stride
 * elements (seq_stride % 8 == 0 and at least (start_pos + seq_len) * heads * 128 when
 * batch > 1), the layout nc_prefill_attention_batched reads.
 * Replaces: the same calls as nc_rope_qknorm_append (src/model.cpp:119-131), once per
 * sequence of a batched prompt pass. */
int nc_rope_qknorm_append_batched(void* q, const void* k, const void* v, void* k_slab,
                                  void* v_slab, long long seq_stride, int batch, int seq_len,
                                  int heads, int start_pos, cudaStream_t stream);

/* nc_rope_qknorm_append_paged for `batch` sequences in one launch, through a DEVICE page table
 * [batch][pages_per_seq] (the one nc_prefill_attention_paged / nc_decode_attention_paged read):
 * q, k, v are [batch, seq_len, heads, 128], all at positions start_pos .. start_pos + seq_len - 1
 * ((start_pos + seq_len - 1) / page_rows < pages_per_seq).  A page id outside [0, num_pages)
 * is not written to and sets bit 0x400 of the device status word.  No counterpart in the
 * reference. */
int nc_rope_qknorm_append_paged_batched(void* q, const void* k, const void* v, void* k_pool,
                                        void* v_pool, int num_pages, int page_rows,
                                        const int* page_table, int pages_per_seq, int batch,
                                        int seq_len, int heads, int start_pos,
                                        cudaStream_t stream);

/* Batched causal prefill (chunked, with cache offset) for `batch` sequences whose caches
 * are slices of one slab: sequence b's rows start at k_slab + b * seq_stride elements
 * (seq_stride >= rows_per_seq * heads * 128).  Sequence b's chunk of seq_q queries sits at
 * positions kv_offset[b] .. kv_offset[b] + seq_q - 1 and its keys [0, kv_offset[b] + seq_q)
 * must already be in the cache (see nc_rope_qknorm_append).
 *   q   [batch, seq_q, heads, 128] (after RoPE + QK-norm), out [batch, seq_q, heads*128].
 *   kv_offset  device array [batch].
 * Replaces: per-sequence flash_attention(seq_q, kv_len, kv_offset) calls of
 * src/model.cpp:134-136 for a chunk appended at start_pos = kv_offset. */
int nc_prefill_attention_batched(void* out, const void* q, const void* k_slab,
                                 const void* v_slab, long long seq_stride, int rows_per_seq,
                                 const int* kv_offset, int batch, int seq_q, int heads,
                                 float scale, cudaStream_t stream);

/* Paged forms of the prompt path, for caches kept in pages (see nc_decode_attention_paged):
 * pools [num_pages][page_rows][heads][128] bf16.
 *
 * nc_rope_qknorm_append_paged: as nc_rope_qknorm_append for one sequence whose cache rows are
 * the pages pages[0..n_pages) (a HOST array of page ids, in position order): position p goes
 * to row p % page_rows of page pages[p / page_rows].  Every page id the chunk
 * [start_pos, start_pos + seq_len) touches is checked on the host (NC_ERR_INVALID_ARG).
 *
 * nc_prefill_attention_paged: as nc_prefill_attention_batched with the keys and values read
 * through a device page table [batch][pages_per_seq] (page_rows a multiple of 128, so that one
 * 128-key block lies in one page).  A key block past the table row or a page id outside
 * [0, num_pages) is read as zeros and sets bit 0x400 of the device status word. */
int nc_rope_qknorm_append_paged(void* q, const void* k, const void* v, void* k_pool,
                                void* v_pool, int num_pages, int page_rows, const int* pages,
                                int n_pages, int seq_len, int heads, int start_pos,
                                cudaStream_t stream);
int nc_prefill_attention_paged(void* out, const void* q, const void* k_pool, const void* v_pool,
                               int num_pages, int page_rows, const int* page_table,
                               int pages_per_seq, const int* kv_offset, int batch, int seq_q,
                               int heads, float scale, cudaStream_t stream);

/* ----------------------------------------------------------------------------------------
 * KV cache.  One slab per layer and per K/V: [n_seqs][max_len][heads][128] bf16, allocated
 * once at full length and zero-filled (no grow-and-copy), with per-sequence lengths tracked
 * on the host and device arrays of per-sequence base pointers for the batched kernels.
 * Replaces: struct KVCache (src/model.h:65-73) and KVCache::allocate/grow/clear
 * (src/model.cpp:52-81), whose growth path reallocates and copies synchronously. */
typedef struct nc_kv_cache nc_kv_cache;

int nc_kv_cache_create(nc_kv_cache** out, int n_layers, int n_seqs, int max_len, int heads);
int nc_kv_cache_destroy(nc_kv_cache* cache);
/* Device base of sequence `seq` in layer `layer` (rows [0, max_len)). */
void* nc_kv_cache_k(nc_kv_cache* cache, int layer, int seq);
void* nc_kv_cache_v(nc_kv_cache* cache, int layer, int seq);
/* Device arrays [n_seqs] of the per-sequence bases of one layer. */
void* const* nc_kv_cache_k_table(nc_kv_cache* cache, int layer);
void* const* nc_kv_cache_v_table(nc_kv_cache* cache, int layer);
/* Elements between consecutive sequences of one slab. */
long long nc_kv_cache_seq_stride(const nc_kv_cache* cache);
int nc_kv_cache_max_len(const nc_kv_cache* cache);
/* Host-side length bookkeeping: rows filled for (layer, seq), like KVCache::current_len. */
int nc_kv_cache_len(const nc_kv_cache* cache, int layer, int seq);
int nc_kv_cache_set_len(nc_kv_cache* cache, int layer, int seq, int len);
/* Resets one sequence (seq >= 0) or all sequences (seq < 0) to length 0 in every layer,
 * like KVCache::clear (src/model.h:72).  Contents are kept. */
int nc_kv_cache_clear(nc_kv_cache* cache, int seq);

/* Prefill one sequence's chunk through the cache: RoPE + QK-norm + append of k/v at the
 * sequence's current length in `layer`, then causal attention of q over the cache; advances
 * that length by seq_len.  q is modified in place (RoPE + QK-norm).  Mirrors the
 * apply_rope_rmsnorm -> append -> flash_attention sequence of src/model.cpp:119-136. */
int nc_kv_cache_prefill(nc_kv_cache* cache, int layer, int seq, void* out, void* q,
                        const void* k, const void* v, int seq_len, float scale,
                        cudaStream_t stream);

/* One decode step for every sequence of the cache in `layer`: q/k_new/v_new are
 * [n_seqs, heads, 128] before RoPE; the new keys/values are appended at each sequence's
 * current length, which then advances by one.  Uses a workspace owned by the cache, so
 * calls on one cache must be ordered on one stream. */
int nc_kv_cache_decode(nc_kv_cache* cache, int layer, void* out, const void* q,
                       const void* k_new, const void* v_new, float scale, cudaStream_t stream);

/* ----------------------------------------------------------------------------------------
 * Skinny GEMM for the decode step: out[M, N] = epilogue(x[M, K] . w[N, K]^T) for 1 <= M <= 64
 * rows (one per sequence of a decode batch), bf16 operands, fp32 accumulation on the tcgen05
 * tensor cores, one bf16 rounding of the result.  w is a weight in the reference layout
 * W[out, in] and is streamed from HBM once; the K dimension is split across up to 12 CTAs of one
 * thread-block cluster when N alone gives too few tiles (partials are summed through
 * distributed shared memory in a fixed order: results are deterministic, no workspace).
 * Optional steps, chosen by `flags`, are fused so that each replaces a separate pass:
 *   NC_GEMM_NORM_INPUT  the product is scaled per row by rsqrt(mean(x[m,:]^2) + 1e-6), i.e.
 *                       the GEMM consumes RMSNorm(x) (kernels/rmsnorm.cu:9-56) without it
 *                       being materialised;
 *   NC_GEMM_RESIDUAL    + residual[m, n] ([M, N] bf16; may equal out), as gemm_half_residual;
 *   NC_GEMM_RELU2       relu(v)^2 (kernels/ops.cu:23-30);
 *   NC_GEMM_TANH_CAP    cap * tanh(v / cap) (kernels/ops.cu:39-46), with cap = `cap`.
 * Order: scale, residual, relu^2, tanh cap.  `seg_cols` (0 = N) splits the output into
 * N / seg_cols segments stored one after another, each [M, seg_cols]: a fused Q|K|V weight
 * then writes q, k and v as three separate [M, 2176] arrays.
 * Requirements: K % 8 == 0; x and w 16-byte aligned; out must not overlap x; `splits` 0 picks
 * the split count, else that many (clamped to [1, 12] and to the number of 64-wide K blocks).
 * Replaces: gemm_half / gemm_half_residual for M <= 16 (kernels/gemm.cu:62-166, the small-M
 * branch) at the decode call sites src/model.cpp:114-116, :139, :149-150, :153, :174-177,
 * together with the rmsnorm / relu_squared / tanh_cap launches around them. */
enum {
    NC_GEMM_NORM_INPUT = 1,
    NC_GEMM_RESIDUAL = 2,
    NC_GEMM_RELU2 = 4,
    NC_GEMM_TANH_CAP = 8
};
int nc_gemm_skinny(void* out, const void* x, const void* w, const void* residual, int M, int N,
                   int K, int flags, float cap, int seg_cols, int splits, cudaStream_t stream);

/* The same product and fused steps for any M, laid out for the prompt pass (M = prompt tokens,
 * hundreds to thousands of rows): out[M, N] = epilogue(x[M, K] . w[N, K]^T) on a persistent
 * tcgen05 kernel with 128 x 256 output tiles, both operands staged by TMA, fp32 accumulation
 * in tensor memory, one bf16 rounding.  Same flags, order and seg_cols as nc_gemm_skinny.
 * Requirements: N % 8 == 0, K % 8 == 0, seg_cols % 8 == 0; x, w, out and residual 16-byte
 * aligned; out must not overlap x (residual may equal out).  Deterministic.  M > 128 runs on
 * CTA pairs (256 x 256 tiles).  Launched as a programmatic dependent of the previous kernel
 * in the stream: its setup may overlap that kernel's tail, and it reads nothing before that
 * kernel has completed.
 * Replaces: gemm_half / gemm_half_residual for M > 16 (kernels/gemm.cu:14-51, the 128 x 128
 * CUTLASS tiles) at the prompt call sites src/model.cpp:114-116, :139, :149-150, :153, together
 * with the rmsnorm / relu_squared launches around them. */
int nc_gemm(void* out, const void* x, const void* w, const void* residual, int M, int N, int K,
            int flags, float cap, int seg_cols, cudaStream_t stream);

/* ----------------------------------------------------------------------------------------
 * The two ends of a decode step.
 * out[r, :] = RMSNorm(table[tokens[r], :]) (eps 1e-6, one bf16 rounding): the embedding gather
 * and the RMSNorm after it in one pass.  dim % 8 == 0, dim <= 8192; out and table 16-byte
 * aligned.  A token id outside [0, vocab) gives a zero row and sets bit 0x800 of the device
 * status word (nc_device_status).
 * Replaces: embedding (kernels/ops.cu:9-20) + rmsnorm (kernels/rmsnorm.cu:9-63), called at
 * src/model.cpp:158-162. */
int nc_embed_rmsnorm(void* out, const void* table, const int* tokens, int rows, int dim,
                     int vocab, cudaStream_t stream);
/* out[r] = index of the first maximum of logits[r, :] (bf16 [rows, cols], cols % 8 == 0,
 * 16-byte aligned), on the device.
 * Replaces: the greedy branch of Engine::sample (src/engine.cpp:88-95) and the device-to-host
 * copy of the logits before it. */
int nc_argmax_rows(int* out, const void* logits, int rows, int cols, cudaStream_t stream);
/* out[r] = a token drawn from row r of the logits (bf16 [rows, vocab], vocab % 8 == 0) as
 * Engine::sample does it (src/engine.cpp:62-131): temperature == 0 is greedy (nc_argmax_rows);
 * otherwise softmax of (l - max) / temperature over the whole row, the top_k largest
 * (top_k <= 1024; top_k <= 0 or >= vocab: no top-k filter), then top_p (>= 1: off) on them in
 * descending order, a renormalisation, and the first entry whose running sum exceeds
 * uniforms[r] (a device array [rows] of draws in [0, 1), which the caller generates; the
 * reference draws them from its mt19937).  With neither filter the row is sampled in index
 * order.  Equal probabilities are taken in ascending index order (the reference's sort leaves
 * their order unspecified).  With top-k, the top-p cut, the renormalisation and the running
 * sums are the reference's sequential fp32 sums; top-p over the whole row (top_k off; vocab <=
 * 65536, else NC_ERR_INVALID_ARG) finds the cut and the draw from exact sums of the
 * probabilities, without a sort; the softmax denominator is a parallel fp32 sum. */
int nc_sample_rows(int* out, const void* logits, int rows, int vocab, float temperature,
                   int top_k, float top_p, const float* uniforms, cudaStream_t stream);

#ifdef __cplusplus
}
#endif

#endif /* NANOCHAT_ATTN_H */

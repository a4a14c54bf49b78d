// TEST INFRASTRUCTURE ONLY.  Compiles the reference's own kernels where they lie
// (kernels/rope.cu, kernels/flash_attention.cu, kernels/rmsnorm.cu and kernels/ops.cu of the
// reference project, pulled in through the include path set by oracle/build_ref.py; nothing is
// copied) into oracle/_ref/, with the namespace renamed to nanochat_ref, and adds a C ABI so
// tests and bench.py's reference arm can call them through ctypes.  The RMSNorm and
// elementwise kernels serve the end-to-end greedy-decode test, where both arms run the same
// non-attention kernels and differ only in the attention path.
#include "rope.cu"
#include "flash_attention.cu"
#include "rmsnorm.cu"
#include "ops.cu"

extern "C" {

int ref_init_rope_tables(void) {
    nanochat_ref::init_rope_tables();
    return (int)cudaGetLastError();
}

// Copies the reference's device tables (d_cos_table / d_sin_table, rope.cu:10-11) out.
int ref_get_rope_tables(float* cos_out, float* sin_out, int n_pos) {
    const size_t n = (size_t)n_pos * (nanochat_ref::HEAD_DIM / 2) * sizeof(float);
    cudaError_t e = cudaMemcpyFromSymbol(cos_out, nanochat_ref::d_cos_table, n);
    if (e == cudaSuccess) e = cudaMemcpyFromSymbol(sin_out, nanochat_ref::d_sin_table, n);
    return (int)e;
}

int ref_apply_rope(void* x, int seq_len, int n_heads, int start_pos, void* stream) {
    nanochat_ref::apply_rope((nv_bfloat16*)x, seq_len, n_heads, start_pos, (cudaStream_t)stream);
    return (int)cudaGetLastError();
}

int ref_apply_rope_rmsnorm(void* x, int seq_len, int n_heads, int start_pos, void* stream) {
    nanochat_ref::apply_rope_rmsnorm((nv_bfloat16*)x, seq_len, n_heads, start_pos,
                                     (cudaStream_t)stream);
    return (int)cudaGetLastError();
}

int ref_flash_attention(void* out, const void* Q, const void* K, const void* V, int seq_q,
                        int kv_len, int heads, float scale, int kv_offset, void* stream) {
    nanochat_ref::flash_attention((nv_bfloat16*)out, (const nv_bfloat16*)Q,
                                  (const nv_bfloat16*)K, (const nv_bfloat16*)V, seq_q, kv_len,
                                  heads, scale, kv_offset, (cudaStream_t)stream);
    return (int)cudaGetLastError();
}

// kernels/rmsnorm.cu:57-61 (parameter-free RMSNorm over rows of `cols`; out may equal x).
int ref_rmsnorm(void* out, const void* x, int rows, int cols, void* stream) {
    nanochat_ref::rmsnorm((nv_bfloat16*)out, (const nv_bfloat16*)x, rows, cols, (cudaStream_t)stream);
    return (int)cudaGetLastError();
}

// kernels/ops.cu:17-19 (token-id gather from the embedding table; tokens are device ints).
int ref_embedding(void* out, const void* weight, const int* tokens, int seq_len, int n_embd,
                  void* stream) {
    nanochat_ref::embedding((nv_bfloat16*)out, (const nv_bfloat16*)weight, tokens, seq_len,
                            n_embd, (cudaStream_t)stream);
    return (int)cudaGetLastError();
}

// kernels/ops.cu:31-35 (in place max(0, x)^2).
int ref_relu_squared(void* x, int n, void* stream) {
    nanochat_ref::relu_squared((nv_bfloat16*)x, n, (cudaStream_t)stream);
    return (int)cudaGetLastError();
}

// kernels/ops.cu:46-50 (in place cap * tanh(x / cap)).
int ref_tanh_cap(void* x, int n, float cap, void* stream) {
    nanochat_ref::tanh_cap((nv_bfloat16*)x, n, cap, (cudaStream_t)stream);
    return (int)cudaGetLastError();
}

}  // extern "C"

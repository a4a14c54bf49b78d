// nanochat_attn_dropin.hpp - the reference engine's own kernel entry points, exported by
// libnanochat_attn_sm100.so with the same names, namespace, C++ linkage and argument meaning,
// so src/model.cpp links against this library instead of kernels/flash_attention.cu and
// kernels/rope.cu without source changes.
//
// The reference functions return void and never check for errors.  These keep the void
// signature; the status of the most recent call on the calling thread is available from
// nc_last_status() (nanochat_attn.h).
#pragma once

#include <cuda_bf16.h>
#include <cuda_runtime.h>

#include "nanochat_attn.h"

namespace nanochat {

// src/model.h:14 (kernels/rope.cu:34-68): in-place RoPE at positions start_pos..
void apply_rope(nv_bfloat16* x, int seq_len, int n_heads, int start_pos, cudaStream_t stream);

// src/model.h:15 (kernels/rope.cu:74-158): in-place RoPE + parameter-free QK-RMSNorm.
void apply_rope_rmsnorm(nv_bfloat16* x, int seq_len, int n_heads, int start_pos,
                        cudaStream_t stream);

// src/model.h:16 (kernels/rope.cu:14-30): builds and uploads the cos/sin table.
void init_rope_tables();

// src/model.h:26-27 (kernels/flash_attention.cu:159-171): causal attention over the cache.
void flash_attention(nv_bfloat16* out, const nv_bfloat16* Q, const nv_bfloat16* K,
                     const nv_bfloat16* V, int seq_q, int kv_len, int heads, float scale,
                     int kv_offset, cudaStream_t stream);

}  // namespace nanochat

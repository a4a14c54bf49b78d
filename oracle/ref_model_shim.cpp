// TEST INFRASTRUCTURE ONLY: a C ABI around the reference engine's own host code.
//
// oracle/build_ref.py compiles the reference's unmodified src/model.cpp and src/engine.cpp
// (with kernels/rmsnorm.cu, kernels/ops.cu and kernels/gemm.cu) together with this file twice:
//   oracle/_ref/libref_model_ref.so  with the reference's kernels/rope.cu and
//                                    kernels/flash_attention.cu (the reference as shipped);
//   oracle/_ref/libref_model_nc.so   without them, linked against libnanochat_attn_sm100.so,
//                                    which then provides nanochat::init_rope_tables,
//                                    apply_rope_rmsnorm and flash_attention (the drop-in).
// The functions below only construct the reference's Model / Engine, load a weights file in
// the reference's format (src/model.cpp:17-35) and call their public methods; nothing of the
// reference's behaviour is changed.  Exceptions become a non-zero return.
#include <cstring>
#include <exception>
#include <vector>

#include "engine.h"
#include "model.h"

using nanochat::Engine;
using nanochat::Model;

extern "C" {

// Model: construction runs init_rope_tables (src/model.cpp:83-86).
void* refm_create() {
    try {
        return new Model();
    } catch (const std::exception&) {
        return nullptr;
    }
}

int refm_load(void* m, const char* weights_path) {
    try {
        static_cast<Model*>(m)->load(weights_path);
        return 0;
    } catch (const std::exception&) {
        return 1;
    }
}

// Model::forward (src/model.cpp:156-183): `tokens` is a host array, `logits_out` device
// memory for VOCAB_SIZE bf16 values (the last position's logits).  Synchronous.
int refm_forward(void* m, const int* tokens, int seq_len, int start_pos, void* logits_out) {
    try {
        static_cast<Model*>(m)->forward(tokens, seq_len, start_pos,
                                        static_cast<nv_bfloat16*>(logits_out));
        return cudaGetLastError() == cudaSuccess ? 0 : 2;
    } catch (const std::exception&) {
        return 1;
    }
}

void refm_destroy(void* m) { delete static_cast<Model*>(m); }

// Engine (src/engine.cpp): greedy generation with temperature 0 (Engine::sample's first
// maximum, src/engine.cpp:90-97), at most max_tokens tokens (stops after token 0 or 1).
void* refe_create() {
    try {
        return new Engine();
    } catch (const std::exception&) {
        return nullptr;
    }
}

int refe_load(void* e, const char* weights_path) {
    try {
        static_cast<Engine*>(e)->load(weights_path);
        return 0;
    } catch (const std::exception&) {
        return 1;
    }
}

// Returns the number of generated tokens written to out (or -1 on failure).
int refe_generate_greedy(void* e, const int* prompt, int n_prompt, int max_tokens, int* out) {
    try {
        nanochat::SamplingParams p;
        p.temperature = 0.0f;
        p.max_tokens = max_tokens;
        std::vector<int> toks(prompt, prompt + n_prompt);
        std::vector<int> gen = static_cast<Engine*>(e)->generate(toks, p);
        std::memcpy(out, gen.data(), gen.size() * sizeof(int));
        return static_cast<int>(gen.size());
    } catch (const std::exception&) {
        return -1;
    }
}

void refe_destroy(void* e) { delete static_cast<Engine*>(e); }

}  // extern "C"

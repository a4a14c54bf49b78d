/*
 * nc_oracle.c - TEST INFRASTRUCTURE ONLY.  A CPU (fp32) restatement of the nanochat
 * reference's attention hot path, used as the parity checker by tests/,
 * __graft_entry__.smoke() and bench.py's cpu_baseline leg.  The product library never links,
 * loads or calls it.
 *
 * Parity pins: (1) the golden vectors in tests/golden/, produced by the reference's own
 * CUDA kernels (kernels/rope.cu, kernels/flash_attention.cu rebuilt for sm_100a by
 * oracle/build_ref.py) on a B200; (2) the reference kernels run side by side in the GPU tests.
 *
 * Reference files cited below are paths inside the reference project.
 * bf16 values are passed as uint16_t bit patterns; rounding is round-to-nearest-even like
 * __float2bfloat16.
 */
#include <math.h>
#include <stdint.h>
#include <stdlib.h>
#include <string.h>

#define HEAD_DIM 128
#define HALF_DIM 64

static inline float bf2f(uint16_t h) {
    uint32_t u = (uint32_t)h << 16;
    float f;
    memcpy(&f, &u, 4);
    return f;
}

static inline uint16_t f2bf(float f) {
    uint32_t u;
    memcpy(&u, &f, 4);
    if ((u & 0x7fffffffu) > 0x7f800000u) return (uint16_t)((u >> 16) | 0x40u); /* quiet NaN */
    u += 0x7fffu + ((u >> 16) & 1u);
    return (uint16_t)(u >> 16);
}

uint16_t orc_f2bf(float f) { return f2bf(f); }
float orc_bf2f(uint16_t h) { return bf2f(h); }

/* kernels/rope.cu:14-30 (init_rope_tables): fp32 host math in the same expression order. */
void orc_rope_tables(float* cos_t, float* sin_t, int max_pos) {
    for (int pos = 0; pos < max_pos; pos++) {
        for (int i = 0; i < HALF_DIM; i++) {
            float freq = 1.0f / powf(10000.0f, (2.0f * i) / HEAD_DIM);
            float angle = pos * freq;
            cos_t[pos * HALF_DIM + i] = cosf(angle);
            sin_t[pos * HALF_DIM + i] = sinf(angle);
        }
    }
}

/* Rotation of one pair (kernels/rope.cu:60-65 and :105-107): y0 = x0*c + x1*s,
 * y1 = -x0*s + x1*c, each with one fused multiply-add. */
static inline void rotate(float x0, float x1, float c, float s, float* y0, float* y1) {
    *y0 = fmaf(x0, c, x1 * s);
    *y1 = fmaf(x1, c, -(x0 * s));
}

/* kernels/rope.cu:34-68 (rope_kernel / apply_rope): in place, bf16 after rotation. */
void orc_apply_rope(uint16_t* x, int seq_len, int heads, int start_pos, const float* cos_t,
                    const float* sin_t) {
    for (int s = 0; s < seq_len; s++) {
        const int pos = start_pos + s;
        for (int h = 0; h < heads; h++) {
            uint16_t* row = x + ((size_t)s * heads + h) * HEAD_DIM;
            for (int i = 0; i < HALF_DIM; i++) {
                float y0, y1;
                rotate(bf2f(row[i]), bf2f(row[i + HALF_DIM]), cos_t[pos * HALF_DIM + i],
                       sin_t[pos * HALF_DIM + i], &y0, &y1);
                row[i] = f2bf(y0);
                row[i + HALF_DIM] = f2bf(y1);
            }
        }
    }
}

/* kernels/rope.cu:74-152 (rope_rmsnorm_kernel): rotate in fp32, sum of squares in fp32,
 * r = 1/sqrt(mean + 1e-6), one bf16 rounding of y*r.  dst may equal src. */
static void rope_norm_row(const uint16_t* src, uint16_t* dst, int pos, const float* cos_t,
                          const float* sin_t) {
    float y[HEAD_DIM];
    float ss = 0.0f;
    for (int i = 0; i < HALF_DIM; i++) {
        rotate(bf2f(src[i]), bf2f(src[i + HALF_DIM]), cos_t[pos * HALF_DIM + i],
               sin_t[pos * HALF_DIM + i], &y[i], &y[i + HALF_DIM]);
    }
    for (int i = 0; i < HEAD_DIM; i++) ss = fmaf(y[i], y[i], ss);
    const float r = 1.0f / sqrtf(ss / HEAD_DIM + 1e-6f);
    for (int i = 0; i < HEAD_DIM; i++) dst[i] = f2bf(y[i] * r);
}

void orc_apply_rope_rmsnorm(uint16_t* x, int seq_len, int heads, int start_pos,
                            const float* cos_t, const float* sin_t) {
    for (int s = 0; s < seq_len; s++)
        for (int h = 0; h < heads; h++) {
            uint16_t* row = x + ((size_t)s * heads + h) * HEAD_DIM;
            rope_norm_row(row, row, start_pos + s, cos_t, sin_t);
        }
}

/* src/model.cpp:119-131: q and k get RoPE + QK-norm, k and v land in cache rows
 * start_pos.. (the reference normalises k in its scratch buffer and then copies it). */
void orc_rope_qknorm_append(uint16_t* q, const uint16_t* k, const uint16_t* v,
                            uint16_t* k_cache, uint16_t* v_cache, int seq_len, int heads,
                            int start_pos, const float* cos_t, const float* sin_t) {
    const size_t row = (size_t)heads * HEAD_DIM;
    orc_apply_rope_rmsnorm(q, seq_len, heads, start_pos, cos_t, sin_t);
    for (int s = 0; s < seq_len; s++)
        for (int h = 0; h < heads; h++) {
            const size_t o = (size_t)s * row + (size_t)h * HEAD_DIM;
            const size_t c = (size_t)(start_pos + s) * row + (size_t)h * HEAD_DIM;
            rope_norm_row(k + o, k_cache + c, start_pos + s, cos_t, sin_t);
            memcpy(v_cache + c, v + o, HEAD_DIM * sizeof(uint16_t));
        }
}

/* kernels/flash_attention.cu:19-171: out[q,h,:] = softmax(scale * Q.K^T) V over keys
 * j < kv_len with j <= q + kv_offset (:37, :74), fp32 scores (:90), exact softmax with expf,
 * bf16 of the normalised fp32 output (:155).  A row with no visible key is 0/0 = NaN. */
static void attend_row(uint16_t* out, const uint16_t* qrow, const uint16_t* K,
                       const uint16_t* V, int n_keys, int heads, int h, float scale,
                       float* scores) {
    const size_t row = (size_t)heads * HEAD_DIM;
    float q[HEAD_DIM];
    for (int d = 0; d < HEAD_DIM; d++) q[d] = bf2f(qrow[d]);
    float m = -INFINITY;
    for (int j = 0; j < n_keys; j++) {
        const uint16_t* krow = K + (size_t)j * row + (size_t)h * HEAD_DIM;
        float dot = 0.0f;
        for (int d = 0; d < HEAD_DIM; d++) dot = fmaf(q[d], bf2f(krow[d]), dot);
        scores[j] = dot * scale;
        if (scores[j] > m) m = scores[j];
    }
    float acc[HEAD_DIM];
    for (int d = 0; d < HEAD_DIM; d++) acc[d] = 0.0f;
    float l = 0.0f;
    for (int j = 0; j < n_keys; j++) {
        const float p = expf(scores[j] - m);
        l += p;
        const uint16_t* vrow = V + (size_t)j * row + (size_t)h * HEAD_DIM;
        for (int d = 0; d < HEAD_DIM; d++) acc[d] = fmaf(p, bf2f(vrow[d]), acc[d]);
    }
    for (int d = 0; d < HEAD_DIM; d++) out[d] = f2bf(acc[d] / l);
}

void orc_flash_attention(uint16_t* out, const uint16_t* Q, const uint16_t* K,
                         const uint16_t* V, int seq_q, int kv_len, int heads, float scale,
                         int kv_offset) {
    const size_t row = (size_t)heads * HEAD_DIM;
    const long total = (long)seq_q * heads;
#pragma omp parallel
    {
        float* scores = NULL;  /* per-thread score buffer, grown on demand */
        int cap = 0;
#pragma omp for schedule(dynamic, 16)
        for (long t = 0; t < total; t++) {
            const int qi = (int)(t / heads);
            const int h = (int)(t % heads);
            int n = qi + kv_offset + 1;
            if (n > kv_len) n = kv_len;
            if (n < 0) n = 0;
            if (n > cap) {
                float* nb = (float*)realloc(scores, sizeof(float) * (size_t)(n > 64 ? n : 64));
                if (!nb) continue;
                scores = nb;
                cap = n > 64 ? n : 64;
            }
            attend_row(out + (size_t)qi * row + (size_t)h * HEAD_DIM,
                       Q + (size_t)qi * row + (size_t)h * HEAD_DIM, K, V, n, heads, h, scale,
                       scores);
        }
        free(scores);
    }
}

/* One fused decode step for `batch` sequences (src/model.cpp:119-136 with seq_len == 1):
 * q_b and k_new_b get RoPE + QK-norm at position kv_len[b]-1, k/v are appended at that row
 * of sequence b's cache, then q attends over the kv_len[b] cached keys.  q is not modified
 * (a copy is normalised), matching nc_decode_attention. */
void orc_decode_step(uint16_t* out, const uint16_t* q, const uint16_t* k_new,
                     const uint16_t* v_new, uint16_t** k_caches, uint16_t** v_caches,
                     const int* kv_len, int batch, int heads, float scale, const float* cos_t,
                     const float* sin_t) {
    const size_t row = (size_t)heads * HEAD_DIM;
    for (int b = 0; b < batch; b++) {
        const int L = kv_len[b];
        uint16_t qn[32 * HEAD_DIM];
        memcpy(qn, q + (size_t)b * row, row * sizeof(uint16_t));
        if (k_new) {
            orc_rope_qknorm_append(qn, k_new + (size_t)b * row, v_new + (size_t)b * row,
                                   k_caches[b], v_caches[b], 1, heads, L - 1, cos_t, sin_t);
        }
        orc_flash_attention(out + (size_t)b * row, qn, k_caches[b], v_caches[b], 1, L, heads,
                            scale, L - 1);
    }
}

/* ---------------------------------------------------------------------------------------
 * Sampling: Engine::sample (src/engine.cpp:88-131) for one row of bf16 logits, converted to
 * float as the engine's logits are.  temperature == 0: the first maximum (:90-96).  Otherwise,
 * in the reference's order and with its fp32 sequential sums: scaled = (l - max) / T,
 * p = expf(scaled), p /= sum (all entries, index order) (:99-110); top_k_filter: the k largest
 * (:62-68); top_p_filter: sort descending, keep entries up to and including the first whose
 * running sum exceeds top_p (:70-84); renormalise (:116-119); return the first entry whose
 * running sum exceeds r (:121-128), else the last.  r is the uniform draw (the reference draws
 * it from its mt19937).  The reference's std::partial_sort / std::sort leave the order of equal
 * probabilities unspecified; here equal values are ordered by ascending index.
 * --------------------------------------------------------------------------------------- */
typedef struct {
    float p;
    int idx;
} orc_prob;

static int prob_desc(const void* a, const void* b) {
    const orc_prob* x = (const orc_prob*)a;
    const orc_prob* y = (const orc_prob*)b;
    if (x->p > y->p) return -1;
    if (x->p < y->p) return 1;
    return x->idx - y->idx;
}

int orc_sample(const uint16_t* logits, int vocab, float temperature, int top_k, float top_p,
               float r) {
    if (temperature == 0.0f) {
        int best = 0;
        for (int i = 1; i < vocab; i++)
            if (bf2f(logits[i]) > bf2f(logits[best])) best = i;
        return best;
    }
    orc_prob* probs = (orc_prob*)malloc(sizeof(orc_prob) * (size_t)vocab);
    float max_logit = bf2f(logits[0]);
    for (int i = 1; i < vocab; i++)
        if (bf2f(logits[i]) > max_logit) max_logit = bf2f(logits[i]);
    float sum = 0.0f;
    for (int i = 0; i < vocab; i++) {
        float scaled = (bf2f(logits[i]) - max_logit) / temperature;
        probs[i].p = expf(scaled);
        probs[i].idx = i;
        sum += probs[i].p;
    }
    for (int i = 0; i < vocab; i++) probs[i].p /= sum;
    int n = vocab;
    if (top_k > 0 && top_k < n) {  /* partial sort: the k largest, in descending order */
        qsort(probs, (size_t)n, sizeof(orc_prob), prob_desc);
        n = top_k;
    }
    if (top_p < 1.0f) {
        qsort(probs, (size_t)n, sizeof(orc_prob), prob_desc);
        float cumsum = 0.0f;
        int cutoff = n;
        for (int i = 0; i < n; i++) {
            cumsum += probs[i].p;
            if (cumsum > top_p) {
                cutoff = i + 1;
                break;
            }
        }
        n = cutoff;
    }
    sum = 0.0f;
    for (int i = 0; i < n; i++) sum += probs[i].p;
    for (int i = 0; i < n; i++) probs[i].p /= sum;
    float cumsum = 0.0f;
    int chosen = probs[n - 1].idx;
    for (int i = 0; i < n; i++) {
        cumsum += probs[i].p;
        if (r < cumsum) {
            chosen = probs[i].idx;
            break;
        }
    }
    free(probs);
    return chosen;
}

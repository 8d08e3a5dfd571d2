/*
 * attn_oracle.c - CPU restatement of the gemma3.c attention hot path.
 *
 * TEST INFRASTRUCTURE ONLY: used by tests/, __graft_entry__.smoke() and the
 * bench's cpu_baseline leg as the checker.  The shipped library never links,
 * loads or calls it.
 *
 * Each function restates one step of the reference (gemma3.c, C11) in plain C
 * and cites the lines it follows.  Parity of this restatement is pinned
 * against the reference's own code compiled from its sources
 * (oracle/_ref/libgemma3_ref.so, see ref_harness.c) and against the golden
 * vectors in tests/golden/ that were produced by that build.
 *
 * Model constants (gemma3.h:36-48): 8 query heads, 4 KV heads, head_dim 256,
 * sliding window 1024, RMSNorm eps 1e-6.
 */
#include <math.h>
#include <stdint.h>
#include <stdlib.h>
#include <string.h>

#define NH 8
#define NKV 4
#define HD 256
#define WINDOW 1024

static float bf16_to_f32(uint16_t h) {
    uint32_t bits = (uint32_t)h << 16;
    float f;
    memcpy(&f, &bits, 4);
    return f;
}

/* Global iff (layer+1) % 6 == 0  (gemma3.h:347-350). */
int oracle_is_global_layer(int layer) { return (layer + 1) % 6 == 0; }

/* RoPE table [max_pos][half][cos,sin]: freq = 1/theta^(2i/d),
 * angle = (float)pos * freq  (gemma3_kernels.c:455-468). */
void oracle_rope_table(float *tab, int max_pos, int head_dim, float theta) {
    int half = head_dim / 2;
    for (int p = 0; p < max_pos; p++)
        for (int i = 0; i < half; i++) {
            float freq = 1.0f / powf(theta, (float)(2 * i) / (float)head_dim);
            float ang = (float)p * freq;
            tab[((size_t)p * half + i) * 2 + 0] = cosf(ang);
            tab[((size_t)p * half + i) * 2 + 1] = sinf(ang);
        }
}

/* In-place per-head RMSNorm with the (1 + w) Gemma gain
 * (gemma3_kernels.c:289-304). */
void oracle_rmsnorm_head(float *x, const uint16_t *w, int n, float eps) {
    float ss = 0.0f;
    for (int i = 0; i < n; i++) ss += x[i] * x[i];
    float r = 1.0f / sqrtf(ss / n + eps);
    for (int i = 0; i < n; i++) x[i] = x[i] * r * (1.0f + bf16_to_f32(w[i]));
}

/* Rotate-half RoPE from the table: pairs (i, i+half)
 * (gemma3_kernels.c:470-484). */
void oracle_rope_apply(float *x, const float *tab, int head_dim, int pos) {
    int half = head_dim / 2;
    const float *t = tab + (size_t)pos * half * 2;
    for (int i = 0; i < half; i++) {
        float c = t[2 * i], s = t[2 * i + 1];
        float a = x[i], b = x[i + half];
        x[i] = a * c - b * s;
        x[i + half] = a * s + b * c;
    }
}

/* Cache row written for position pos: global layers append at pos, local
 * layers use the 1024-row ring at pos % 1024 (gemma3_transformer.c:240-248). */
int oracle_cache_slot(int is_global, int pos) {
    return is_global ? pos : pos % WINDOW;
}

/* Number of cache rows attended at position pos: pos+1 on global layers,
 * min(pos+1, 1024) ring rows on local layers (gemma3_transformer.c:319-346).
 * Every attended row is unmasked (the mask written there is all zeros). */
int oracle_attn_rows(int is_global, int pos) {
    if (is_global) return pos + 1;
    return pos < WINDOW ? pos + 1 : WINDOW;
}

/* Softmax: max, exp(x-max) with running sum, multiply by 1/sum
 * (gemma3_kernels.c:396-415). */
static void softmax_inplace(float *x, int n) {
    float m = x[0];
    for (int i = 1; i < n; i++) m = x[i] > m ? x[i] : m;
    float s = 0.0f;
    for (int i = 0; i < n; i++) { x[i] = expf(x[i] - m); s += x[i]; }
    float inv = 1.0f / s;
    for (int i = 0; i < n; i++) x[i] *= inv;
}

/* GQA over an fp32 cache laid out [row][kv_head][256]; query head h reads
 * kv head h / (NH/NKV) (gemma3_kernels.c:527-597).  scores: [rows] scratch. */
void oracle_gqa(float *out, const float *q, const float *kc, const float *vc,
                int rows, float scale, float *scores) {
    int group = NH / NKV, stride = NKV * HD;
    for (int h = 0; h < NH; h++) {
        int g = h / group;
        const float *qh = q + h * HD;
        float *oh = out + h * HD;
        for (int r = 0; r < rows; r++) {
            const float *k = kc + (size_t)r * stride + g * HD;
            float d = 0.0f;
            for (int i = 0; i < HD; i++) d += qh[i] * k[i];
            scores[r] = d * scale;
        }
        softmax_inplace(scores, rows);
        for (int i = 0; i < HD; i++) oh[i] = 0.0f;
        for (int r = 0; r < rows; r++) {
            const float *v = vc + (size_t)r * stride + g * HD;
            float w = scores[r];
            for (int i = 0; i < HD; i++) oh[i] += w * v[i];
        }
    }
}

/* The per-token attention core for T consecutive tokens of one layer
 * (gemma3_transformer.c:641-692): QK-norm (if both gains are given), RoPE,
 * append to the cache (kc/vc: fp32 [rows][4][256], rows = max_seq for a
 * global layer and 1024 for a local one), then GQA over the attended rows
 * with scale 1/sqrt(256).  Q and K are normalised/rotated in place. */
void oracle_attn_core_tokens(float *kc, float *vc, float *Q, float *K,
                             const float *V, const uint16_t *q_norm,
                             const uint16_t *k_norm, const float *rope,
                             int is_global, int T, int start_pos, int max_seq,
                             float *out) {
    float *scores = (float *)malloc((size_t)(is_global ? max_seq : WINDOW) * sizeof(float));
    float scale = 1.0f / sqrtf((float)HD);
    for (int t = 0; t < T; t++) {
        int pos = start_pos + t;
        float *q = Q + (size_t)t * NH * HD;
        float *k = K + (size_t)t * NKV * HD;
        const float *v = V + (size_t)t * NKV * HD;
        if (q_norm && k_norm) {
            for (int h = 0; h < NH; h++) oracle_rmsnorm_head(q + h * HD, q_norm, HD, 1e-6f);
            for (int h = 0; h < NKV; h++) oracle_rmsnorm_head(k + h * HD, k_norm, HD, 1e-6f);
        }
        for (int h = 0; h < NH; h++) oracle_rope_apply(q + h * HD, rope, HD, pos);
        for (int h = 0; h < NKV; h++) oracle_rope_apply(k + h * HD, rope, HD, pos);
        int slot = oracle_cache_slot(is_global, pos);
        memcpy(kc + (size_t)slot * NKV * HD, k, NKV * HD * sizeof(float));
        memcpy(vc + (size_t)slot * NKV * HD, v, NKV * HD * sizeof(float));
        oracle_gqa(out + (size_t)t * NH * HD, q, kc, vc,
                   oracle_attn_rows(is_global, pos), scale, scores);
    }
    free(scores);
}

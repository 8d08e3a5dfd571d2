/*
 * ref_harness.c - exposes the gemma3.c reference attention path as plain C
 * entry points so that the test-suite and the CPU baseline can call the
 * reference's OWN code through ctypes.
 *
 * TEST INFRASTRUCTURE ONLY.  This translation unit textually includes the
 * reference's gemma3_transformer.c (from REF_DIR, read-only; nothing is copied
 * into this repository) so that its file-static helpers -- cache_kv
 * (gemma3_transformer.c:236-251) and layer_attention (:258-356) -- become
 * reachable.  It is linked with the reference's gemma3_kernels.c and
 * gemma3_threads.c compiled with the `make blas-threads` flags
 * (Makefile:62-73).  Output goes to oracle/_ref/ only.
 */
#include "gemma3_transformer.c"

#include <stdint.h>

/* ---------------------------------------------------------------------- */
/* Configuration identical to default_config() (gemma3.c:94-109).          */
/* ---------------------------------------------------------------------- */
static gemma3_config harness_cfg(int max_context) {
    gemma3_config c;
    c.vocab_size = GEMMA3_VOCAB_SIZE;
    c.hidden_size = GEMMA3_HIDDEN_SIZE;
    c.intermediate_size = GEMMA3_INTERMEDIATE_SIZE;
    c.num_layers = GEMMA3_NUM_LAYERS;
    c.num_heads = GEMMA3_NUM_HEADS;
    c.num_kv_heads = GEMMA3_NUM_KV_HEADS;
    c.head_dim = GEMMA3_HEAD_DIM;
    c.max_context = max_context;
    c.sliding_window = GEMMA3_SLIDING_WINDOW;
    c.rmsnorm_eps = GEMMA3_RMSNORM_EPS;
    c.rope_theta_local = GEMMA3_ROPE_THETA_LOCAL;
    c.rope_theta_global = GEMMA3_ROPE_THETA_GLOBAL;
    return c;
}

int ref_is_global_layer(int layer) { return gemma3_is_global_layer(layer); }

/* ---------------------------------------------------------------------- */
/* One layer's KV cache, sized exactly as gemma3_kv_cache_alloc does       */
/* (gemma3_transformer.c:189-200): max_seq rows for a global layer, the    */
/* sliding window (1024 rows) for a local one; fp32 [rows][4][256].        */
/* ---------------------------------------------------------------------- */
void *ref_layer_cache_new(int is_global, int max_seq) {
    layer_kv_cache *c = (layer_kv_cache *)calloc(1, sizeof(layer_kv_cache));
    if (!c) return NULL;
    int rows = is_global ? max_seq : GEMMA3_SLIDING_WINDOW;
    size_t kv = (size_t)GEMMA3_NUM_KV_HEADS * GEMMA3_HEAD_DIM;
    c->k = (float *)calloc((size_t)rows * kv, sizeof(float));
    c->v = (float *)calloc((size_t)rows * kv, sizeof(float));
    if (!c->k || !c->v) { free(c->k); free(c->v); free(c); return NULL; }
    return c;
}
void ref_layer_cache_free(void *p) {
    layer_kv_cache *c = (layer_kv_cache *)p;
    if (!c) return;
    free(c->k); free(c->v); free(c);
}
float *ref_layer_cache_k(void *p) { return ((layer_kv_cache *)p)->k; }
float *ref_layer_cache_v(void *p) { return ((layer_kv_cache *)p)->v; }
int ref_layer_cache_pos(void *p) { return ((layer_kv_cache *)p)->pos; }

/* ---------------------------------------------------------------------- */
/* The attention core for T consecutive tokens of one layer: the body of   */
/* the batched-prefill token loop (gemma3_transformer.c:641-692), which is */
/* also what layer_attention does between its projections (:294-352).      */
/* Q [T][2048], K [T][1024] are overwritten with their normed+roped form,  */
/* exactly as the reference does in place; V [T][1024] is read only.       */
/* ---------------------------------------------------------------------- */
void ref_attn_core_tokens(void *cache_p, float *Q, float *K, float *V,
                          const uint16_t *q_norm, const uint16_t *k_norm,
                          const float *rope_freqs, int is_global, int T,
                          int start_pos, int max_seq, float *out) {
    layer_kv_cache *cache = (layer_kv_cache *)cache_p;
    gemma3_config cfg_v = harness_cfg(max_seq);
    const gemma3_config *cfg = &cfg_v;
    int num_heads = cfg->num_heads, num_kv_heads = cfg->num_kv_heads;
    int head_dim = cfg->head_dim;
    int q_size = num_heads * head_dim, kv_size = num_kv_heads * head_dim;
    float *mask = (float *)malloc((size_t)max_seq * sizeof(float));
    float *scores = (float *)malloc((size_t)max_seq * sizeof(float));
    float scale = 1.0f / sqrtf((float)head_dim);
    for (int i = 0; i < T; i++) {
        int pos = start_pos + i;
        float *qi = Q + (size_t)i * q_size;
        float *ki = K + (size_t)i * kv_size;
        float *vi = V + (size_t)i * kv_size;
        if (q_norm && k_norm) {
            for (int h = 0; h < num_heads; h++)
                gemma3_rmsnorm_bf16(qi + h * head_dim, qi + h * head_dim, q_norm,
                                    head_dim, cfg->rmsnorm_eps);
            for (int h = 0; h < num_kv_heads; h++)
                gemma3_rmsnorm_bf16(ki + h * head_dim, ki + h * head_dim, k_norm,
                                    head_dim, cfg->rmsnorm_eps);
        }
        for (int h = 0; h < num_heads; h++)
            gemma3_rope_apply_precomputed(qi + h * head_dim, rope_freqs, head_dim, pos);
        for (int h = 0; h < num_kv_heads; h++)
            gemma3_rope_apply_precomputed(ki + h * head_dim, rope_freqs, head_dim, pos);
        cache_kv(cache, ki, vi, kv_size, is_global, cfg->sliding_window, pos);
        int seq_len;
        if (is_global) {
            seq_len = pos + 1;
            gemma3_causal_mask(mask, seq_len, pos);
        } else {
            int window = cfg->sliding_window;
            seq_len = (pos < window) ? pos + 1 : window;
            for (int s = 0; s < seq_len; s++) mask[s] = 0.0f;
        }
        gemma3_gqa(out + (size_t)i * q_size, qi, cache->k, cache->v, num_heads,
                   num_kv_heads, seq_len, head_dim, scale, mask, scores);
    }
    free(mask);
    free(scores);
}

/* Bare gemma3_gqa over an externally-filled fp32 cache (decode step only). */
void ref_gqa(float *out, const float *q, const float *kc, const float *vc,
             int seq_len) {
    float *mask = (float *)calloc((size_t)seq_len, sizeof(float));
    float *scores = (float *)malloc((size_t)seq_len * sizeof(float));
    gemma3_gqa(out, q, kc, vc, GEMMA3_NUM_HEADS, GEMMA3_NUM_KV_HEADS, seq_len,
               GEMMA3_HEAD_DIM, 1.0f / sqrtf((float)GEMMA3_HEAD_DIM), mask, scores);
    free(mask);
    free(scores);
}

/* ---------------------------------------------------------------------- */
/* The reference's layer_attention (gemma3_transformer.c:258-356) for T     */
/* consecutive tokens, with the BF16 projections.  Besides the layer       */
/* output [T][2560] it returns what the device path needs to be compared:  */
/* the raw projections q/k/v (pre-norm, same matvec as inside              */
/* layer_attention: matvec_bf16_dispatch with no pool) and the attention   */
/* output attn [T][2048] (the o_proj input).                               */
/* ---------------------------------------------------------------------- */
void ref_layer_attention_tokens(float *out, const float *x, const uint16_t *wq,
                                const uint16_t *wk, const uint16_t *wv,
                                const uint16_t *wo, const uint16_t *q_norm,
                                const uint16_t *k_norm, void *cache_p,
                                const float *rope_freqs, int layer_idx, int T,
                                int start_pos, int max_seq, float *q_raw,
                                float *k_raw, float *v_raw, float *attn) {
    layer_kv_cache *cache = (layer_kv_cache *)cache_p;
    gemma3_config cfg = harness_cfg(max_seq);
    int H = cfg.hidden_size, qs = cfg.num_heads * cfg.head_dim;
    int kvs = cfg.num_kv_heads * cfg.head_dim;
    float *qb = (float *)malloc(qs * sizeof(float));
    float *kb = (float *)malloc(kvs * sizeof(float));
    float *vb = (float *)malloc(kvs * sizeof(float));
    float *ab = (float *)malloc(qs * sizeof(float));
    float *mask = (float *)malloc((size_t)max_seq * sizeof(float));
    float *scores = (float *)malloc((size_t)max_seq * sizeof(float));
    float *tmp = (float *)malloc((size_t)cfg.intermediate_size * sizeof(float));
    for (int i = 0; i < T; i++) {
        const float *xi = x + (size_t)i * H;
        if (q_raw) matvec_bf16_dispatch(q_raw + (size_t)i * qs, wq, xi, qs, H, tmp, NULL);
        if (k_raw) matvec_bf16_dispatch(k_raw + (size_t)i * kvs, wk, xi, kvs, H, tmp, NULL);
        if (v_raw) matvec_bf16_dispatch(v_raw + (size_t)i * kvs, wv, xi, kvs, H, tmp, NULL);
        layer_attention(out + (size_t)i * H, xi, wq, wk, wv, wo, q_norm, k_norm,
                        cache, qb, kb, vb, ab, mask, scores, tmp, rope_freqs,
                        NULL, &cfg, layer_idx, start_pos + i);
        if (attn) memcpy(attn + (size_t)i * qs, ab, qs * sizeof(float));
    }
    free(qb); free(kb); free(vb); free(ab); free(mask); free(scores); free(tmp);
}

/* ---------------------------------------------------------------------- */
/* The reference's SafeTensors loader: st_load (gemma3_safetensors.c:393-486) */
/* and gemma3_load_weights (:651-713), declared the way gemma3.c:49-55     */
/* declares them.  ref_st_load_slots fills, in gemma3_weights_t order,      */
/* slots[0] = embed_tokens, slots[1 + 13 l + j] = layer l's j-th weight     */
/* (input_layernorm, q/k/v/o_proj, q/k_norm, post_attention_layernorm,      */
/* gate/up/down_proj, pre/post_feedforward_layernorm), slots[1 + 13 * 34] = */
/* the final norm: the pointers the reference model would read (NULL where  */
/* the loader found no tensor).  Returns a handle for ref_st_free, or NULL  */
/* when the loader fails.                                                   */
/* ---------------------------------------------------------------------- */
typedef struct st_context st_context;
st_context *st_load(const char *model_dir);
void st_free(st_context *ctx);
gemma3_weights_t *gemma3_load_weights(st_context *st);
void gemma3_free_weights(gemma3_weights_t *w);

typedef struct { st_context *st; gemma3_weights_t *w; } ref_st_handle;

int ref_st_num_slots(void) { return 2 + 13 * GEMMA3_NUM_LAYERS; }

void *ref_st_load_slots(const char *dir, const uint16_t **slots) {
    st_context *st = st_load(dir);
    if (!st) return NULL;
    gemma3_weights_t *w = gemma3_load_weights(st);
    if (!w) { st_free(st); return NULL; }
    slots[0] = w->embed_tokens;
    for (int l = 0; l < GEMMA3_NUM_LAYERS; l++) {
        const uint16_t **s = slots + 1 + 13 * l;
        s[0] = w->layers[l].input_layernorm;
        s[1] = w->layers[l].q_proj;
        s[2] = w->layers[l].k_proj;
        s[3] = w->layers[l].v_proj;
        s[4] = w->layers[l].o_proj;
        s[5] = w->layers[l].q_norm;
        s[6] = w->layers[l].k_norm;
        s[7] = w->layers[l].post_attention_layernorm;
        s[8] = w->layers[l].gate_proj;
        s[9] = w->layers[l].up_proj;
        s[10] = w->layers[l].down_proj;
        s[11] = w->layers[l].pre_feedforward_layernorm;
        s[12] = w->layers[l].post_feedforward_layernorm;
    }
    slots[1 + 13 * GEMMA3_NUM_LAYERS] = w->norm;
    ref_st_handle *h = (ref_st_handle *)malloc(sizeof(ref_st_handle));
    h->st = st;
    h->w = w;
    return h;
}

void ref_st_free(void *p) {
    ref_st_handle *h = (ref_st_handle *)p;
    if (!h) return;
    gemma3_free_weights(h->w);
    st_free(h->st);
    free(h);
}

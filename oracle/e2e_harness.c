/*
 * e2e_harness.c - end-to-end greedy decoding on a random-init Gemma-3-4B,
 * with and without the B200 attention path.  TEST INFRASTRUCTURE ONLY.
 *
 * Arm "reference": the reference's own gemma3_transformer_prefill for the
 * prompt (gemma3_transformer.c:791-825) and gemma3_transformer_forward
 * (:400-512) for every generated token, host KV cache.
 * Arm "cuda": the same model and the same reference kernels for everything
 * except the attention core, which goes through include/gemma3_cuda.h the way
 * the USE_CUDA hook does it: the prompt with one gemma3_cuda_attn_prefill per
 * layer (replacing the token loop of gemma3_transformer.c:641-692), every
 * generated token with gemma3_cuda_attn_decode (replacing :294-352).  The
 * layer structure around the call restates gemma3_transformer_forward
 * (:427-499): input norm, q/k/v matvec, attention, o_proj, post-attention
 * norm + residual, pre-FFN norm, GELU MLP (layer_mlp, :362-398), post-FFN
 * norm + residual; final norm and tied-embedding logits (:502-509).
 *
 * Arm "cuda, all blocks" (use_cuda 2): every transformer block on the device
 * through gemma3_cuda_prefill_forward / gemma3_cuda_forward (projections,
 * norms, residuals and MLP included); embeddings, final norm and logits stay
 * on the host.  Arm "cuda, greedy" (use_cuda 3): token ids in, token ids out
 * through gemma3_cuda_prefill_greedy / gemma3_cuda_greedy_step.
 *
 * Weights are random BF16 (truncated fp32 draws): projections and
 * embeddings ~N(0, 0.02), norm weights ~N(0, 0.1) (gain 1+w), drawn with a
 * counter-based generator (splitmix64 + Box-Muller) on the thread pool.
 */
#include "gemma3_transformer.c"

#include <stdint.h>

#include "gemma3_cuda.h"

typedef struct {
    uint16_t *data;
    size_t n;
    uint64_t seed;
    float std;
} fill_task;

static uint64_t sm64(uint64_t x) {
    x += 0x9E3779B97F4A7C15ull;
    x = (x ^ (x >> 30)) * 0xBF58476D1CE4E5B9ull;
    x = (x ^ (x >> 27)) * 0x94D049BB133111EBull;
    return x ^ (x >> 31);
}

static void fill_worker(void *arg, int tid, int nth) {
    fill_task *t = (fill_task *)arg;
    size_t pairs = (t->n + 1) / 2, chunk = (pairs + nth - 1) / nth;
    size_t lo = (size_t)tid * chunk, hi = lo + chunk < pairs ? lo + chunk : pairs;
    for (size_t i = lo; i < hi; i++) {
        uint64_t r = sm64(t->seed ^ (i * 0xD1B54A32D192ED03ull));
        float u1 = ((float)(r >> 40) + 0.5f) * (1.0f / 16777216.0f);
        float u2 = (float)(r & 0xFFFFFF) * (1.0f / 16777216.0f);
        float rad = sqrtf(-2.0f * logf(u1)) * t->std;
        float a = rad * cosf(6.2831853f * u2), b = rad * sinf(6.2831853f * u2);
        t->data[2 * i] = gemma3_f32_to_bf16_single(a);
        if (2 * i + 1 < t->n) t->data[2 * i + 1] = gemma3_f32_to_bf16_single(b);
    }
}

static uint16_t *fill(gemma3_thread_pool *pool, size_t n, uint64_t seed, float std) {
    uint16_t *p = (uint16_t *)malloc(n * sizeof(uint16_t));
    if (!p) return NULL;
    fill_task t = {p, n, seed, std};
    gemma3_thread_pool_run(pool, fill_worker, &t);
    return p;
}

static gemma3_config e2e_cfg(int max_context) {
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

static gemma3_weights_t *make_weights(gemma3_thread_pool *pool, uint64_t seed) {
    gemma3_weights_t *w = (gemma3_weights_t *)calloc(1, sizeof(gemma3_weights_t));
    const size_t H = GEMMA3_HIDDEN_SIZE, I = GEMMA3_INTERMEDIATE_SIZE;
    const size_t QS = GEMMA3_NUM_HEADS * GEMMA3_HEAD_DIM, KS = GEMMA3_NUM_KV_HEADS * GEMMA3_HEAD_DIM;
    uint64_t s = seed * 1000003ull;
    w->embed_tokens = fill(pool, (size_t)GEMMA3_VOCAB_SIZE * H, s++, 0.02f);
    for (int l = 0; l < GEMMA3_NUM_LAYERS; l++) {
        w->layers[l].input_layernorm = fill(pool, H, s++, 0.1f);
        w->layers[l].q_proj = fill(pool, QS * H, s++, 0.02f);
        w->layers[l].k_proj = fill(pool, KS * H, s++, 0.02f);
        w->layers[l].v_proj = fill(pool, KS * H, s++, 0.02f);
        w->layers[l].o_proj = fill(pool, H * QS, s++, 0.02f);
        w->layers[l].q_norm = fill(pool, GEMMA3_HEAD_DIM, s++, 0.1f);
        w->layers[l].k_norm = fill(pool, GEMMA3_HEAD_DIM, s++, 0.1f);
        w->layers[l].post_attention_layernorm = fill(pool, H, s++, 0.1f);
        w->layers[l].gate_proj = fill(pool, I * H, s++, 0.02f);
        w->layers[l].up_proj = fill(pool, I * H, s++, 0.02f);
        w->layers[l].down_proj = fill(pool, H * I, s++, 0.02f);
        w->layers[l].pre_feedforward_layernorm = fill(pool, H, s++, 0.1f);
        w->layers[l].post_feedforward_layernorm = fill(pool, H, s++, 0.1f);
    }
    w->norm = fill(pool, H, s++, 0.1f);
    return w;
}

static void free_weights(gemma3_weights_t *w) {
    free((void *)w->embed_tokens);
    for (int l = 0; l < GEMMA3_NUM_LAYERS; l++) {
        const uint16_t *ps[] = {w->layers[l].input_layernorm, w->layers[l].q_proj, w->layers[l].k_proj,
                                w->layers[l].v_proj, w->layers[l].o_proj, w->layers[l].q_norm,
                                w->layers[l].k_norm, w->layers[l].post_attention_layernorm,
                                w->layers[l].gate_proj, w->layers[l].up_proj, w->layers[l].down_proj,
                                w->layers[l].pre_feedforward_layernorm, w->layers[l].post_feedforward_layernorm};
        for (size_t i = 0; i < sizeof ps / sizeof ps[0]; i++) free((void *)ps[i]);
    }
    free((void *)w->norm);
    free(w);
}

static float *g_top_out = NULL;  /* optional top-1 logit per step */

static void top2(const float *x, int n, int *arg, float *margin) {
    int a = gemma3_argmax(x, n);
    float best = x[a], second = -INFINITY;
    for (int i = 0; i < n; i++)
        if (i != a && x[i] > second) second = x[i];
    *arg = a;
    *margin = best - second;
    if (g_top_out) *g_top_out++ = best;
}

/* Everything of one layer after attention (gemma3_transformer.c:463-498):
 * o_proj, post-attention norm + residual, pre-FFN norm, MLP, post-FFN norm
 * + residual.  x [H] is updated in place. */
static void layer_tail(float *x, const float *attn, const gemma3_weights_t *w, int l, activation_buffers *buf,
                       const gemma3_config *cfg, gemma3_thread_pool *pool) {
    const int H = cfg->hidden_size, QS = cfg->num_heads * cfg->head_dim;
    matvec_bf16_dispatch(buf->proj_out, w->layers[l].o_proj, attn, H, QS, buf->matvec_tmp, pool);
    gemma3_rmsnorm_bf16_inplace(buf->proj_out, w->layers[l].post_attention_layernorm, H, cfg->rmsnorm_eps);
    gemma3_vec_add(x, x, buf->proj_out, H);
    gemma3_rmsnorm_bf16(buf->x_norm, x, w->layers[l].pre_feedforward_layernorm, H, cfg->rmsnorm_eps);
    layer_mlp(buf->mlp_out, buf->x_norm, w->layers[l].gate_proj, w->layers[l].up_proj, w->layers[l].down_proj,
              buf->mlp_gate, buf->mlp_up, buf->matvec_tmp, pool, cfg, l, 0);
    gemma3_rmsnorm_bf16_inplace(buf->mlp_out, w->layers[l].post_feedforward_layernorm, H, cfg->rmsnorm_eps);
    gemma3_vec_add(x, x, buf->mlp_out, H);
}

static void logits_of(float *logits, const float *x, const gemma3_weights_t *w, activation_buffers *buf,
                      const gemma3_config *cfg, gemma3_thread_pool *pool) {
    gemma3_rmsnorm_bf16(buf->x_norm, x, w->norm, cfg->hidden_size, cfg->rmsnorm_eps);
    matvec_bf16_dispatch(logits, w->embed_tokens, buf->x_norm, cfg->vocab_size, cfg->hidden_size, buf->matvec_tmp,
                         pool);
}

/*
 * Runs one arm.  use_cuda: 0 = reference forward, 1 = device attention path,
 * 2 = all transformer blocks on the device, 3 = greedy decoding on the device
 * (kv_dtype GEMMA3_CUDA_KV_F32 / _BF16).  Prompt = n_prompt uniform token ids
 * in [0, vocab) from `seed`; then n_steps greedy tokens.  Writes the generated
 * tokens, the top-1 minus top-2 logit margin and (top_out, may be NULL) the
 * top-1 logit of each step.  Returns 0, or a negative gemma3_error.
 */
int e2e_greedy(int n_prompt, int n_steps, uint64_t seed, int use_cuda, int kv_dtype, int *tokens_out,
               float *margins_out, float *top_out) {
    g_top_out = top_out;
    const int max_ctx = n_prompt + n_steps + 1;
    gemma3_config cfg_v = e2e_cfg(max_ctx);
    const gemma3_config *cfg = &cfg_v;
    const int H = cfg->hidden_size, QS = cfg->num_heads * cfg->head_dim, KS = cfg->num_kv_heads * cfg->head_dim;
    gemma3_thread_pool *pool = gemma3_thread_pool_create(0);
    gemma3_weights_t *w = make_weights(pool, seed);
    activation_buffers *buf = alloc_buffers(cfg);
    float *rope_l = (float *)malloc((size_t)max_ctx * cfg->head_dim * sizeof(float));
    float *rope_g = (float *)malloc((size_t)max_ctx * cfg->head_dim * sizeof(float));
    gemma3_rope_precompute(rope_l, max_ctx, cfg->head_dim, cfg->rope_theta_local);
    gemma3_rope_precompute(rope_g, max_ctx, cfg->head_dim, cfg->rope_theta_global);
    float *logits = (float *)malloc((size_t)cfg->vocab_size * sizeof(float));
    int *prompt = (int *)malloc(n_prompt * sizeof(int));
    for (int i = 0; i < n_prompt; i++) prompt[i] = (int)(sm64(seed * 7919ull + i) % (uint64_t)cfg->vocab_size);
    int rc = 0;

    if (!use_cuda) {
        gemma3_kv_cache *cache = gemma3_kv_cache_alloc(cfg, max_ctx);
        int pos = 0, tok = 0;
        /* the prompt goes through the reference's own prefill, as gemma3_generate
         * does (gemma3.c:328 -> gemma3_transformer_prefill, batched sgemm in a
         * USE_BLAS build, gemma3_transformer.c:791-825) */
        gemma3_transformer_prefill(logits, prompt, n_prompt, 0, w, cache, buf, cfg, rope_l, rope_g, pool);
        pos = n_prompt;
        for (int s = 0; s < n_steps; s++, pos++) {
            top2(logits, cfg->vocab_size, &tok, &margins_out[s]);
            tokens_out[s] = tok;
            gemma3_transformer_forward(logits, tok, pos, w, cache, buf, cfg, 1, rope_l, rope_g, pool);
        }
        gemma3_kv_cache_free(cache);
    } else {
        gemma3_cuda_config cc;
        gemma3_cuda_config_default(&cc);
        cc.max_context = max_ctx;
        cc.max_prefill = n_prompt;
        cc.kv_dtype = kv_dtype;
        gemma3_cuda_ctx *ctx = gemma3_cuda_init(&cc);
        if (!ctx || gemma3_cuda_upload_rope(ctx, rope_l, rope_g, max_ctx, cfg->head_dim)) {
            fprintf(stderr, "e2e: %s\n", gemma3_cuda_last_error());
            rc = GEMMA3_CUDA_ERR_GENERATION_FAILED;
            goto done;
        }
        for (int l = 0; l < cfg->num_layers; l++)
            gemma3_cuda_set_qk_norm(ctx, l, w->layers[l].q_norm, w->layers[l].k_norm);
        if (use_cuda >= 2) {
            /* every block on the device; embeddings, final norm and logits on the host
             * (use_cuda 2) or on the device too (use_cuda 3) */
            for (int l = 0; l < cfg->num_layers && !rc; l++) {
                const gemma3_cuda_layer_weights lw = {
                    w->layers[l].input_layernorm, w->layers[l].q_proj, w->layers[l].k_proj, w->layers[l].v_proj,
                    w->layers[l].o_proj, w->layers[l].q_norm, w->layers[l].k_norm,
                    w->layers[l].post_attention_layernorm, w->layers[l].gate_proj, w->layers[l].up_proj,
                    w->layers[l].down_proj, w->layers[l].pre_feedforward_layernorm,
                    w->layers[l].post_feedforward_layernorm};
                rc = gemma3_cuda_set_layer_weights(ctx, l, &lw);
            }
            float *X = (float *)malloc((size_t)n_prompt * H * sizeof(float));
            const float es = sqrtf((float)H);
            for (int i = 0; i < n_prompt; i++) {
                gemma3_embed_bf16(X + (size_t)i * H, w->embed_tokens, prompt[i], H);
                for (int j = 0; j < H; j++) X[(size_t)i * H + j] *= es;
            }
            if (use_cuda == 3) {
                /* token ids in, token ids out: embedding, blocks, final norm, logits and argmax on the device */
                if (!rc) rc = gemma3_cuda_set_embeddings(ctx, w->embed_tokens, cfg->vocab_size, w->norm);
                int tok = 0, seq = 0, pos = n_prompt;
                float top = 0.f;
                if (!rc) rc = gemma3_cuda_prefill_greedy(ctx, 0, prompt, n_prompt, 0, &tok, &top);
                for (int s = 0; s < n_steps && !rc; s++, pos++) {
                    tokens_out[s] = tok;
                    margins_out[s] = 0.f;
                    if (g_top_out) *g_top_out++ = top;
                    rc = gemma3_cuda_greedy_step(ctx, 1, &seq, &pos, &tok, &tok, &top);
                }
            } else {
                if (!rc) rc = gemma3_cuda_prefill_forward(ctx, 0, X, n_prompt, 0);
                if (!rc) logits_of(logits, X + (size_t)(n_prompt - 1) * H, w, buf, cfg, pool);
                int pos = n_prompt, tok = 0, seq = 0;
                for (int s = 0; s < n_steps && !rc; s++, pos++) {
                    top2(logits, cfg->vocab_size, &tok, &margins_out[s]);
                    tokens_out[s] = tok;
                    float *x = buf->x;
                    gemma3_embed_bf16(x, w->embed_tokens, tok, H);
                    for (int j = 0; j < H; j++) x[j] *= es;
                    rc = gemma3_cuda_forward(ctx, 1, &seq, &pos, x);
                    if (!rc) logits_of(logits, x, w, buf, cfg, pool);
                }
            }
            if (rc) fprintf(stderr, "e2e: %s\n", gemma3_cuda_last_error());
            free(X);
            gemma3_cuda_free(ctx);
            goto done;
        }
        /* prompt: per layer, q/k/v for every token, one prefill call, then the tail */
        float *X = (float *)malloc((size_t)n_prompt * H * sizeof(float));
        float *Q = (float *)malloc((size_t)n_prompt * QS * sizeof(float));
        float *K = (float *)malloc((size_t)n_prompt * KS * sizeof(float));
        float *V = (float *)malloc((size_t)n_prompt * KS * sizeof(float));
        float *A = (float *)malloc((size_t)n_prompt * QS * sizeof(float));
        const float es = sqrtf((float)H);
        for (int i = 0; i < n_prompt; i++) {
            gemma3_embed_bf16(X + (size_t)i * H, w->embed_tokens, prompt[i], H);
            for (int j = 0; j < H; j++) X[(size_t)i * H + j] *= es;
        }
        for (int l = 0; l < cfg->num_layers && !rc; l++) {
            for (int i = 0; i < n_prompt; i++) {
                gemma3_rmsnorm_bf16(buf->x_norm, X + (size_t)i * H, w->layers[l].input_layernorm, H,
                                    cfg->rmsnorm_eps);
                matvec_bf16_dispatch(Q + (size_t)i * QS, w->layers[l].q_proj, buf->x_norm, QS, H, buf->matvec_tmp, pool);
                matvec_bf16_dispatch(K + (size_t)i * KS, w->layers[l].k_proj, buf->x_norm, KS, H, buf->matvec_tmp, pool);
                matvec_bf16_dispatch(V + (size_t)i * KS, w->layers[l].v_proj, buf->x_norm, KS, H, buf->matvec_tmp, pool);
            }
            rc = gemma3_cuda_attn_prefill(ctx, l, 0, Q, K, V, n_prompt, 0, A);
            for (int i = 0; i < n_prompt && !rc; i++)
                layer_tail(X + (size_t)i * H, A + (size_t)i * QS, w, l, buf, cfg, pool);
        }
        if (!rc) logits_of(logits, X + (size_t)(n_prompt - 1) * H, w, buf, cfg, pool);
        /* generation: one decode call per layer per token */
        int pos = n_prompt, tok = 0, seq = 0;
        for (int s = 0; s < n_steps && !rc; s++, pos++) {
            top2(logits, cfg->vocab_size, &tok, &margins_out[s]);
            tokens_out[s] = tok;
            float *x = buf->x;
            gemma3_embed_bf16(x, w->embed_tokens, tok, H);
            for (int j = 0; j < H; j++) x[j] *= es;
            for (int l = 0; l < cfg->num_layers && !rc; l++) {
                gemma3_rmsnorm_bf16(buf->x_norm, x, w->layers[l].input_layernorm, H, cfg->rmsnorm_eps);
                matvec_bf16_dispatch(buf->q, w->layers[l].q_proj, buf->x_norm, QS, H, buf->matvec_tmp, pool);
                matvec_bf16_dispatch(buf->k, w->layers[l].k_proj, buf->x_norm, KS, H, buf->matvec_tmp, pool);
                matvec_bf16_dispatch(buf->v, w->layers[l].v_proj, buf->x_norm, KS, H, buf->matvec_tmp, pool);
                rc = gemma3_cuda_attn_decode(ctx, l, 1, &seq, &pos, buf->q, buf->k, buf->v, buf->attn_out);
                if (!rc) layer_tail(x, buf->attn_out, w, l, buf, cfg, pool);
            }
            if (!rc) logits_of(logits, x, w, buf, cfg, pool);
        }
        if (rc) fprintf(stderr, "e2e: %s\n", gemma3_cuda_last_error());
        free(X); free(Q); free(K); free(V); free(A);
        gemma3_cuda_free(ctx);
    }
done:
    free(prompt);
    free(logits);
    free(rope_l);
    free(rope_g);
    free_buffers(buf);
    free_weights(w);
    gemma3_thread_pool_destroy(pool);
    return rc;
}

/*
 * gemma3_cuda.h - C-ABI of the B200 (sm_100a) attention hot path for gemma3.c.
 *
 * This is the drop-in boundary for the attention core of gemma3.c: per-head
 * QK-RMSNorm, RoPE from the host's precomputed table, KV-cache append and GQA
 * softmax(QK^T/16)V over the cache, with the 1024-row sliding window on local
 * layers and full causal attention on every 6th (global) layer.
 *
 * Shape of the API follows the reference's GPU-backend header
 * (gemma3_metal.h:20-50): an opaque context created once at model set-up,
 * a RoPE upload, per-call entry points and a cache reset.  The context owns
 * the device-resident KV cache that replaces the host cache of
 * gemma3_transformer.c:76-88 / :180-233.
 *
 * Conventions
 *  - plain C11, no CUDA or torch types in any signature;
 *  - every call returns GEMMA3_CUDA_OK (0) or a negative code whose values
 *    equal the reference's gemma3_error enum (gemma3.h:57-67); the text of the
 *    last failure on the calling thread is gemma3_cuda_last_error();
 *  - there is NO CPU fallback: if the device or the kernels are unusable the
 *    calls fail;
 *  - one host thread drives a context; all work is ordered on the context's
 *    own CUDA stream.  Host-pointer entry points synchronise that stream
 *    before returning; `_dev` entry points only enqueue.
 *
 * Layouts at the boundary are the reference's: Q [T][8*256], K/V [T][4*256]
 * fp32 (gemma3_transformer.c:614-639 Q_all/K_all/V_all), attention output
 * [T][8*256] fp32 (attn_out_all, the o_proj input), QK-norm gains BF16 [256]
 * (gemma3_transformer.c:65-66), RoPE table fp32 [max_pos][128][cos,sin]
 * (gemma3_kernels.c:455-468).
 */
#ifndef GEMMA3_CUDA_H
#define GEMMA3_CUDA_H

#include <stddef.h>
#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

/* Return codes: same values as gemma3_error (gemma3.h:57-67). */
#define GEMMA3_CUDA_OK 0
#define GEMMA3_CUDA_ERR_INVALID_ARG (-1)
#define GEMMA3_CUDA_ERR_OUT_OF_MEMORY (-4)
#define GEMMA3_CUDA_ERR_GENERATION_FAILED (-7) /* device fault, timeout, launch failure */
#define GEMMA3_CUDA_ERR_CONTEXT_OVERFLOW (-8)  /* pos >= max_context */

/* Element type of the device KV cache. */
#define GEMMA3_CUDA_KV_F32 0  /* the reference's cache dtype (bit-exact rows) */
#define GEMMA3_CUDA_KV_BF16 1 /* half the bytes; round-to-nearest-even */

/* Model dimensions + device options.  The dimension fields mirror the
 * reference's gemma3_config (gemma3.h:82-95); only Gemma-3-4B's attention
 * geometry (8 q heads, 4 kv heads, head_dim 256, window 1024) is supported
 * and anything else is rejected with GEMMA3_CUDA_ERR_INVALID_ARG. */
typedef struct {
    int num_layers;      /* 34 */
    int num_heads;       /* 8 */
    int num_kv_heads;    /* 4 */
    int head_dim;        /* 256 */
    int sliding_window;  /* 1024 */
    float rmsnorm_eps;   /* 1e-6 */
    int max_context;     /* rows of a global-layer cache per sequence */
    int max_batch;       /* number of sequence slots held in the cache */
    int kv_dtype;        /* GEMMA3_CUDA_KV_F32 or GEMMA3_CUDA_KV_BF16 */
    int device;          /* CUDA device ordinal */
    int max_prefill;     /* largest T accepted by gemma3_cuda_attn_prefill */
    /* Context-parallel split of the GLOBAL layers' KV range: this context
     * holds positions [kv_rank*S, (kv_rank+1)*S), S = ceil(max_context /
     * kv_ranks).  kv_ranks == 1 holds everything.  Local layers are never
     * split. */
    int kv_rank;
    int kv_ranks;
} gemma3_cuda_config;

typedef struct gemma3_cuda_ctx gemma3_cuda_ctx;

/* Fills *cfg with Gemma-3-4B's dimensions and single-GPU defaults
 * (max_context 8192, max_batch 1, fp32 cache, device 0, max_prefill 8192). */
void gemma3_cuda_config_default(gemma3_cuda_config *cfg);

/* Creates a context and allocates its device KV cache.  Replaces
 * gemma3_metal_init (gemma3_metal.h:26) and the cache allocation of
 * gemma3_kv_cache_alloc (gemma3_transformer.c:180-214).  NULL on failure
 * (reason in gemma3_cuda_last_error()). */
gemma3_cuda_ctx *gemma3_cuda_init(const gemma3_cuda_config *cfg);

/* Frees every device resource of the context.  Replaces gemma3_metal_free
 * (gemma3_metal.h:29) / gemma3_kv_cache_free (gemma3_transformer.c:216). */
void gemma3_cuda_free(gemma3_cuda_ctx *ctx);

/* Uploads the host RoPE tables bit-for-bit (fp32 [max_context][head_dim/2][2]
 * as built by gemma3_rope_precompute, gemma3_kernels.c:455-468).  Replaces
 * gemma3_metal_upload_rope (gemma3_metal.h:36-38). */
int gemma3_cuda_upload_rope(gemma3_cuda_ctx *ctx, const float *rope_local,
                            const float *rope_global, int max_context,
                            int head_dim);

/* Host helper that builds a RoPE table exactly as gemma3_rope_precompute
 * does (gemma3_kernels.c:455-468), for callers that have no table. */
void gemma3_cuda_rope_precompute(float *freqs, int max_pos, int head_dim,
                                 float theta);

/* Sets the QK-norm gains of one layer (BF16 [head_dim] each, the stored
 * weights w; the kernels apply 1+w as gemma3_kernels.c:301 does).  Passing
 * NULL for either disables QK-norm for that layer, as the reference's
 * `if (q_norm && k_norm)` does (gemma3_transformer.c:295). */
int gemma3_cuda_set_qk_norm(gemma3_cuda_ctx *ctx, int layer,
                            const uint16_t *q_norm, const uint16_t *k_norm);

/* Prefill attention core for T consecutive tokens of sequence slot `seq` at
 * positions start_pos..start_pos+T-1 of layer `layer`: QK-norm, RoPE,
 * cache append and causal / sliding-window GQA.  Replaces the per-token loop
 * of gemma3_transformer_prefill_batched (gemma3_transformer.c:641-692) with
 * one call per layer.  Q [T][2048], K/V [T][1024] are the raw projections,
 * out [T][2048] receives the attention output.  Host pointers. */
int gemma3_cuda_attn_prefill(gemma3_cuda_ctx *ctx, int layer, int seq,
                             const float *Q, const float *K, const float *V,
                             int T, int start_pos, float *out);
/* Same, all four arrays in device memory; enqueues only. */
int gemma3_cuda_attn_prefill_dev(gemma3_cuda_ctx *ctx, int layer, int seq,
                                 const float *Q, const float *K, const float *V,
                                 int T, int start_pos, float *out);

/* Decode attention core for B sequences, one new token each: sequence slot
 * seq_ids[b] at position pos[b].  Replaces gemma3_transformer.c:294-352 of
 * layer_attention (QK-norm, RoPE, cache_kv, seq_len/mask, gemma3_gqa) for a
 * batch.  Q [B][2048], K/V [B][1024] raw projections, out [B][2048].
 * seq_ids / pos are host arrays (B <= max_batch, distinct slots).  Host
 * pointers for Q/K/V/out. */
int gemma3_cuda_attn_decode(gemma3_cuda_ctx *ctx, int layer, int B,
                            const int *seq_ids, const int *pos, const float *Q,
                            const float *K, const float *V, float *out);
/* Same with Q/K/V/out in device memory; enqueues only. */
int gemma3_cuda_attn_decode_dev(gemma3_cuda_ctx *ctx, int layer, int B,
                                const int *seq_ids, const int *pos,
                                const float *Q, const float *K, const float *V,
                                float *out);

/* ---- Q/K/V and O projections (BF16 weights on the tensor cores) -------- */

/* Uploads one layer's projection weights, BF16 [out][in] row-major exactly
 * as the reference stores them (gemma3_layer_weights.q_proj / k_proj /
 * v_proj / o_proj, consumed by layer_attention, gemma3_transformer.c:258-356):
 * wq [2048][2560], wk and wv [1024][2560], wo [2560][2048].  Host pointers;
 * the device keeps its own copy (about 31 MB per layer). */
int gemma3_cuda_set_proj_weights(gemma3_cuda_ctx *ctx, int layer,
                                 const uint16_t *wq, const uint16_t *wk,
                                 const uint16_t *wv, const uint16_t *wo);

/* Projections of T tokens, all pointers in device memory (enqueues only).
 * qkv: x [T][2560] (the normed layer input) -> q [T][2048], k [T][1024],
 * v [T][1024]; replaces the three matvec_bf16_dispatch calls of
 * gemma3_transformer.c:290-292 (decode) and the three cblas_sgemm calls of
 * :614-639 (batched prefill).  o: attn [T][2048] -> out [T][2560]; replaces
 * gemma3_transformer.c:355 and :694-699.  The activations are rounded to
 * BF16 once, the weights are used as stored, sums accumulate in fp32.
 * T <= max(max_prefill, max_batch). */
int gemma3_cuda_project_qkv_dev(gemma3_cuda_ctx *ctx, int layer, int T,
                                const float *x, float *q, float *k, float *v);
int gemma3_cuda_project_o_dev(gemma3_cuda_ctx *ctx, int layer, int T,
                              const float *attn, float *out);

/* The whole of layer_attention (gemma3_transformer.c:258-356) for a batch of
 * B decode tokens: x [B][2560] -> QKV projections -> QK-norm, RoPE, cache
 * append, GQA -> O projection -> out [B][2560], without a host round trip
 * between the steps.  seq_ids / pos as for gemma3_cuda_attn_decode.  The
 * host-pointer form copies x in and out; _dev takes device pointers and
 * enqueues only. */
int gemma3_cuda_layer_decode(gemma3_cuda_ctx *ctx, int layer, int B,
                             const int *seq_ids, const int *pos,
                             const float *x, float *out);
int gemma3_cuda_layer_decode_dev(gemma3_cuda_ctx *ctx, int layer, int B,
                                 const int *seq_ids, const int *pos,
                                 const float *x, float *out);

/* Same for T prefill tokens of sequence slot `seq` at positions
 * start_pos.. (the attention part of one layer of
 * gemma3_transformer_prefill_batched, gemma3_transformer.c:613-699). */
int gemma3_cuda_layer_prefill(gemma3_cuda_ctx *ctx, int layer, int seq,
                              const float *x, int T, int start_pos, float *out);
int gemma3_cuda_layer_prefill_dev(gemma3_cuda_ctx *ctx, int layer, int seq,
                                  const float *x, int T, int start_pos,
                                  float *out);

/* ---- Whole transformer blocks on the device ------------------------------ */

/* One layer's weights exactly as gemma3_layer_weights holds them (BF16,
 * gemma3.h): norm gains [2560] (q_norm / k_norm [256]), projections
 * [out][in] row-major: q [2048][2560], k / v [1024][2560], o [2560][2048],
 * gate / up [10240][2560], down [2560][10240].  post_attention_layernorm,
 * pre_feedforward_layernorm and post_feedforward_layernorm may be NULL (the
 * reference then skips that norm, gemma3_transformer.c:463,473,492). */
typedef struct {
    const uint16_t *input_layernorm;
    const uint16_t *q_proj, *k_proj, *v_proj, *o_proj;
    const uint16_t *q_norm, *k_norm;
    const uint16_t *post_attention_layernorm;
    const uint16_t *gate_proj, *up_proj, *down_proj;
    const uint16_t *pre_feedforward_layernorm, *post_feedforward_layernorm;
} gemma3_cuda_layer_weights;

/* Uploads one layer's weights (about 190 MB of device memory per layer). */
int gemma3_cuda_set_layer_weights(gemma3_cuda_ctx *ctx, int layer,
                                  const gemma3_cuda_layer_weights *w);

/* All num_layers blocks of gemma3_transformer_forward (gemma3_transformer.c:
 * 427-499) for a batch of B decode tokens: x [B][2560] is the residual stream
 * (the scaled embeddings on entry, the last block's output on return: the
 * caller applies the final norm and the vocabulary projection).  seq_ids /
 * pos as for gemma3_cuda_attn_decode.  Host pointer (copied in and out) or,
 * for _dev, device pointer updated in place (enqueues only). */
int gemma3_cuda_forward(gemma3_cuda_ctx *ctx, int B, const int *seq_ids,
                        const int *pos, float *x);
int gemma3_cuda_forward_dev(gemma3_cuda_ctx *ctx, int B, const int *seq_ids,
                            const int *pos, float *x);

/* Same for T prompt tokens of sequence slot `seq` at positions
 * start_pos.. (the layer loop of gemma3_transformer_prefill_batched,
 * gemma3_transformer.c:601-740): x [T][2560] in / out. */
int gemma3_cuda_prefill_forward(gemma3_cuda_ctx *ctx, int seq, float *x, int T,
                                int start_pos);
int gemma3_cuda_prefill_forward_dev(gemma3_cuda_ctx *ctx, int seq, float *x,
                                    int T, int start_pos);

/* ---- Greedy decoding on the device ---------------------------------------- */

/* Uploads the tied embedding table (BF16 [vocab][2560], gemma3_weights_t.
 * embed_tokens) and the final norm gains (BF16 [2560], .norm).  Lookups use
 * the BF16 table exactly; the vocabulary projection uses an fp16 copy.
 * About 2.7 GB of device memory at vocab = 262208. */
int gemma3_cuda_set_embeddings(gemma3_cuda_ctx *ctx, const uint16_t *embed,
                               int vocab, const uint16_t *final_norm);

/* A prompt of T token ids (host) for sequence slot `seq` at positions
 * start_pos..: embedding lookup and scale (gemma3_transformer.c:411-418),
 * all blocks, then for the last token the final norm, the tied-embedding
 * logits (:502-509) and the greedy choice (gemma3_argmax: the first index of
 * the largest logit).  Writes the next token id and (top_logit, may be
 * NULL) its logit.  Needs gemma3_cuda_set_layer_weights for every layer. */
int gemma3_cuda_prefill_greedy(gemma3_cuda_ctx *ctx, int seq, const int *tokens,
                               int T, int start_pos, int *next_token,
                               float *top_logit);

/* One greedy decode step for B sequences: token ids (host) at positions
 * pos[b] in slots seq_ids[b] -> next token ids (host) and (top_logits, may
 * be NULL) their logits.  Only the ids cross the host boundary. */
int gemma3_cuda_greedy_step(gemma3_cuda_ctx *ctx, int B, const int *seq_ids,
                            const int *pos, const int *tokens,
                            int *next_tokens, float *top_logits);

/* ---- SafeTensors checkpoints ----------------------------------------------- */

/* Checks a checkpoint directory the way gemma3_load_weights reads it
 * (gemma3_safetensors.c:393-486, :651-713): every *.safetensors file, the
 * tensor names "language_model.model.layers.<l>.<...>.weight" (or
 * "model.layers..." for text-only checkpoints), BF16, and the Gemma 3 4B
 * shapes for num_layers layers.  Host only (no device needed); writes the
 * vocabulary size (rows of embed_tokens) to vocab_out when not NULL. */
int gemma3_cuda_safetensors_check(const char *model_dir, int num_layers,
                                  int *vocab_out);

/* Checks, then uploads every layer (gemma3_cuda_set_layer_weights) and the
 * embeddings / final norm (gemma3_cuda_set_embeddings) straight from the
 * memory-mapped files.  Nothing is uploaded if the check fails. */
int gemma3_cuda_load_safetensors(gemma3_cuda_ctx *ctx, const char *model_dir);

/* Context-parallel decode on a global layer whose KV range is split across
 * kv_ranks contexts (one per GPU).  Step 1 runs on every rank and writes this
 * rank's log-sum-exp partial for each (sequence, q head) into `partial`
 * (device, fp32 [B][8][2+256]: running max m and sum l in the log2 domain,
 * then the unnormalised output).  Step 2 merges n_parts such partials
 * ([n_parts][B][8][258], device) into out [B][2048] (device).  The exchange
 * between the steps (an all-gather over NVLink) is done by the caller, or by
 * gemma3_cuda_attn_decode_dev when a communicator is attached. */
int gemma3_cuda_attn_decode_partial_dev(gemma3_cuda_ctx *ctx, int layer, int B,
                                        const int *seq_ids, const int *pos,
                                        const float *Q, const float *K,
                                        const float *V, float *partial);
int gemma3_cuda_merge_partials_dev(gemma3_cuda_ctx *ctx, int n_parts, int B,
                                   const float *partials, float *out);

/* Context-parallel prefill of a global layer (the reference fills its global
 * caches through the same prefill loop, gemma3_transformer.c:641-692).  Each
 * rank appends the call's cache rows whose positions it holds and attends
 * every query token to its own keys only.  Step 1 writes, per token and q
 * head, that output normalised over this rank's keys into out [T][2048] and
 * its (m, l) -- reference max in the log2 domain and softmax sum -- into
 * ml [T][8][2] (queries with no key on this rank: zeros, l = 0).  Step 2
 * merges n_parts such results, outs [n_parts][T][2048] and
 * mls [n_parts][T][8][2], into out [T][2048].  Device pointers; enqueue only.
 * gemma3_cuda_attn_prefill[_dev] on such a layer does partial -> NCCL
 * all-gather -> merge itself when a communicator is attached. */
int gemma3_cuda_attn_prefill_partial_dev(gemma3_cuda_ctx *ctx, int layer, int seq,
                                         const float *Q, const float *K,
                                         const float *V, int T, int start_pos,
                                         float *out, float *ml);
int gemma3_cuda_merge_prefill_partials_dev(gemma3_cuda_ctx *ctx, int n_parts, int T,
                                           const float *outs, const float *mls,
                                           float *out);

/* NCCL communicator for the context-parallel split (optional).  Rank 0 calls
 * gemma3_cuda_comm_unique_id and ships the 128 opaque bytes to every rank
 * (any host channel); each rank then calls gemma3_cuda_comm_init with its
 * kv_rank / kv_ranks.  With a communicator attached, decode on a global layer
 * of a split context performs partial -> all-gather -> merge internally. */
int gemma3_cuda_comm_unique_id(void *id_128_bytes);
int gemma3_cuda_comm_init(gemma3_cuda_ctx *ctx, const void *id_128_bytes);

/* Exchange used by the context-parallel split on global layers.  No
 * counterpart in the reference (its attention runs on one CPU); it replaces
 * the all-gather of the (m, l, O) partials:
 *   GEMMA3_CUDA_XCHG_NCCL  ncclAllGather of the partials, then a merge kernel;
 *   GEMMA3_CUDA_XCHG_PEER  the kernel that merges this rank's splits stores
 *                          its partial directly into every rank's receive
 *                          buffer over NVLink (P2P stores to CUDA-IPC mapped
 *                          memory) and raises a per-rank flag; the final
 *                          merge waits on the flags (bounded, about 2 s, then
 *                          GEMMA3_CUDA_ERR_GENERATION_FAILED) -- no library
 *                          collective on the data path.
 * gemma3_cuda_peer_init is collective over the kv_ranks contexts (after
 * gemma3_cuda_comm_init, same node, GPUs with peer access); it maps every
 * rank's buffers and selects GEMMA3_CUDA_XCHG_PEER.  Every rank must then
 * issue the same sequence of global-layer decode calls; after a failed
 * exchange the ranks' epochs may disagree, so free and re-create the
 * contexts. */
#define GEMMA3_CUDA_XCHG_NCCL 0
#define GEMMA3_CUDA_XCHG_PEER 1
int gemma3_cuda_peer_init(gemma3_cuda_ctx *ctx);
int gemma3_cuda_set_exchange(gemma3_cuda_ctx *ctx, int mode);

/* Marks every cache empty (counters only in the reference,
 * gemma3_transformer.c:226-233; here the device cache is also zeroed, as the
 * Metal backend does at gemma3_metal.m:989-997).  On a context with the peer
 * exchange set up it also clears the exchange epoch and flags: after a failed
 * exchange, every rank of the group calls it (with no exchange in flight) to
 * bring the group back in step. */
int gemma3_cuda_reset(gemma3_cuda_ctx *ctx);

/* Debug/test: copies one sequence's cache of one layer to the host in the
 * reference layout fp32 [rows][4][256] (rows = max_context for a global
 * layer -- this rank's shard rows when split -- and 1024 for a local one). */
int gemma3_cuda_export_cache(gemma3_cuda_ctx *ctx, int layer, int seq,
                             float *k, float *v);
/* Test/bench: fills rows [0, rows) of one sequence's cache from host fp32
 * [rows][4][256] arrays (converted to the cache dtype). */
int gemma3_cuda_import_cache(gemma3_cuda_ctx *ctx, int layer, int seq,
                             const float *k, const float *v, int rows);
/* Bench: fills rows [0, rows) of one sequence's cache on the device with
 * seeded pseudo-random N(0,1) values (no host traffic). */
int gemma3_cuda_fill_cache_random(gemma3_cuda_ctx *ctx, int layer, int seq,
                                  int rows, uint64_t seed);

/* The context's CUDA stream (a cudaStream_t) for callers that time or order
 * work against it; and a blocking synchronise that reports device errors,
 * including the bounded-wait timeout flag raised by the kernels. */
void *gemma3_cuda_stream(gemma3_cuda_ctx *ctx);
int gemma3_cuda_synchronize(gemma3_cuda_ctx *ctx);

/* Number of kernels this context has launched since creation (instrumentation
 * for the bench's launch count). */
long long gemma3_cuda_launch_count(gemma3_cuda_ctx *ctx);

/* Instrumentation (no counterpart in the reference, which has no timers).
 * gemma3_cuda_profile(ctx, 1) starts recording a CUDA event pair around
 * every launch of the two dominant kernels (and clears earlier records);
 * gemma3_cuda_profile_read sums, for kernel 0 = split-KV decode,
 * 1 = tensor-core prefill or 2 = projection GEMM (with its split-K
 * reduction), the launches, their device time in ms and their algorithmic
 * work: K/V bytes read (decode) or FLOPs (prefill, projections). */
int gemma3_cuda_profile(gemma3_cuda_ctx *ctx, int enable);
int gemma3_cuda_profile_read(gemma3_cuda_ctx *ctx, int kernel, long long *launches,
                             double *ms, double *work);

/* GQA decode that allocates no memory.  No counterpart in the reference: it
 * exists for callers that cannot allocate device memory -- hosts that may not
 * stall on cudaMalloc's implicit device synchronisation inside a serving
 * loop, processes whose device memory budget is fixed up front, embedders
 * that supply every buffer themselves.  It runs the same
 * split-KV kernels as gemma3_cuda_attn_decode_dev on a cache the caller owns,
 * keeping its scratch (scaled queries and split partials) in a static device
 * array of 4.6 MB that every GPU loading this library holds until exit.
 *   q      device fp32 [B][8][256]: the query heads after their RMSNorm and
 *          rotary embedding, unscaled (the 1/16 score scale is applied here);
 *   kv     device cache, layout [B][K,V][4][rows][256] in kv_dtype, 16-byte
 *          aligned (it is streamed with bulk copies; a misaligned pointer is
 *          rejected with GEMMA3_CUDA_ERR_INVALID_ARG before anything runs);
 *   nrows  host int[B], rows 0..nrows[b]-1 of sequence b are attended
 *          (1 <= nrows[b] <= rows);
 *   out    device fp32 [B][8*256];
 *   stream cudaStream_t to enqueue on (NULL = legacy default stream).
 * Limits: 1 <= B <= 64 (larger B is rejected with GEMMA3_CUDA_ERR_INVALID_ARG).
 * The first call on a device resolves the array's address on that device
 * (the current one), so make it before any stream capture.  All calls share
 * the one array: calls that overlap on the GPU (other streams, other host
 * threads) race and must be serialised by the caller.  Enqueues only: the
 * return code covers the arguments and the launches.  A failure on the device
 * (a bounded wait in the split kernel that gave up) cannot be returned by an
 * enqueue-only call, so it fills all of out with NaN instead; check out once
 * the stream has reached it. */
int gemma3_cuda_gqa_decode_noalloc(const float *q, const void *kv, int kv_dtype,
                                   int rows, int B, const int *nrows, float *out,
                                   void *stream);

/* Test hook for failure detection (no counterpart in the reference, which
 * has no device code): runs a kernel whose bounded wait can never complete.
 * After the wait limit (about 2 s) the kernel sets the context's status word
 * and returns; this call then reports GEMMA3_CUDA_ERR_GENERATION_FAILED
 * ("bounded wait timed out"), clears the status, and the context remains
 * usable for further calls. */
int gemma3_cuda_selftest_wait_timeout(gemma3_cuda_ctx *ctx);

/* Text of the last failure on this thread ("" if none). */
const char *gemma3_cuda_last_error(void);

#ifdef __cplusplus
}
#endif

#endif /* GEMMA3_CUDA_H */

// layer_kernels.cuh - the non-attention parts of a Gemma 3 transformer block
// on the device: RMSNorm with (1 + w) BF16 gains, residual adds, and the
// GELU-tanh gated MLP activation.  The matrix products (gate / up / down)
// run on proj_gemm_sm100.
//
// Reference: gemma3_transformer_forward (gemma3_transformer.c:427-499) and
// layer_mlp (:362-398); gemma3_rmsnorm_bf16 (gemma3_kernels.c:289-304),
// gemma3_gelu_tanh_inplace (:348-358), gemma3_vec_mul / gemma3_vec_add.
// Every row of the residual stream is fp32 [2560]; the inputs of the next
// matrix product are written as fp16 (range-checked, see proj_kernels.cuh).
// Launched with programmatic dependent launch (griddepcontrol.wait first).
#pragma once
#include "proj_kernels.cuh"

namespace g3 {

constexpr int kHiddenDim = 2560;
constexpr int kNormThreads = 256;  // one CTA per row, 10 elements per thread
constexpr int kNormPer = kHiddenDim / kNormThreads;

// Sum over the CTA (256 threads = 8 warps).
__device__ __forceinline__ float block_sum(float v, float *red) {
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) v += __shfl_xor_sync(0xffffffffu, v, o);
    const int w = threadIdx.x >> 5, l = threadIdx.x & 31;
    __syncthreads();  // red is reused by consecutive calls
    if (l == 0) red[w] = v;
    __syncthreads();
    float t = l < kNormThreads / 32 ? red[l] : 0.f;
#pragma unroll
    for (int o = 4; o > 0; o >>= 1) t += __shfl_xor_sync(0xffffffffu, t, o);
    return __shfl_sync(0xffffffffu, t, 0);
}

// y = v * (1 / sqrtf(mean(v^2) + eps)) * (1 + w), as gemma3_rmsnorm_bf16.
__device__ __forceinline__ void rms_apply(float (&v)[kNormPer], const uint16_t *w, float eps, float *red) {
    float ss = 0.f;
#pragma unroll
    for (int i = 0; i < kNormPer; ++i) ss = fmaf(v[i], v[i], ss);
    ss = block_sum(ss, red);
    const float r = 1.0f / sqrtf(ss / (float)kHiddenDim + eps);
#pragma unroll
    for (int i = 0; i < kNormPer; ++i) {
        const int c = threadIdx.x + i * kNormThreads;
        v[i] = v[i] * r * (1.0f + bf16_bits_to_f(w[c]));
    }
}

__device__ __forceinline__ __half to_half_rc(float v, unsigned *err) {
    if (!(fabsf(v) <= 65504.f)) raise_status(err, kErrRange);
    return __float2half_rn(v);
}

// xn[row] = rmsnorm(x[row], w) in fp16 (the pre-attention norm of the first
// layer; later layers get theirs from residual_norm_rows).
__global__ void __launch_bounds__(kNormThreads) rms_norm_rows_f16(const float *__restrict__ x,
                                                                  const uint16_t *__restrict__ w, __half *__restrict__ xn,
                                                                  float eps, unsigned *err) {
    __shared__ float red[8];
    pdl_launch_dependents();
    pdl_wait();
    const size_t base = (size_t)blockIdx.x * kHiddenDim;
    float v[kNormPer];
#pragma unroll
    for (int i = 0; i < kNormPer; ++i) v[i] = x[base + threadIdx.x + i * kNormThreads];
    rms_apply(v, w, eps, red);
#pragma unroll
    for (int i = 0; i < kNormPer; ++i) xn[base + threadIdx.x + i * kNormThreads] = to_half_rc(v[i], err);
}

// One residual step of the block, per row:
//     delta = sum of the nparts partial sums delta + s * part_stride, in order
//             (the split-K partials of the projection before it)
//     d = w_post ? rmsnorm(delta, w_post) : delta;  x += d;
//     if (xn) xn = (w_pre ? rmsnorm(x, w_pre) : x) in fp16
// i.e. the post-attention (post-feed-forward) norm, the residual add, and the
// pre-feed-forward (next layer's pre-attention) norm of
// gemma3_transformer.c:463-468, :472-478, :491-498 and :436-437.
__global__ void __launch_bounds__(kNormThreads) residual_norm_rows(const float *__restrict__ delta, int nparts,
                                                                   size_t part_stride,
                                                                   const uint16_t *__restrict__ w_post,
                                                                   float *__restrict__ x,
                                                                   const uint16_t *__restrict__ w_pre,
                                                                   __half *__restrict__ xn, float eps, unsigned *err) {
    __shared__ float red[8];
    pdl_launch_dependents();
    pdl_wait();
    const size_t base = (size_t)blockIdx.x * kHiddenDim;
    float d[kNormPer];
#pragma unroll
    for (int i = 0; i < kNormPer; ++i) d[i] = delta[base + threadIdx.x + i * kNormThreads];
    for (int s = 1; s < nparts; ++s) {
        const float *ds = delta + (size_t)s * part_stride;
#pragma unroll
        for (int i = 0; i < kNormPer; ++i) d[i] += ds[base + threadIdx.x + i * kNormThreads];
    }
    if (w_post) rms_apply(d, w_post, eps, red);
#pragma unroll
    for (int i = 0; i < kNormPer; ++i) {
        const size_t c = base + threadIdx.x + i * kNormThreads;
        d[i] += x[c];
        x[c] = d[i];
    }
    if (!xn) return;
    if (w_pre) rms_apply(d, w_pre, eps, red);
#pragma unroll
    for (int i = 0; i < kNormPer; ++i) xn[base + threadIdx.x + i * kNormThreads] = to_half_rc(d[i], err);
}

// h = gelu_tanh(gate) * up in fp16 (layer_mlp, gemma3_transformer.c:385-386;
// gelu_tanh(x) = 0.5 x (1 + tanh(sqrt(2/pi) (x + 0.044715 x^3)))).
// gate and up are [rows][inter] each, at gu and gu + rows * inter.
__global__ void __launch_bounds__(256) gelu_mul_f16(const float *__restrict__ gate, const float *__restrict__ up,
                                                    __half *__restrict__ h, size_t n, unsigned *err) {
    pdl_launch_dependents();
    pdl_wait();
    const float k0 = 0.7978845608028654f, k1 = 0.044715f;
    for (size_t i = (size_t)blockIdx.x * blockDim.x + threadIdx.x; i < n; i += (size_t)gridDim.x * blockDim.x) {
        const float g = gate[i];
        const float inner = k0 * (g + k1 * g * g * g);
        h[i] = to_half_rc(0.5f * g * (1.0f + tanhf(inner)) * up[i], err);
    }
}

// x[row] = embed[tokens[row]] * scale in fp32 (gemma3_embed_bf16,
// gemma3_kernels.c:322-328, then the sqrt(hidden_size) scale of
// gemma3_transformer.c:411-418).  A token id outside [0, vocab) writes zeros
// and raises kErrBadIndex.
__global__ void __launch_bounds__(kNormThreads) embed_rows(const int *__restrict__ tokens,
                                                           const uint16_t *__restrict__ embed, int vocab, float scale,
                                                           float *__restrict__ x, unsigned *err) {
    pdl_launch_dependents();
    pdl_wait();
    const int tok = tokens[blockIdx.x];
    const bool ok = tok >= 0 && tok < vocab;
    if (!ok && threadIdx.x == 0) raise_status(err, kErrBadIndex);
    const uint16_t *row = embed + (size_t)(ok ? tok : 0) * kHiddenDim;
#pragma unroll
    for (int i = 0; i < kNormPer; ++i) {
        const int c = threadIdx.x + i * kNormThreads;
        x[(size_t)blockIdx.x * kHiddenDim + c] = ok ? bf16_bits_to_f(row[c]) * scale : 0.f;
    }
}

// Per row: the first index of the largest of n logits and its value, as
// gemma3_argmax (gemma3_kernels.c:799-811: strict ">" scanning from index 0,
// so the lowest index wins a tie).  A NaN ranks below every number here.
// One CTA of 1024 threads per row.
constexpr int kArgmaxThreads = 1024;
__device__ __forceinline__ bool arg_gt(float a, float b) { return a > b || (b != b && a == a); }
// candidate (va, ia) beats (vb, ib): ia < 0 marks "no candidate"
__device__ __forceinline__ bool arg_better(float va, int ia, float vb, int ib) {
    if (ib < 0) return ia >= 0;
    if (ia < 0) return false;
    return arg_gt(va, vb) || (!arg_gt(vb, va) && ia < ib);
}
__global__ void __launch_bounds__(kArgmaxThreads) argmax_rows(const float *__restrict__ logits, size_t ld, int n,
                                                               int *__restrict__ idx_out, float *__restrict__ val_out) {
    __shared__ float sv[32];
    __shared__ int si[32];
    pdl_launch_dependents();
    pdl_wait();
    const float *row = logits + (size_t)blockIdx.x * ld;
    float best = 0.f;
    int bi = -1;
    for (int i = threadIdx.x; i < n; i += kArgmaxThreads) {
        const float v = row[i];
        if (bi < 0 || arg_gt(v, best)) {
            best = v;
            bi = i;
        }
    }
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) {
        const float ov = __shfl_xor_sync(0xffffffffu, best, o);
        const int oi = __shfl_xor_sync(0xffffffffu, bi, o);
        if (arg_better(ov, oi, best, bi)) {
            best = ov;
            bi = oi;
        }
    }
    const int w = threadIdx.x >> 5, l = threadIdx.x & 31;
    if (l == 0) {
        sv[w] = best;
        si[w] = bi;
    }
    __syncthreads();
    if (w == 0) {
        best = sv[l];
        bi = si[l];
#pragma unroll
        for (int o = 16; o > 0; o >>= 1) {
            const float ov = __shfl_xor_sync(0xffffffffu, best, o);
            const int oi = __shfl_xor_sync(0xffffffffu, bi, o);
            if (arg_better(ov, oi, best, bi)) {
                best = ov;
                bi = oi;
            }
        }
        if (l == 0) {
            idx_out[blockIdx.x] = bi < 0 ? 0 : bi;
            if (val_out) val_out[blockIdx.x] = best;
        }
    }
}

}  // namespace g3

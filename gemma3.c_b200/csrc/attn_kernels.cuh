// attn_kernels.cuh - the device side of the gemma3.c attention hot path.
//
//   prologue_*        per-head QK-RMSNorm (gemma3_kernels.c:289-304), RoPE
//                     from the uploaded table (gemma3_kernels.c:470-484) and
//                     the KV-cache append (gemma3_transformer.c:236-251),
//                     fused into one pass over the token's q/k/v rows;
//   decode_splitkv    GQA decode over the cache (gemma3_kernels.c:527-597):
//                     one CTA per (sequence, kv head, key range), both query
//                     heads of the group share every K/V row, 16-byte
//                     coalesced bulk-copied rows, warp-shuffle reductions,
//                     online softmax in the log2 domain;
//   merge_partials    log-sum-exp merge of the (m, l, O) partials;
//   merge_partials_push / merge_peer_partials
//                     the same merge across the GPUs of a context-parallel
//                     split: partials stored into every rank's buffer over
//                     NVLink, flags, bounded wait, final merge;
//   prefill_fa_sm100  causal / sliding-window flash attention for prefill on
//                     the 5th-generation tensor core: persistent CTAs, TMA-
//                     staged K/V tiles, tcgen05.mma (fp16 x fp16 -> fp32)
//                     into TMEM, online softmax by eight warps with P written
//                     back to TMEM as the A operand of the PV MMA.
//
// Device KV-cache layout (per layer): [seq][K|V][kv_head][row][256] in the
// cache dtype (fp32 or bf16), rows = max_context (global layer, or this
// rank's shard of it) or 1024 (local ring).  Each (seq, K|V, head) plane is
// contiguous, so a run of rows is one linear bulk copy and one TMA box.
#pragma once
#include <cuda_bf16.h>
#include <cuda_fp16.h>
#include <cuda_runtime.h>
#include <climits>
#include <cstdint>

#include "sm100_ptx.cuh"

namespace g3 {

constexpr int kHeads = 8;
constexpr int kKvHeads = 4;
constexpr int kHeadDim = 256;
constexpr int kWindow = 1024;
constexpr int kMaxDecodeBatch = 256;
constexpr int kMaxSplitFused = 128;  // splits the in-kernel merge can hold (host caps nsplit at this)
// softmax(x/16) evaluated as 2^(x * log2(e)/16)
constexpr float kScaleLog2 = 0.0901684400555602f;

template <typename T>
struct KvType;
template <>
struct KvType<float> {
    __device__ static __forceinline__ float to_f(float x) { return x; }
    __device__ static __forceinline__ float from_f(float x) { return x; }
};
template <>
struct KvType<__nv_bfloat16> {
    __device__ static __forceinline__ float to_f(__nv_bfloat16 x) { return __bfloat162float(x); }
    __device__ static __forceinline__ __nv_bfloat16 from_f(float x) { return __float2bfloat16_rn(x); }
};

__device__ __forceinline__ float bf16_bits_to_f(uint16_t h) { return __uint_as_float((uint32_t)h << 16); }

// A head row (256 values) is handled by one warp: lane l owns dims 4l..4l+3
// and 128+4l..128+4l+3, i.e. the four rotate-half pairs (i, i+128) of its i's,
// so RoPE never leaves the lane and the RMSNorm sum is one warp reduction.
struct HeadRow {
    float a[4];  // x[4l + j]
    float b[4];  // x[128 + 4l + j]
};

__device__ __forceinline__ void load_head_row(const float *x, int lane, HeadRow &r) {
    const float4 u = *reinterpret_cast<const float4 *>(x + 4 * lane);
    const float4 v = *reinterpret_cast<const float4 *>(x + 128 + 4 * lane);
    r.a[0] = u.x; r.a[1] = u.y; r.a[2] = u.z; r.a[3] = u.w;
    r.b[0] = v.x; r.b[1] = v.y; r.b[2] = v.z; r.b[3] = v.w;
}

// RMSNorm with the (1+w) gain when w != null (gemma3_kernels.c:289-304),
// then RoPE from the table row (gemma3_kernels.c:470-484).  The gain and
// table loads are issued first, so their latency overlaps the sum of squares
// and its warp reduction.
__device__ __forceinline__ void norm_rope_row(HeadRow &r, const uint16_t *w, float eps, const float *rope_row,
                                              int lane) {
    const float4 c0 = *reinterpret_cast<const float4 *>(rope_row + 8 * lane);      // (cos,sin) of i = 4l, 4l+1
    const float4 c1 = *reinterpret_cast<const float4 *>(rope_row + 8 * lane + 4);  // i = 4l+2, 4l+3
    uint2 wa = make_uint2(0u, 0u), wb = make_uint2(0u, 0u);
    if (w) {
        wa = *reinterpret_cast<const uint2 *>(w + 4 * lane);
        wb = *reinterpret_cast<const uint2 *>(w + 128 + 4 * lane);
    }
    if (w) {
        float ss = 0.f;
#pragma unroll
        for (int j = 0; j < 4; ++j) ss += r.a[j] * r.a[j] + r.b[j] * r.b[j];
#pragma unroll
        for (int o = 16; o > 0; o >>= 1) ss += __shfl_xor_sync(0xffffffffu, ss, o);
        const float rr = 1.0f / sqrtf(ss / (float)kHeadDim + eps);
        const uint16_t ga[4] = {(uint16_t)(wa.x & 0xffff), (uint16_t)(wa.x >> 16), (uint16_t)(wa.y & 0xffff),
                                (uint16_t)(wa.y >> 16)};
        const uint16_t gb[4] = {(uint16_t)(wb.x & 0xffff), (uint16_t)(wb.x >> 16), (uint16_t)(wb.y & 0xffff),
                                (uint16_t)(wb.y >> 16)};
#pragma unroll
        for (int j = 0; j < 4; ++j) {
            r.a[j] = r.a[j] * rr * (1.0f + bf16_bits_to_f(ga[j]));
            r.b[j] = r.b[j] * rr * (1.0f + bf16_bits_to_f(gb[j]));
        }
    }
    const float cs[4] = {c0.x, c0.z, c1.x, c1.z}, sn[4] = {c0.y, c0.w, c1.y, c1.w};
#pragma unroll
    for (int j = 0; j < 4; ++j) {
        const float x0 = r.a[j], x1 = r.b[j];
        r.a[j] = x0 * cs[j] - x1 * sn[j];
        r.b[j] = x0 * sn[j] + x1 * cs[j];
    }
}

template <typename KVT>
__device__ __forceinline__ void store4(KVT *dst, const float (&v)[4]);
template <>
__device__ __forceinline__ void store4<float>(float *dst, const float (&v)[4]) {
    *reinterpret_cast<float4 *>(dst) = make_float4(v[0], v[1], v[2], v[3]);
}
template <>
__device__ __forceinline__ void store4<__nv_bfloat16>(__nv_bfloat16 *dst, const float (&v)[4]) {
    *reinterpret_cast<uint2 *>(dst) = make_uint2(pack_bf16x2(v[0], v[1]), pack_bf16x2(v[2], v[3]));
}
__device__ __forceinline__ void store4_half(__half *dst, const float (&v)[4]) {
    *reinterpret_cast<uint2 *>(dst) = make_uint2(pack_f16x2(v[0], v[1]), pack_f16x2(v[2], v[3]));
}
// Rounds 4 values to the cache dtype and back (what the cache will hold).
template <typename KVT>
__device__ __forceinline__ void through_dtype(float (&v)[4]) {
#pragma unroll
    for (int j = 0; j < 4; ++j) v[j] = KvType<KVT>::to_f(KvType<KVT>::from_f(v[j]));
}

struct LayerDev {
    void *kv;          // cache base of the layer
    int rows;          // rows per (seq, head) plane
    int is_global;
    int shard_lo;      // first position held (global layers; 0 otherwise)
    int shard_hi;      // one past the last position held
    const uint16_t *qn;  // QK-norm gains or null
    const uint16_t *kn;
    const float *rope;   // [max_pos][128][2]
};

template <typename KVT>
__device__ __forceinline__ KVT *plane(const LayerDev &L, int seq, int kv_sel, int head) {
    return reinterpret_cast<KVT *>(L.kv) + (((size_t)seq * 2 + kv_sel) * kKvHeads + head) * (size_t)L.rows * kHeadDim;
}

// Cache row of position pos, or -1 if this context does not hold it
// (gemma3_transformer.c:240-248: global append at pos, local ring pos%1024).
__device__ __forceinline__ int cache_row(const LayerDev &L, int pos) {
    if (!L.is_global) return pos % kWindow;
    if (pos < L.shard_lo || pos >= L.shard_hi) return -1;
    return pos - L.shard_lo;
}

// ------------------------------------------------------------------------
// Prefill prologue: grid (T, 16).  q -> qst fp16 [8][T][256]; k, v ->
// cache (cache dtype) and the fp16 linear staging [4][st_rows][256] at row
// pos - kv_pos0.  The staged k/v value is the cached value (rounded to the
// cache dtype first), so the tensor-core prefill sees exactly what a later
// decode reads.  On a local layer only the last 1024 tokens are written into
// the ring (earlier ones would be overwritten by later tokens of the same
// call anyway).  A value outside the fp16 range raises kErrRange.
//
// The prefill MMAs run in fp16 rather than bf16: both have the same
// tensor-core rate, but bf16's 8-bit significand alone puts ~2% (max|err| /
// RMS per head) between bf16-operand attention and the fp32 reference on
// N(0,1) data, above the 1e-2 parity bar; fp16's 11-bit significand is ~8x
// tighter.
// ------------------------------------------------------------------------
__device__ __forceinline__ void check_half_range(const HeadRow &r, unsigned *err) {
    bool bad = false;
#pragma unroll
    for (int j = 0; j < 4; ++j) bad |= !(fabsf(r.a[j]) <= 65504.f) || !(fabsf(r.b[j]) <= 65504.f);
    if (bad) raise_status(err, kErrRange);
}

__device__ __forceinline__ __half to_half_checked(float x, unsigned *err) {
    if (!(fabsf(x) <= 65504.f)) raise_status(err, kErrRange);
    return __float2half_rn(x);
}

template <typename KVT>
__global__ void __launch_bounds__(512) prologue_prefill(const float *__restrict__ Q, const float *__restrict__ K,
                                                        const float *__restrict__ V, LayerDev L, float eps, int seq,
                                                        int T, int start_pos, int kv_pos0, int kv_end,
                                                        __half *__restrict__ qst, __half *__restrict__ kst,
                                                        __half *__restrict__ vst, int st_rows, unsigned *err) {
    // dependent launch: reads inputs and writes the staging only after the
    // previous kernel of the stream (the last layer's attention, which reads
    // the same staging) has completed
    pdl_launch_dependents();
    pdl_wait();
    const int t = blockIdx.x, y = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const int pos = start_pos + t;
    const float *rope_row = L.rope + (size_t)pos * kHeadDim;
    HeadRow r;
    if (y < kHeads) {
        load_head_row(Q + ((size_t)t * kHeads + y) * kHeadDim, lane, r);
        norm_rope_row(r, L.qn && L.kn ? L.qn : nullptr, eps, rope_row, lane);
        __half *o = qst + ((size_t)y * T + t) * kHeadDim;
        check_half_range(r, err);
        store4_half(o + 4 * lane, r.a);
        store4_half(o + 128 + 4 * lane, r.b);
        return;
    }
    const bool ring_ok = L.is_global || (pos >= start_pos + T - kWindow);
    const int row = ring_ok ? cache_row(L, pos) : -1;
    const int sel = y < kHeads + kKvHeads ? 0 : 1;
    const int h = y - kHeads - sel * kKvHeads;
    load_head_row((sel ? V : K) + ((size_t)t * kKvHeads + h) * kHeadDim, lane, r);
    if (!sel) norm_rope_row(r, L.qn && L.kn ? L.kn : nullptr, eps, rope_row, lane);
    if (row >= 0) {
        KVT *dst = plane<KVT>(L, seq, sel, h) + (size_t)row * kHeadDim;
        store4<KVT>(dst + 4 * lane, r.a);
        store4<KVT>(dst + 128 + 4 * lane, r.b);
    }
    if (pos < kv_pos0 || pos >= kv_end) return;  // a key the attention does not see here
    through_dtype<KVT>(r.a);
    through_dtype<KVT>(r.b);
    check_half_range(r, err);
    __half *sdst = (sel ? vst : kst) + ((size_t)h * st_rows + (pos - kv_pos0)) * kHeadDim;
    store4_half(sdst + 4 * lane, r.a);
    store4_half(sdst + 128 + 4 * lane, r.b);
}

// Copies the cached rows of positions [kv_pos0, start_pos) into the fp16
// staging buffer (rows 0..).  grid (n_rows, 2*4), block 32: each thread moves
// 8 elements.
template <typename KVT>
__global__ void __launch_bounds__(32) stage_prefix(LayerDev L, int seq, int kv_pos0, __half *__restrict__ kst,
                                                   __half *__restrict__ vst, int st_rows, unsigned *err) {
    const int r = blockIdx.x, sel = blockIdx.y >> 2, h = blockIdx.y & 3;
    const int pos = kv_pos0 + r;
    const int row = cache_row(L, pos);
    const KVT *src = plane<KVT>(L, seq, sel, h) + (size_t)row * kHeadDim;
    __half *dst = (sel ? vst : kst) + ((size_t)h * st_rows + r) * kHeadDim;
    const int d = threadIdx.x * 8;
    __align__(16) __half w[8];
#pragma unroll
    for (int j = 0; j < 8; ++j) w[j] = to_half_checked(KvType<KVT>::to_f(src[d + j]), err);
    *reinterpret_cast<uint4 *>(dst + d) = *reinterpret_cast<const uint4 *>(w);
}

// ------------------------------------------------------------------------
// Split-KV decode.
// grid (nsplit, 4 kv heads, B), block 256 (8 warps).  The CTA streams rows
// [split*chunk, min(nrows, (split+1)*chunk)) of its (seq, kv head) K and V
// planes through an NS-stage shared-memory ring filled by 1-D bulk copies
// (one per plane per tile: the rows are contiguous).  Warp w takes rows
// w, w+8, ... of each tile; each lane owns 8 of the 256 dims (16 bytes of a
// bf16 row: fully coalesced, conflict-free shared loads).  Both query heads
// of the GQA group are scored against every row.
// ------------------------------------------------------------------------
struct DecodeParams {
    const float *q;        // [B][8][256], pre-scaled by log2(e)/16 (used when qraw is null)
    const float *qraw;     // raw projections [B][2048] / [B][1024]: when set, the kernel
    const float *kraw;     //   normalises + rotates its own two q heads and the CTA holding
    const float *vraw;     //   the new token's cache row appends k/v (fused prologue)
    float eps;
    unsigned *tickets;     // [B][4] arrival counters, all zero between calls: when set,
                           //   the last split of each (seq, kv head) merges the partials
    LayerDev L;
    int chunk;             // rows per split (multiple of the tile)
    int nsplit;
    float *partial;        // [B][8][nsplit][258] when write_partial
    float *out;            // [B][2048] when !write_partial
    int write_partial;
    unsigned *err;
};
template <int kRows>
struct DecodeRowsT {
    int B;
    int seq[kRows];
    int nrows[kRows];  // rows attended in this context's planes
    int pos[kRows];    // position of the new token
};
using DecodeRows = DecodeRowsT<kMaxDecodeBatch>;
// Small batches: ~100 bytes of kernel parameters instead of ~3 KB.  Measured
// on B200 (standalone probe): a dependent kernel with a 3 KB parameter block
// is launched ~10 us into the kernel before it, with small parameters ~5 us,
// which matters for calls of ~12 us (B = 1..8 decode).
constexpr int kSmallDecodeBatch = 8;
using DecodeRowsSmall = DecodeRowsT<kSmallDecodeBatch>;

// Decode prologue as its own kernel, for calls whose CTAs stream long key
// ranges: grid (B), block 512 = 16 warps, warp y < 8 query head y, 8..11 key
// head, 12..15 value head.  q goes to qout [B][8][256] fp32 (scaled by
// log2(e)/16); k and v are appended to the cache.  Short-range calls fold
// this work into decode_splitkv instead (see DecodeParams::qraw).
template <typename KVT>
__global__ void __launch_bounds__(512) prologue_decode(const float *__restrict__ Q, const float *__restrict__ K,
                                                       const float *__restrict__ V, LayerDev L, float eps,
                                                       const __grid_constant__ DecodeRows rows,
                                                       float *__restrict__ qout) {
    pdl_launch_dependents();
    pdl_wait();
    const int b = blockIdx.x, y = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const int pos = rows.pos[b], seq = rows.seq[b];
    const float *rope_row = L.rope + (size_t)pos * kHeadDim;
    HeadRow r;
    if (y < kHeads) {
        load_head_row(Q + ((size_t)b * kHeads + y) * kHeadDim, lane, r);
        norm_rope_row(r, L.qn && L.kn ? L.qn : nullptr, eps, rope_row, lane);
        float *o = qout + ((size_t)b * kHeads + y) * kHeadDim;
#pragma unroll
        for (int j = 0; j < 4; ++j) {
            r.a[j] *= kScaleLog2;
            r.b[j] *= kScaleLog2;
        }
        store4<float>(o + 4 * lane, r.a);
        store4<float>(o + 128 + 4 * lane, r.b);
        return;
    }
    const int row = cache_row(L, pos);
    const int sel = y < kHeads + kKvHeads ? 0 : 1;
    const int h = y - kHeads - sel * kKvHeads;
    load_head_row((sel ? V : K) + ((size_t)b * kKvHeads + h) * kHeadDim, lane, r);
    if (!sel) norm_rope_row(r, L.qn && L.kn ? L.kn : nullptr, eps, rope_row, lane);
    if (row >= 0) {
        KVT *dst = plane<KVT>(L, seq, sel, h) + (size_t)row * kHeadDim;
        store4<KVT>(dst + 4 * lane, r.a);
        store4<KVT>(dst + 128 + 4 * lane, r.b);
    }
}


template <typename KVT>
struct DecodeCfg;
// extra dynamic shared memory of a fused-prologue launch: q (2 heads, fp32)
// + the new token's k and v rows (cache dtype)
template <typename KVT>
constexpr int kFusedExtra = 2 * kHeadDim * sizeof(float) + 2 * kHeadDim * sizeof(KVT);
template <>
struct DecodeCfg<__nv_bfloat16> {
    static constexpr int TK = 32;  // rows per tile (16 KB per plane)
    static constexpr int NS = 3;
};
template <>
struct DecodeCfg<float> {
    static constexpr int TK = 16;  // rows per tile (16 KB per plane)
    static constexpr int NS = 3;
};

// Lane `lane` owns 8 dims of a row.  bf16: dims 8*lane..8*lane+7 (one 16-B
// chunk).  fp32: dims 4*lane..+3 and 128+4*lane..+3 (two 16-B chunks, each
// warp-contiguous).
template <typename KVT>
__device__ __forceinline__ int lane_dim(int lane, int j);
template <>
__device__ __forceinline__ int lane_dim<__nv_bfloat16>(int lane, int j) { return 8 * lane + j; }
template <>
__device__ __forceinline__ int lane_dim<float>(int lane, int j) { return (j < 4 ? 4 * lane + j : 128 + 4 * lane + j - 4); }

template <typename KVT>
__device__ __forceinline__ void load_row8(const KVT *row, int lane, float (&x)[8]);
template <>
__device__ __forceinline__ void load_row8<__nv_bfloat16>(const __nv_bfloat16 *row, int lane, float (&x)[8]) {
    uint4 u = *reinterpret_cast<const uint4 *>(row + 8 * lane);
    const uint32_t w[4] = {u.x, u.y, u.z, u.w};
#pragma unroll
    for (int j = 0; j < 4; ++j) {
        x[2 * j] = __uint_as_float(w[j] << 16);
        x[2 * j + 1] = __uint_as_float(w[j] & 0xffff0000u);
    }
}
template <>
__device__ __forceinline__ void load_row8<float>(const float *row, int lane, float (&x)[8]) {
    float4 a = *reinterpret_cast<const float4 *>(row + 4 * lane);
    float4 b = *reinterpret_cast<const float4 *>(row + 128 + 4 * lane);
    x[0] = a.x; x[1] = a.y; x[2] = a.z; x[3] = a.w;
    x[4] = b.x; x[5] = b.y; x[6] = b.z; x[7] = b.w;
}

// kFused: the form for short key ranges, with the q/k/v prologue folded in
// (DecodeParams::qraw) and the in-kernel merge (DecodeParams::tickets); the
// plain form is compiled without that code, which measurably slows the long
// streaming loop even when it is not executed.


// Running online-softmax state of one warp for the two query heads of a GQA
// group: max m and sum l (log2 domain) and the lane's 8 dims of O.
struct DecAcc {
    float m0, m1, l0, l1;
    float o0[8], o1[8];
    __device__ __forceinline__ void reset() {
        m0 = m1 = -INFINITY;
        l0 = l1 = 0.f;
#pragma unroll
        for (int j = 0; j < 8; ++j) o0[j] = o1[j] = 0.f;
    }
};

// One tile of rows [0, nr) of K (kt) and V (vt) in shared memory: warp w
// scores rows w, w+8, ... against both query heads, rescales its state to
// the new running max and accumulates P.V.
template <typename KVT>
__device__ __forceinline__ void decode_tile(const KVT *kt, const KVT *vt, int nr, int warp, int lane,
                                            const float (&q0)[8], const float (&q1)[8], DecAcc &a) {
    constexpr int RW = DecodeCfg<KVT>::TK / 8;  // rows per warp per tile
    float sc0[RW], sc1[RW];
#pragma unroll
    for (int r = 0; r < RW; ++r) {
        const int row = warp + 8 * r;
        float k[8];
        if (row < nr) {
            load_row8<KVT>(kt + (size_t)row * kHeadDim, lane, k);
        } else {
#pragma unroll
            for (int j = 0; j < 8; ++j) k[j] = 0.f;
        }
        float x = 0.f, c = 0.f;
#pragma unroll
        for (int j = 0; j < 8; ++j) {
            x = fmaf(q0[j], k[j], x);
            c = fmaf(q1[j], k[j], c);
        }
        sc0[r] = x;
        sc1[r] = c;
    }
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) {
#pragma unroll
        for (int r = 0; r < RW; ++r) {
            sc0[r] += __shfl_xor_sync(0xffffffffu, sc0[r], o);
            sc1[r] += __shfl_xor_sync(0xffffffffu, sc1[r], o);
        }
    }
    float mx0 = a.m0, mx1 = a.m1;
#pragma unroll
    for (int r = 0; r < RW; ++r) {
        if (warp + 8 * r < nr) {
            mx0 = fmaxf(mx0, sc0[r]);
            mx1 = fmaxf(mx1, sc1[r]);
        }
    }
    // A warp with no valid row in this tile keeps mx == m == -inf; its
    // rescale factor must then be 1, not 2^(-inf - -inf) = NaN.
    const float al0 = mx0 == -INFINITY ? 1.f : ex2_approx(a.m0 - mx0);
    const float al1 = mx1 == -INFINITY ? 1.f : ex2_approx(a.m1 - mx1);
    a.m0 = mx0;
    a.m1 = mx1;
    a.l0 *= al0;
    a.l1 *= al1;
#pragma unroll
    for (int j = 0; j < 8; ++j) {
        a.o0[j] *= al0;
        a.o1[j] *= al1;
    }
#pragma unroll
    for (int r = 0; r < RW; ++r) {
        const int row = warp + 8 * r;
        if (row < nr) {
            const float p0 = ex2_approx(sc0[r] - a.m0), p1 = ex2_approx(sc1[r] - a.m1);
            a.l0 += p0;
            a.l1 += p1;
            float v[8];
            load_row8<KVT>(vt + (size_t)row * kHeadDim, lane, v);
#pragma unroll
            for (int j = 0; j < 8; ++j) {
                a.o0[j] = fmaf(p0, v[j], a.o0[j]);
                a.o1[j] = fmaf(p1, v[j], a.o1[j]);
            }
        }
    }
}

// Combines the 8 warps' states through shared memory: acc (16 KB,
// [warp][head][256]) and wm / wl.  Thread t gets, for head hh = t / 128 of
// the group and dims d, d + 1 (d = 2 (t % 128)), the CTA's max M, sum Ls and
// unnormalised O (A, Bv).  The caller synchronises before reusing acc.
template <typename KVT>
__device__ __forceinline__ void combine_warps(const DecAcc &a, float *acc, float (*wm)[2], float (*wl)[2], int warp,
                                              int lane, float &M, float &Ls, float &A, float &Bv) {
#pragma unroll
    for (int j = 0; j < 8; ++j) {
        acc[(warp * 2 + 0) * kHeadDim + lane_dim<KVT>(lane, j)] = a.o0[j];
        acc[(warp * 2 + 1) * kHeadDim + lane_dim<KVT>(lane, j)] = a.o1[j];
    }
    if (lane == 0) {
        wm[warp][0] = a.m0;
        wm[warp][1] = a.m1;
        wl[warp][0] = a.l0;
        wl[warp][1] = a.l1;
    }
    __syncthreads();
    const int hh = threadIdx.x >> 7;
    const int d = (threadIdx.x & 127) * 2;
    M = -INFINITY;
#pragma unroll
    for (int w = 0; w < 8; ++w) M = fmaxf(M, wm[w][hh]);
    Ls = 0.f;
    A = 0.f;
    Bv = 0.f;
    if (M != -INFINITY) {
#pragma unroll
        for (int w = 0; w < 8; ++w) {
            if (wm[w][hh] == -INFINITY) continue;  // warp saw no row
            const float f = ex2_approx(wm[w][hh] - M);
            Ls += wl[w][hh] * f;
            A += acc[(w * 2 + hh) * kHeadDim + d] * f;
            Bv += acc[(w * 2 + hh) * kHeadDim + d + 1] * f;
        }
    }
}

// Log-sum-exp merge of n partials [m, l, O[256]] of the two heads of a group
// (partial i of head 2g + th at base + th * hstride + i * 258, read through
// L2: other CTAs wrote them).  Thread t writes the normalised O of head
// hh = t / 128, dims d, d + 1 into out_g (the group's 512 outputs).  One
// online pass, 16 partials (32 loads) in flight per thread.
__device__ __forceinline__ void merge_group(const float *base, size_t hstride, int n, float *out_g) {
    constexpr int C = 16;
    const int hh = threadIdx.x >> 7, d = (threadIdx.x & 127) * 2;
    const float *bh = base + hh * hstride;
    float Mx = -INFINITY, Lt = 0.f, At = 0.f, Bt = 0.f;
    for (int i0 = 0; i0 < n; i0 += C) {
        float2 ml[C], o[C];
#pragma unroll
        for (int j = 0; j < C; ++j) {
            if (i0 + j < n) {
                const float *pp = bh + (size_t)(i0 + j) * (kHeadDim + 2);
                ml[j] = __ldcg(reinterpret_cast<const float2 *>(pp));
                o[j] = __ldcg(reinterpret_cast<const float2 *>(pp + 2 + d));
            } else {
                ml[j] = make_float2(-INFINITY, 0.f);
                o[j] = make_float2(0.f, 0.f);
            }
        }
        float cm = Mx;
#pragma unroll
        for (int j = 0; j < C; ++j) cm = fmaxf(cm, ml[j].x);
        if (cm == -INFINITY) continue;  // no rows so far
        const float sc = Mx == -INFINITY ? 0.f : ex2_approx(Mx - cm);
        Lt *= sc;
        At *= sc;
        Bt *= sc;
#pragma unroll
        for (int j = 0; j < C; ++j) {
            const float f = ml[j].x == -INFINITY ? 0.f : ex2_approx(ml[j].x - cm);
            Lt += ml[j].y * f;
            At += o[j].x * f;
            Bt += o[j].y * f;
        }
        Mx = cm;
    }
    const float inv = Lt > 0.f ? 1.0f / Lt : 0.f;
    *reinterpret_cast<float2 *>(out_g + hh * kHeadDim + d) = make_float2(At * inv, Bt * inv);
}

template <typename KVT, bool kFused>
__global__ void __launch_bounds__(256, 2) decode_splitkv(const DecodeParams p, const __grid_constant__ DecodeRows rows) {
    constexpr int TK = DecodeCfg<KVT>::TK;
    constexpr int NS = DecodeCfg<KVT>::NS;
    constexpr uint32_t kPlaneTile = TK * kHeadDim * sizeof(KVT);
    extern __shared__ __align__(128) unsigned char smem[];
    KVT *kbuf = reinterpret_cast<KVT *>(smem);
    KVT *vbuf = reinterpret_cast<KVT *>(smem + NS * kPlaneTile);
    __shared__ uint64_t full[NS], empty[NS];
    __shared__ float wm[8][2], wl[8][2];
    __shared__ int s_abort, s_last;

    const int split = blockIdx.x, g = blockIdx.y, b = blockIdx.z;
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const int seq = rows.seq[b];
    const int n = rows.nrows[b];
    const int r0 = split * p.chunk;
    const int r1 = min(n, r0 + p.chunk);
    const int ntiles = r1 > r0 ? (r1 - r0 + TK - 1) / TK : 0;

    const KVT *Kp = plane<KVT>(p.L, seq, 0, g) + (size_t)r0 * kHeadDim;
    const KVT *Vp = plane<KVT>(p.L, seq, 1, g) + (size_t)r0 * kHeadDim;

    // Dependent launch: the next kernel may start its set-up now; this one
    // touches global memory only after the previous kernel has completed.
    pdl_launch_dependents();
    if (threadIdx.x == 0) {
        s_abort = 0;
        for (int s = 0; s < NS; ++s) {
            mbar_init(&full[s], 1);
            mbar_init(&empty[s], 8);
        }
        fence_mbar_init();
    }
    __syncthreads();
    pdl_wait();

    // q and fresh-row buffers of the fused prologue live after the ring.
    float(*qsm)[kHeadDim] = reinterpret_cast<float(*)[kHeadDim]>(smem + 2 * NS * kPlaneTile);
    KVT(*newkv)[kHeadDim] = reinterpret_cast<KVT(*)[kHeadDim]>(smem + 2 * NS * kPlaneTile + 2 * kHeadDim * sizeof(float));
    const int slot = kFused ? cache_row(p.L, rows.pos[b]) : -1;  // cache row of the new token
    const bool owner = slot >= r0 && slot < r1;

    // Thread 0 fills the ring.  In the fused form the new token's row may
    // not be in global memory yet when its tile is copied, so that tile is
    // copied around the row and thread 0 writes the fresh row (built by the
    // prologue below) into shared memory itself before arming the barrier.
    auto issue = [&](int i) {
        const int s = i % NS;
        const int base = r0 + i * TK;
        const int nr = min(TK, r1 - base);
        const uint32_t row_b = kHeadDim * sizeof(KVT);
        KVT *ks = kbuf + (size_t)s * TK * kHeadDim, *vs = vbuf + (size_t)s * TK * kHeadDim;
        const KVT *kg = Kp + (size_t)i * TK * kHeadDim, *vg = Vp + (size_t)i * TK * kHeadDim;
        if (kFused && owner && slot >= base && slot < base + nr) {
            const int rr = slot - base, after = nr - rr - 1;
            constexpr int kVec = kHeadDim * sizeof(KVT) / 16;
            for (int c = 0; c < kVec; ++c) {
                reinterpret_cast<uint4 *>(ks + (size_t)rr * kHeadDim)[c] = reinterpret_cast<const uint4 *>(newkv[0])[c];
                reinterpret_cast<uint4 *>(vs + (size_t)rr * kHeadDim)[c] = reinterpret_cast<const uint4 *>(newkv[1])[c];
            }
            // order these generic writes before later bulk copies into the same slot
            fence_proxy_async_smem();
            mbar_expect_tx(&full[s], 2 * (uint32_t)(nr - 1) * row_b);
            if (rr > 0) {
                bulk_g2s(ks, kg, rr * row_b, &full[s]);
                bulk_g2s(vs, vg, rr * row_b, &full[s]);
            }
            if (after > 0) {
                bulk_g2s(ks + (size_t)(rr + 1) * kHeadDim, kg + (size_t)(rr + 1) * kHeadDim, after * row_b, &full[s]);
                bulk_g2s(vs + (size_t)(rr + 1) * kHeadDim, vg + (size_t)(rr + 1) * kHeadDim, after * row_b, &full[s]);
            }
            return;
        }
        mbar_expect_tx(&full[s], 2 * (uint32_t)nr * row_b);
        bulk_g2s(ks, kg, nr * row_b, &full[s]);
        bulk_g2s(vs, vg, nr * row_b, &full[s]);
    };
    // Tiles ahead of the one holding the new token's row (owner CTA only)
    // go out right away; that tile and the rest of the first fill after the
    // prologue has built the row.
    int early = 0;
    if (threadIdx.x == 0) {
        while (early < NS && early < ntiles &&
               !(kFused && owner && slot >= r0 + early * TK && slot < r0 + (early + 1) * TK))
            issue(early++);
    }

    // Fused prologue (gemma3_transformer.c:294-316): while the first tiles
    // are in flight, warps 0-1 normalise + rotate the two query heads of the
    // group, and in the CTA whose key range holds the new token's cache row,
    // warps 2-3 build that k/v row, append it to the cache and keep it in
    // shared memory: the bulk-copied copy of that row may be stale.
    if constexpr (kFused) {
        const float *rope_row = p.L.rope + (size_t)rows.pos[b] * kHeadDim;
        const uint16_t *qn = p.L.qn && p.L.kn ? p.L.qn : nullptr;
        const uint16_t *kn = p.L.qn && p.L.kn ? p.L.kn : nullptr;
        HeadRow r;
        if (warp < 2) {
            load_head_row(p.qraw + ((size_t)b * kHeads + 2 * g + warp) * kHeadDim, lane, r);
            norm_rope_row(r, qn, p.eps, rope_row, lane);
#pragma unroll
            for (int j = 0; j < 4; ++j) {
                r.a[j] *= kScaleLog2;
                r.b[j] *= kScaleLog2;
            }
            store4<float>(&qsm[warp][4 * lane], r.a);
            store4<float>(&qsm[warp][128 + 4 * lane], r.b);
        } else if (warp < 4 && owner) {
            const int sel = warp - 2;
            load_head_row((sel ? p.vraw : p.kraw) + ((size_t)b * kKvHeads + g) * kHeadDim, lane, r);
            if (!sel) norm_rope_row(r, kn, p.eps, rope_row, lane);
            KVT *dst = plane<KVT>(p.L, seq, sel, g) + (size_t)slot * kHeadDim;
            store4<KVT>(dst + 4 * lane, r.a);
            store4<KVT>(dst + 128 + 4 * lane, r.b);
            store4<KVT>(&newkv[sel][4 * lane], r.a);
            store4<KVT>(&newkv[sel][128 + 4 * lane], r.b);
        }
        __syncthreads();
        if (threadIdx.x == 0)
            for (int i = early; i < NS && i < ntiles; ++i) issue(i);
    }

    // Query rows of the two heads sharing kv head g, the lane's 8 dims.
    float q0[8], q1[8];
    {
        const float *qa = kFused ? &qsm[0][0] : p.q + ((size_t)b * kHeads + 2 * g) * kHeadDim;
        const float *qb = qa + kHeadDim;
#pragma unroll
        for (int j = 0; j < 8; ++j) {
            q0[j] = qa[lane_dim<KVT>(lane, j)];
            q1[j] = qb[lane_dim<KVT>(lane, j)];
        }
    }
    DecAcc acc_st;
    acc_st.reset();

    for (int i = 0; i < ntiles; ++i) {
        const int s = i % NS;
        if (!mbar_wait(&full[s], (i / NS) & 1, p.err)) {
            s_abort = 1;
            break;
        }
        if (s_abort) break;
        const int nr = min(TK, r1 - (r0 + i * TK));
        decode_tile<KVT>(kbuf + (size_t)s * TK * kHeadDim, vbuf + (size_t)s * TK * kHeadDim, nr, warp, lane, q0, q1,
                         acc_st);
        __syncwarp();
        if (lane == 0) mbar_arrive(&empty[s]);
        if (threadIdx.x == 0 && i + NS < ntiles) {
            if (!mbar_wait(&empty[s], (i / NS) & 1, p.err)) {
                s_abort = 1;
                break;
            }
            issue(i + NS);
        }
    }
    // Wait out any copies still in flight before the ring is reused
    // (only reachable after an aborted wait).
    if (threadIdx.x == 0 && s_abort) {
        for (int i = 0; i < ntiles && i < NS; ++i) mbar_wait(&full[i % NS], 0, nullptr);
    }
    __syncthreads();

    // Combine the 8 warps' (m, l, o) through shared memory (the K ring is
    // free now).
    float *acc = reinterpret_cast<float *>(smem);
    float M, Ls, A, Bv;
    combine_warps<KVT>(acc_st, acc, wm, wl, warp, lane, M, Ls, A, Bv);
    const int hh = threadIdx.x >> 7;
    const int d = (threadIdx.x & 127) * 2;
    const int h = 2 * g + hh;
    if (p.write_partial) {
        float *dst = p.partial + (((size_t)b * kHeads + h) * p.nsplit + split) * (kHeadDim + 2);
        if (threadIdx.x == 0 || threadIdx.x == 128) {
            dst[0] = M;
            dst[1] = Ls;
        }
        dst[2 + d] = A;
        dst[3 + d] = Bv;
        if (kFused && p.tickets) {
            // Split-K style completion: the last split of this (seq, kv head)
            // to finish merges all partials; no CTA ever waits for another.
            __syncthreads();
            if (threadIdx.x == 0)
                s_last = atom_add_acqrel_gpu(&p.tickets[b * kKvHeads + g], 1u) == (unsigned)(p.nsplit - 1);
            __syncthreads();
            if (!s_last) return;
            merge_group(p.partial + ((size_t)b * kHeads + 2 * g) * p.nsplit * (kHeadDim + 2),
                        (size_t)p.nsplit * (kHeadDim + 2), p.nsplit, p.out + (size_t)b * kHeads * kHeadDim + 2 * g * kHeadDim);
            if (threadIdx.x == 0) p.tickets[b * kKvHeads + g] = 0u;
        }
    } else {
        const float inv = Ls > 0.f ? 1.0f / Ls : 0.f;
        float2 *dst = reinterpret_cast<float2 *>(p.out + (size_t)b * kHeads * kHeadDim + h * kHeadDim + d);
        *dst = make_float2(A * inv, Bv * inv);
    }
}

// ------------------------------------------------------------------------
// Log-sum-exp merge of n partials per (seq, head).  grid (B*8), block 256
// (one thread per dim).  Partial (b, h, part) lives at
// partials + b*bstride + h*hstride + part*pstride: [m, l, O[256]].
// Writes out [B][2048] (normalised) or, with emit_partial, one merged
// partial per (b, h) at emit [B][8][258].
// ------------------------------------------------------------------------
__global__ void __launch_bounds__(256) merge_partials(const float *__restrict__ partials, int nparts, size_t bstride,
                                                      size_t hstride, size_t pstride, float *__restrict__ out,
                                                      float *__restrict__ emit) {
    pdl_launch_dependents();
    pdl_wait();
    const int b = blockIdx.x / kHeads, h = blockIdx.x % kHeads, d = threadIdx.x;
    const float *base = partials + (size_t)b * bstride + (size_t)h * hstride;
    float M = -INFINITY;
    for (int i = 0; i < nparts; ++i) M = fmaxf(M, base[(size_t)i * pstride]);
    float L = 0.f, O = 0.f;
    if (M != -INFINITY) {
        for (int i = 0; i < nparts; ++i) {
            const float *pp = base + (size_t)i * pstride;
            if (pp[0] == -INFINITY) continue;  // empty key range
            const float f = ex2_approx(pp[0] - M);
            L += pp[1] * f;
            O += pp[2 + d] * f;
        }
    }
    if (emit) {
        float *e = emit + ((size_t)b * kHeads + h) * (kHeadDim + 2);
        if (d == 0) {
            e[0] = M;
            e[1] = L;
        }
        e[2 + d] = O;
    } else {
        out[(size_t)b * kHeads * kHeadDim + h * kHeadDim + d] = L > 0.f ? O / L : 0.f;
    }
}

// ------------------------------------------------------------------------
// Log-sum-exp merge of prefill outputs over disjoint key ranges (context-
// parallel ranks): part r holds, per token and head, the output O_r
// normalised over its keys and (m_r, l_r) from PrefillParams::ml_out.
// out = sum_r w_r O_r / sum_r w_r with w_r = l_r 2^(m_r - M), M the largest
// m_r among the parts with l_r > 0.  grid (T * 8), block 256 (one dim each);
// part r's outputs at outs + r * pstride, its (m, l) at mls + r * mstride
// (float2 units).
__global__ void __launch_bounds__(256) merge_prefill_partials(const float *__restrict__ outs, size_t pstride,
                                                             const float2 *__restrict__ mls, size_t mstride,
                                                             int nparts, float *__restrict__ out) {
    pdl_launch_dependents();
    pdl_wait();
    const int th = blockIdx.x, d = threadIdx.x;  // th = token * 8 + head
    float M = -INFINITY;
    for (int r = 0; r < nparts; ++r) {
        const float2 ml = mls[r * mstride + th];
        if (ml.y > 0.f) M = fmaxf(M, ml.x);
    }
    float W = 0.f, O = 0.f;
    if (M != -INFINITY) {
        for (int r = 0; r < nparts; ++r) {
            const float2 ml = mls[r * mstride + th];
            if (!(ml.y > 0.f)) continue;
            const float w = ml.y * ex2_approx(ml.x - M);
            W += w;
            O += w * outs[r * pstride + (size_t)th * kHeadDim + d];
        }
    }
    out[(size_t)th * kHeadDim + d] = W > 0.f ? O / W : 0.f;
}

// ------------------------------------------------------------------------
// Context-parallel exchange over peer memory (global layers split across
// GPUs).  Every rank owns a receive buffer [2 parity][R ranks][B][8][258]
// and flags [2 parity][8]; each rank maps all ranks' buffers (CUDA IPC).
// merge_partials_push merges this rank's split partials and stores the
// merged (m, l, O) of each (seq, head) straight into slot `me` of every
// rank's receive buffer over NVLink; its last CTA (grid ticket) then raises
// flag `me` of every rank to the exchange's epoch.  merge_peer_partials
// waits (bounded) until all R flags of this rank carry the epoch and merges
// the R partials into the output.  Exchange t uses parity t & 1: a rank can
// only start exchange t+2 after every rank has pushed t+1, which each rank
// does only after its merge of t, so a parity is never overwritten while a
// rank still reads it.
// ------------------------------------------------------------------------
constexpr int kMaxPeers = 8;
struct PeerXchg {
    float *gather[kMaxPeers];    // rank r's receive buffer (mapped here)
    unsigned *flags[kMaxPeers];  // rank r's flags [2][kMaxPeers]
    unsigned *counter;           // this rank's grid ticket (0 between calls)
    size_t rank_stride;          // floats per rank slot: max_batch * 8 * 258
    size_t parity_stride;        // R * rank_stride
    unsigned epoch;              // > 0, same sequence on every rank
    int me, R;
};

__device__ __forceinline__ unsigned ld_acquire_sys(const unsigned *p) {
    unsigned v;
    asm volatile("ld.acquire.sys.global.u32 %0, [%1];" : "=r"(v) : "l"(p) : "memory");
    return v;
}
__device__ __forceinline__ void st_release_sys(unsigned *p, unsigned v) {
    asm volatile("st.release.sys.global.u32 [%0], %1;" ::"l"(p), "r"(v) : "memory");
}

__global__ void __launch_bounds__(256) merge_partials_push(const float *__restrict__ partials, int nparts,
                                                           size_t bstride, size_t hstride, size_t pstride,
                                                           const PeerXchg px) {
    pdl_launch_dependents();
    pdl_wait();
    const int b = blockIdx.x / kHeads, h = blockIdx.x % kHeads, d = threadIdx.x;
    const float *base = partials + (size_t)b * bstride + (size_t)h * hstride;
    float M = -INFINITY;
    for (int i = 0; i < nparts; ++i) M = fmaxf(M, base[(size_t)i * pstride]);
    float L = 0.f, O = 0.f;
    if (M != -INFINITY) {
        for (int i = 0; i < nparts; ++i) {
            const float *pp = base + (size_t)i * pstride;
            if (pp[0] == -INFINITY) continue;
            const float f = ex2_approx(pp[0] - M);
            L += pp[1] * f;
            O += pp[2 + d] * f;
        }
    }
    const size_t off = (size_t)(px.epoch & 1u) * px.parity_stride + (size_t)px.me * px.rank_stride +
                       ((size_t)b * kHeads + h) * (kHeadDim + 2);
    for (int r = 0; r < px.R; ++r) {
        float *e = px.gather[r] + off;
        if (d == 0) {
            e[0] = M;
            e[1] = L;
        }
        e[2 + d] = O;
    }
    __threadfence_system();
    __syncthreads();
    if (threadIdx.x == 0) {
        if (atomicAdd(px.counter, 1u) == gridDim.x - 1) {
            // every CTA's stores are fenced before its ticket: publish
            *px.counter = 0u;
            __threadfence_system();
            for (int r = 0; r < px.R; ++r) st_release_sys(px.flags[r] + (px.epoch & 1u) * kMaxPeers + px.me, px.epoch);
        }
    }
}

__global__ void __launch_bounds__(256) merge_peer_partials(const PeerXchg px, float *__restrict__ out,
                                                           unsigned *err) {
    pdl_launch_dependents();
    pdl_wait();
    __shared__ int ok;
    const unsigned par = px.epoch & 1u;
    if (threadIdx.x == 0) {
        const unsigned *f = px.flags[px.me] + par * kMaxPeers;
        const uint64_t t0 = globaltimer_ns();
        bool good = true;
        for (int r = 0; good && r < px.R; ++r) {
            for (uint32_t i = 1; ld_acquire_sys(f + r) != px.epoch; ++i) {
                if ((i & 63u) == 0 && (*(volatile unsigned *)err || globaltimer_ns() - t0 > kWaitLimitNs)) {
                    good = false;
                    break;
                }
            }
        }
        if (!good) raise_status(err, kErrWaitTimeout);
        ok = good;
    }
    __syncthreads();
    if (!ok) return;
    const int b = blockIdx.x / kHeads, h = blockIdx.x % kHeads, d = threadIdx.x;
    const float *base = px.gather[px.me] + (size_t)par * px.parity_stride + ((size_t)b * kHeads + h) * (kHeadDim + 2);
    float M = -INFINITY;
    for (int r = 0; r < px.R; ++r) M = fmaxf(M, __ldcg(base + (size_t)r * px.rank_stride));
    float L = 0.f, O = 0.f;
    if (M != -INFINITY) {
        for (int r = 0; r < px.R; ++r) {
            const float *pp = base + (size_t)r * px.rank_stride;
            const float m = __ldcg(pp);
            if (m == -INFINITY) continue;
            const float f = ex2_approx(m - M);
            L += __ldcg(pp + 1) * f;
            O += __ldcg(pp + 2 + d) * f;
        }
    }
    out[(size_t)b * kHeads * kHeadDim + h * kHeadDim + d] = L > 0.f ? O / L : 0.f;
}

// ------------------------------------------------------------------------
// Prefill flash attention on tcgen05 / TMEM (persistent CTAs).
//
// Work unit = (block of 64 query tokens, kv head g); the MMA M dimension
// stacks the two query heads of the group (rows 0-63 head 2g, 64-127 head
// 2g+1), so each K/V tile feeds both.  One CTA per SM walks the units
// heaviest first (snake rounds over the cost-sorted list).
// Per key tile of 128 rows:
//     S[128x128] = Q[128x256] . K^T   16 MMAs (K=16), A = Q and B = K from
//                                      shared memory into TMEM
//     softmax    warps 0-7: row r is shared by threads r (keys 0-63, O cols
//                0-127) and r+128 (keys 64-127, O cols 128-255); S is freed
//                for the next tile's MMAs as soon as it is in registers; P
//                goes back to TMEM as fp16 pairs (two buffers), in two chunks
//     O[128x256] += P[128x128] . V    8 MMAs (K=16); A = P from TMEM, B = V
//                                      (MN-major) from shared memory
// A tcgen05.mma of M=128, K=16 costs at least ~64 cycles whatever its N, so
// S is computed 128 keys at a time (N=128: full rate) rather than 64 (half
// rate); the PV MMAs (N=256) run at full rate either way.  Warp 8 issues
// the TMA loads, warp 9 the S MMAs, warp 10 the PV MMAs (one lane each), so
// each MMA goes to the tensor pipe as soon as its own operands are ready.
// Warps 11-14 write each finished unit's O / l while the softmax warps work
// on the next unit.  Operands are fp16 (see prologue_prefill), accumulation
// fp32.
//
// TMEM columns (512): S 0-127 (fp32), P 128-191 and 192-255 (fp16 pairs),
// O 256-511 (fp32).  With P apart from S, S(j+1) runs while the softmax of
// tile j computes its exponentials; had P been written over S (two S
// buffers), S(j+2) would wait for PV(j), which waits for the softmax of j,
// and that chain of S + softmax + PV per two tiles was measured at ~1.2x
// the period of this layout.
//
// Online softmax with a lazily updated reference max: P = 2^(s*c - m) is
// computed against the row's current reference m, which is only raised
// (rescaling l and the TMEM-resident O by 2^(m_old - m_new)) when the tile
// max exceeds it by more than kRescaleLog2; otherwise P <= 2^kRescaleLog2 =
// 256, exact in fp16, and the result is mathematically unchanged.
//
// Shared memory (1024-aligned, 128-B swizzle for every MMA operand):
//     Q 64 KB: 4 dim-blocks x [128 rows x 128 B], resident for the unit
//     ring of 5 slots x 32 KB, filled in the order the MMAs consume them:
//         K half h of a tile: 2 dim-blocks (2h, 2h+1) x [128 keys x 128 B]
//         V half h of a tile: 4 dim-blocks x [64 keys (64h..) x 128 B]
//       per unit of n tiles: K0, K1, V0, K2, V1, ..., K(n-1), V(n-2), V(n-1)
//       (each item two slots), so S(j+1) never waits behind V(j)
//     barriers, row-max (bf16) / row-sum exchange
// All mbarrier phases run on per-CTA counters (tile counter gi, unit counter
// uk, ring position) that continue across units.
// ------------------------------------------------------------------------
constexpr int kPfMaxCtas = 160;
constexpr int kPfTK = 128;  // keys per tile
struct PrefillParams {
    float *out;       // [T][8][256]
    int T;
    int start_pos;
    int kv_pos0;      // position of K/V row 0
    int kv_end;       // one past the last key position staged (keys >= kv_end are not attended)
    float2 *ml_out;   // null, or [T][8] (m, l) of every output row: its reference max (log2
                      // domain) and softmax sum, so that outputs over disjoint key ranges of
                      // the same queries (context-parallel ranks) can be merged
    int is_global;
    int nqb;          // query blocks of 64 tokens
    unsigned *err;
    // Work schedule.  sched 0: cost-sorted units dealt to the CTAs in
    // snake-order rounds.  sched 1 (local layers, whose units are all of
    // near-equal cost, when the unit count is not a multiple of the grid):
    // the nunits - nfull units left over after the full rounds are cut into
    // `split` key-range pieces each and run FIRST, one piece per CTA (piece
    // q = blockIdx.x: unit nfull + q / split, part q % split); then come the
    // nfull units in full snake rounds.  Each piece writes its unnormalised
    // (O, m, l) to scratch slot q; the last piece of a unit to finish
    // (ticket q / split) merges the unit's pieces into out while its CTA
    // already computes the next unit.  Keeping the rounds keeps the units
    // that share K/V tiles close in time (L2 reuse), which a contiguous cut
    // of the unit list per CTA loses.
    int sched;
    int nfull;           // units in full rounds (a multiple of gridDim.x)
    int split;           // pieces per left-over unit (2..4)
    float *pscratch;     // [kPfMaxCtas][128][256]
    float2 *pml;         // [kPfMaxCtas][128] (m, l), m in the log2 domain
    unsigned *ptickets;  // [kPfMaxCtas], zero between launches
};

// bar.red.and over `count` threads on named barrier `id`: true iff every
// participating thread passed pred != 0.
__device__ __forceinline__ bool named_bar_and(uint32_t id, uint32_t count, bool pred) {
    uint32_t r;
    asm volatile(
        "{\n\t.reg .pred p, q;\n\t"
        "setp.ne.u32 q, %1, 0;\n\t"
        "bar.red.and.pred p, %2, %3, q;\n\t"
        "selp.u32 %0, 1, 0, p;\n\t}"
        : "=r"(r)
        : "r"((uint32_t)pred), "r"(id), "r"(count)
        : "memory");
    return r != 0;
}

constexpr int kPfSoftmaxThreads = 256;
constexpr int kPfThreads = kPfSoftmaxThreads + 96 + 128;  // + producer, two MMA warps, 4 epilogue warps
constexpr int kPfWarpTma = 8;
constexpr int kPfWarpMma = 9;  // S MMAs; also owns the TMEM allocation
constexpr int kPfWarpPv = 10;  // PV MMAs
constexpr int kPfWarpEpi = 11; // 11-14: epilogue, one per TMEM lane quadrant
constexpr float kRescaleLog2 = 8.0f;

constexpr uint32_t kPfQBytes = 128 * 256 * 2;
constexpr uint32_t kPfSlot = 32768;
constexpr int kPfSlots = 5;
constexpr uint32_t kPfOffQ = 0;
constexpr uint32_t kPfOffRing = kPfOffQ + kPfQBytes;
constexpr uint32_t kPfOffBar = kPfOffRing + kPfSlots * kPfSlot;
constexpr uint32_t kPfOffRed = kPfOffBar + 256;
// row-max exchange: bf16 [2 parity][2 half][128] (1 KB); row sums fp32 [2 half][128] (1 KB)
// + the rows' reference maxima for the piece partials, fp32 [128] (512 B)
constexpr uint32_t kPfSmem = kPfOffRed + 2560;  // 232,192 B: needs a 1024-aligned base (checked)
constexpr uint32_t kTmemCols = 512;
constexpr uint32_t kTmemS = 0;
constexpr uint32_t kTmemP = 128;  // buffer b at kTmemP + 64 b
constexpr uint32_t kTmemO = 256;

// Ring item of tile j of a unit of n tiles (items of 2 slots each):
// K(0) = 0, K(j) = 2j - 1; V(j) = 2j + 2 for j < n - 1, V(n-1) = 2n - 1.
__device__ __forceinline__ int pf_item_k(int j) { return j == 0 ? 0 : 2 * j - 1; }
__device__ __forceinline__ int pf_item_v(int j, int n) { return j < n - 1 ? 2 * j + 2 : 2 * n - 1; }

// The unit list: index -> (query block, kv head), costliest blocks first
// (causal rows grow with the block index; local-layer blocks are equal).
struct PfUnit {
    int t0, qlo, qhi, j0, ntiles, g;
    int slot, tix;    // piece of a cut unit: scratch slot and ticket; -1 for a whole unit
    int first, nparts;  // the unit's pieces occupy slots first .. first + nparts - 1
};
// Unit k of this CTA: the cost-sorted list is dealt out in rounds of
// gridDim.x, alternating direction each round (snake order), which evens out
// the per-CTA totals of the causal cost ramp.  -1 when the round is short.
__device__ __forceinline__ int pf_unit_index(int k, int nunits) {
    const int G = gridDim.x;
    const int idx = k * G + ((k & 1) ? (G - 1 - (int)blockIdx.x) : (int)blockIdx.x);
    return idx < nunits ? idx : -1;
}
__device__ __forceinline__ int pf_unit_rounds(int nunits) { return (nunits + gridDim.x - 1) / gridDim.x; }

__device__ __forceinline__ PfUnit pf_unit(const PrefillParams &p, int idx) {
    PfUnit u;
    const int qb = p.nqb - 1 - idx / kKvHeads;
    u.g = idx % kKvHeads;
    u.t0 = qb * 64;
    u.qlo = p.start_pos + u.t0;
    u.qhi = p.start_pos + min(u.t0 + 64, p.T) - 1;
    const int kmin = max(p.kv_pos0, p.is_global ? 0 : u.qlo - (kWindow - 1));
    const int kmax = min(u.qhi, p.kv_end - 1);  // >= kmin: the host launches only queries >= kv_pos0
    u.j0 = (kmin - p.kv_pos0) / kPfTK;
    u.ntiles = (kmax - p.kv_pos0) / kPfTK + 1 - u.j0;
    u.slot = u.tix = u.first = -1;
    u.nparts = 1;
    return u;
}

// Items of this CTA (units or pieces of cut units), in processing order.
__device__ __forceinline__ int pf_count(const PrefillParams &p, int nunits) {
    if (!p.sched) return pf_unit_rounds(nunits);
    return 1 + p.nfull / (int)gridDim.x;
}
// Item k; false when this CTA has no unit / piece in that round.
__device__ __forceinline__ bool pf_get(const PrefillParams &p, int nunits, int k, PfUnit &u) {
    if (!p.sched) {
        const int idx = pf_unit_index(k, nunits);
        if (idx < 0) return false;
        u = pf_unit(p, idx);
        return true;
    }
    if (k > 0) {
        u = pf_unit(p, pf_unit_index(k - 1, p.nfull));
        return true;
    }
    const int q = blockIdx.x;
    const int idx = p.nfull + q / p.split, part = q % p.split;
    if (idx >= nunits) return false;
    u = pf_unit(p, idx);
    const int n = u.ntiles, np = min(p.split, n);
    if (part >= np) return false;  // a unit of fewer tiles than `split` has fewer pieces
    const int lo = n * part / np, hi = n * (part + 1) / np;
    u.j0 += lo;
    u.ntiles = hi - lo;
    u.slot = q;
    u.first = q - part;
    u.nparts = np;
    u.tix = q / p.split;
    return true;
}

__global__ void __launch_bounds__(kPfThreads, 1)
    prefill_fa_sm100(const __grid_constant__ CUtensorMap tmQ, const __grid_constant__ CUtensorMap tmK,
                     const __grid_constant__ CUtensorMap tmV, const PrefillParams p) {
    extern __shared__ __align__(1024) unsigned char smem_raw[];
    // The 128-byte-swizzled TMA / MMA tiles need 1024-byte alignment and the
    // layout uses all of the 227 KB, so there is no room to realign: refuse
    // to run (status bit, no memory touched) if the base is not aligned.
    if (smem_u32(smem_raw) & 1023u) {
        if (threadIdx.x == 0) raise_status(p.err, kErrBadIndex);
        return;
    }
    unsigned char *sm = smem_raw;
    unsigned char *sQ = sm + kPfOffQ;
    unsigned char *sR = sm + kPfOffRing;
    __nv_bfloat16 *redm = reinterpret_cast<__nv_bfloat16 *>(sm + kPfOffRed);  // [2 parity][2 half][128] maxima
    float *reds = reinterpret_cast<float *>(sm + kPfOffRed + 1024);             // [2 half][128] row sums
    float *redmx = reinterpret_cast<float *>(sm + kPfOffRed + 2048);            // [128] row reference maxima
    uint64_t *bars = reinterpret_cast<uint64_t *>(sm + kPfOffBar);
    uint64_t *q_full = bars + 0;    // Q tile landed (TMA)
    uint64_t *q_empty = bars + 1;   // the unit's S MMAs have read Q
    uint64_t *r_full = bars + 2;    // [5] ring slot landed
    uint64_t *r_empty = bars + 7;   // [5] ring slot read by its MMAs
    uint64_t *s_full = bars + 12;   // S written
    uint64_t *s_free = bars + 13;   // 256 arrivals: the softmax has read S
    uint64_t *p_empty = bars + 14;  // [2] PV done: P buffer read, O updated
    uint64_t *mma_done = bars + 16;
    uint64_t *mma_done_pv = bars + 17;
    uint64_t *p_full = bars + 18;   // [2 buffers][2 chunks], 256 arrivals: P chunk written over S
    uint64_t *fin_bar = bars + 22;  // 256 arrivals, once per unit
    uint64_t *o_free = bars + 23;   // 128 arrivals: the epilogue warps have read O
    uint32_t *tmem_slot = reinterpret_cast<uint32_t *>(bars + 24);
    volatile int *s_abort = reinterpret_cast<volatile int *>(bars + 25);
    uint64_t *epi_bar = bars + 26;  // 128 arrivals: epilogue-internal steps
    volatile int *s_last = reinterpret_cast<volatile int *>(bars + 28);  // epilogue: piece merges

    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const int nunits = p.nqb * kKvHeads;

    if (threadIdx.x == 0) {
        for (int i = 0; i < 24; ++i) mbar_init(&bars[i], 1);
        for (int b = 0; b < 4; ++b) mbar_init(&p_full[b], kPfSoftmaxThreads);
        mbar_init(s_free, kPfSoftmaxThreads);
        mbar_init(fin_bar, kPfSoftmaxThreads);
        mbar_init(o_free, 128);
        mbar_init(epi_bar, 128);
        *s_abort = 0;
        fence_mbar_init();
    }
    if (warp == kPfWarpMma) tmem_alloc(tmem_slot, kTmemCols);
    tc_fence_before();
    __syncthreads();
    tc_fence_after();
    const uint32_t tmem = *tmem_slot;
    // dependent launch: the set-up above overlaps the prologue's tail; global
    // memory (staging, outputs, tickets) is touched only after it completed
    pdl_launch_dependents();
    pdl_wait();

    const int nitems = pf_count(p, nunits);
    if (warp == kPfWarpTma) {
        // ------------------------------------------------ TMA producer
        if (lane == 0) {
            prefetch_tmap(&tmQ);
            prefetch_tmap(&tmK);
            prefetch_tmap(&tmV);
            int uk = 0, rb = 0;  // unit counter, ring position of the unit's first slot
            int last_pos[kPfSlots];  // last ring position issued per slot (for the abort drain)
            int q_issued = 0;        // Q copies issued
#pragma unroll
            for (int s = 0; s < kPfSlots; ++s) last_pos[s] = -1;
            for (int k = 0; k < nitems && !*s_abort; ++k) {
                PfUnit u;
                if (!pf_get(p, nunits, k, u)) continue;
                const int ukc = uk++;
                const int n = u.ntiles;
                bool ok = true;
                for (int t = 0; ok && t < 2 * n; ++t) {
                    if (t == 1) {
                        // Q of this unit (after its first K tile, whose copy then
                        // overlaps the wait), once the previous unit's S MMAs
                        // have read theirs
                        if (ukc >= 1 && !mbar_wait(q_empty, (ukc - 1) & 1, p.err)) { ok = false; break; }
                        mbar_expect_tx(q_full, kPfQBytes);
                        for (int c = 0; c < 4; ++c)
                            for (int hh = 0; hh < 2; ++hh)
                                tma_load_3d(sQ + c * 16384 + hh * 8192, &tmQ, 64 * c, u.t0, 2 * u.g + hh, q_full);
                        q_issued = ukc + 1;
                    }
                    const bool isv = t == 2 * n - 1 || (t > 0 && !(t & 1));
                    const int j = t == 2 * n - 1 ? n - 1 : isv ? (t - 2) / 2 : (t + 1) / 2;
                    const int krow = (u.j0 + j) * kPfTK;
                    for (int h = 0; h < 2; ++h) {
                        const int pos = rb + 2 * t + h, s = pos % kPfSlots, ph = pos / kPfSlots;
                        if (ph >= 1 && !mbar_wait(&r_empty[s], (ph - 1) & 1, p.err)) { ok = false; break; }
                        mbar_expect_tx(&r_full[s], kPfSlot);
                        if (isv)
                            tma_load_4d(sR + s * kPfSlot, &tmV, 0, krow + 64 * h, 0, u.g, &r_full[s]);
                        else
                            tma_load_4d(sR + s * kPfSlot, &tmK, 0, krow, 2 * h, u.g, &r_full[s]);
                        last_pos[s] = pos;
                    }
                }
                if (!ok) { *s_abort = 1; break; }
                rb += 4 * n;
            }
            // wait (bounded) for the copies in flight before the CTA exits
            if (*s_abort) {
                if (q_issued >= 1) mbar_wait(q_full, (q_issued - 1) & 1, nullptr);
                for (int s = 0; s < kPfSlots; ++s)
                    if (last_pos[s] >= 0) mbar_wait(&r_full[s], (last_pos[s] / kPfSlots) & 1, nullptr);
            }
        }
    } else if (warp == kPfWarpMma) {
        // ------------------------------------------------ S = Q.K^T
        if (lane == 0) {
            constexpr uint32_t idS = idesc_f16_f32(128, kPfTK, 0, 0);
            // Descriptors are built once; per MMA only the start-address field
            // (bits 0-13, address >> 4, no carry for addresses < 256 KB)
            // advances.
            const uint64_t dQ = smem_desc_sw128(smem_u32(sQ), 16, 1024);
            const uint64_t dR = smem_desc_sw128(smem_u32(sR), 16, 1024);
            bool ok = true;
            int gi = 0, uk = 0, rb = 0;
            for (int k = 0; ok && k < nitems; ++k) {
                PfUnit u;
                if (!pf_get(p, nunits, k, u)) continue;
                const int ukc = uk++;
                const int n = u.ntiles;
                if (*s_abort || !mbar_wait(q_full, ukc & 1, p.err)) { ok = false; break; }
                for (int i = 0; i < n; ++i, ++gi) {
                    if (*s_abort) { ok = false; break; }
                    const int pos0 = rb + 2 * pf_item_k(i);
                    const int s0 = pos0 % kPfSlots, s1 = (pos0 + 1) % kPfSlots;
                    if (!mbar_wait(&r_full[s0], (pos0 / kPfSlots) & 1, p.err) ||
                        !mbar_wait(&r_full[s1], ((pos0 + 1) / kPfSlots) & 1, p.err)) {
                        ok = false;
                        break;
                    }
                    // S is free once the softmax has loaded the previous one
                    if (gi >= 1 && !mbar_wait(s_free, (gi - 1) & 1, p.err)) { ok = false; break; }
                    tc_fence_after();
                    const uint32_t dS = tmem + kTmemS;
#pragma unroll
                    for (int kk = 0; kk < 16; ++kk) {
                        const int s = kk < 8 ? s0 : s1;
                        const uint64_t a = dQ + (uint64_t)(((kk >> 2) * 16384 + (kk & 3) * 32) >> 4);
                        const uint64_t b =
                            dR + (uint64_t)((s * kPfSlot + ((kk >> 2) & 1) * 16384 + (kk & 3) * 32) >> 4);
                        tc_mma_f16(dS, a, b, idS, kk > 0 ? 1u : 0u);
                    }
                    tc_commit(&r_empty[s0]);
                    tc_commit(&r_empty[s1]);
                    tc_commit(s_full);
                }
                if (!ok) break;
                tc_commit(q_empty);
                rb += 4 * n;
            }
            if (!ok) *s_abort = 1;
            // Drain: every tcgen05 operation this thread issued has completed.
            tc_commit(mma_done);
            mbar_wait(mma_done, 0, nullptr);
        }
    } else if (warp == kPfWarpPv) {
        // ------------------------------------------------ O += P.V
        if (lane == 0) {
            constexpr uint32_t idO = idesc_f16_f32(128, 256, 0, 1);
            const uint64_t dR = smem_desc_sw128(smem_u32(sR), 8192, 1024);
            bool ok = true;
            int gi = 0, uk = 0, rb = 0;
            for (int k = 0; ok && k < nitems; ++k) {
                PfUnit u;
                if (!pf_get(p, nunits, k, u)) continue;
                const int ukc = uk++;
                const int n = u.ntiles;
                for (int i = 0; i < n; ++i, ++gi) {
                    if (*s_abort) { ok = false; break; }
                    const int b = gi & 1;
                    const int pos0 = rb + 2 * pf_item_v(i, n);
                    const int s0 = pos0 % kPfSlots, s1 = (pos0 + 1) % kPfSlots;
                    if (!mbar_wait(&r_full[s0], (pos0 / kPfSlots) & 1, p.err) ||
                        !mbar_wait(&r_full[s1], ((pos0 + 1) / kPfSlots) & 1, p.err)) {
                        ok = false;
                        break;
                    }
                    // the first PV of a unit overwrites O: the previous unit's
                    // epilogue must have read it
                    if (i == 0 && ukc >= 1 && !mbar_wait(o_free, (ukc - 1) & 1, p.err)) { ok = false; break; }
                    const uint32_t aP = tmem + kTmemP + b * 64;
                    // P arrives in two chunks (keys 32c..32c+31 of each half):
                    // chunk c feeds the MMAs of keys 16kk.. for kk = 2c, 2c+1
                    // (V half 0) and 4+2c, 5+2c (V half 1)
                    for (int c = 0; c < 2 && ok; ++c) {
                        if (!mbar_wait(&p_full[2 * b + c], (gi >> 1) & 1, p.err)) { ok = false; break; }
                        tc_fence_after();
#pragma unroll
                        for (int q = 0; q < 4; ++q) {
                            const int kk = (q >> 1) * 4 + 2 * c + (q & 1);
                            const int s = kk < 4 ? s0 : s1;
                            tc_mma_f16_ts(tmem + kTmemO, aP + kk * 8,
                                          dR + (uint64_t)((s * kPfSlot + (kk & 3) * 2048) >> 4), idO,
                                          (i > 0 || c > 0 || q > 0) ? 1u : 0u);
                        }
                    }
                    if (!ok) break;
                    tc_commit(&r_empty[s0]);
                    tc_commit(&r_empty[s1]);
                    tc_commit(&p_empty[b]);
                }
                rb += 4 * n;
            }
            if (!ok) *s_abort = 1;
            tc_commit(mma_done_pv);
            mbar_wait(mma_done_pv, 0, nullptr);
        }
    } else if (warp >= kPfWarpEpi) {
        // ------------------------------------------------ epilogue warps
        // O / (l_half0 + l_half1) -> out[t][2g+hh][:], one warp per TMEM lane
        // quadrant, thread = row.  Per 32-column chunk, each group of 4
        // lanes transposes its 4 rows x 4 blocks of 8 floats with two xor-
        // shuffle stages, so that a store instruction writes 8 rows x 64
        // contiguous bytes (8 L1 wavefronts) instead of 32 rows x 16 bytes
        // (32 wavefronts): all CTAs of a local layer finish their units
        // together, and the scattered form kept the LSU busy for ~8k cycles
        // per unit, stalling the softmax warps' TMEM loads.  O is released
        // to the next unit's PV right after the last TMEM read.
        const int quad = warp & 3;
        const int row = quad * 32 + lane;
        const uint32_t lane_base = tmem + ((uint32_t)(quad * 32) << 16);
        bool ok = true;
        int gi = 0, uk = 0, eph = 0;
        auto epi_sync = [&]() {
            mbar_arrive(epi_bar);
            const bool w = mbar_wait(epi_bar, eph & 1, p.err);
            ++eph;
            return __all_sync(0xffffffffu, w);
        };
        for (int k = 0; ok && k < nitems; ++k) {
            PfUnit u;
            if (!pf_get(p, nunits, k, u)) continue;
            const int ukc = uk++;
            gi += u.ntiles;
            const int gl = gi - 1;  // the unit's last tile
            if (!__all_sync(0xffffffffu, !*s_abort && mbar_wait(fin_bar, ukc & 1, p.err) &&
                                             mbar_wait(&p_empty[gl & 1], (gl >> 1) & 1, p.err))) {
                ok = false;
                break;
            }
            tc_fence_after();
            const float lt = reds[row] + reds[128 + row];
            // a piece of a cut unit leaves O unnormalised, with (m, l) beside it
            const bool piece = u.slot >= 0;
            const float inv = piece ? 1.0f : lt > 0.f ? 1.0f / lt : 0.f;
            if (piece) p.pml[(size_t)u.slot * 128 + row] = make_float2(redmx[row], lt);
            const int nvalid = min(64, p.T - u.t0);
            if (p.ml_out && !piece && (row & 63) < nvalid)
                p.ml_out[(size_t)(u.t0 + (row & 63)) * kHeads + 2 * u.g + (row >> 6)] = make_float2(redmx[row], lt);
            const int q4 = lane & 3, r4 = quad * 32 + (lane & ~3);  // group's first row
#pragma unroll 1
            for (int cc = 0; cc < 8; ++cc) {
                float o[32];
                tmem_ld32(lane_base + kTmemO + cc * 32, o);
                tc_wait_ld();
                if (cc == 7) {
                    // all of O read from TMEM: the next unit's PV may overwrite it
                    tc_fence_before();
                    mbar_arrive(o_free);
                }
                float4 v[8];
#pragma unroll
                for (int k = 0; k < 8; ++k)
                {
                    const float2 i2 = make_float2(inv, inv);
                    const float2 lo = fmul2(make_float2(o[4 * k], o[4 * k + 1]), i2);
                    const float2 hi = fmul2(make_float2(o[4 * k + 2], o[4 * k + 3]), i2);
                    v[k] = make_float4(lo.x, lo.y, hi.x, hi.y);
                }
                // lane q4 of the group: blocks kb = (v[kb], v[kb + 4]) of row r4 + q4
                // -> block q4 of row r4 + kb (cols 4 q4.. and 16 + 4 q4..)
#pragma unroll
                for (int m = 2; m >= 1; m >>= 1) {
                    const bool up = (q4 & m) != 0;
#pragma unroll
                    for (int k0 = 0; k0 < 8; ++k0) {
                        if ((k0 & 3) & m) continue;
                        float4 &a = v[k0], &b = v[k0 | m];
                        const float4 snd = up ? a : b;
                        float4 rcv;
                        rcv.x = __shfl_xor_sync(0xffffffffu, snd.x, m);
                        rcv.y = __shfl_xor_sync(0xffffffffu, snd.y, m);
                        rcv.z = __shfl_xor_sync(0xffffffffu, snd.z, m);
                        rcv.w = __shfl_xor_sync(0xffffffffu, snd.w, m);
                        if (up) a = rcv; else b = rcv;
                    }
                }
#pragma unroll
                for (int k = 0; k < 4; ++k) {
                    const int r = r4 + k;
                    if (!piece && (r & 63) >= nvalid) continue;
                    float *rd = piece ? p.pscratch + ((size_t)u.slot * 128 + r) * kHeadDim
                                      : p.out + ((size_t)(u.t0 + (r & 63)) * kHeads + 2 * u.g + (r >> 6)) * kHeadDim;
                    *reinterpret_cast<float4 *>(rd + cc * 32 + 4 * q4) = v[k];
                    *reinterpret_cast<float4 *>(rd + cc * 32 + 16 + 4 * q4) = v[k + 4];
                }
            }
            if (piece) {
                // Every piece of the cut unit publishes; the last to arrive
                // merges them (the CTA's MMA / softmax warps meanwhile run
                // the next item).  No waiting on the other CTAs.
                __threadfence();
                if (!epi_sync()) { ok = false; break; }
                if (threadIdx.x == kPfWarpEpi * 32) {
                    const unsigned old = atomicAdd(&p.ptickets[u.tix], 1u);
                    *s_last = old == (unsigned)(u.nparts - 1) ? 1 : 0;
                    if (*s_last) p.ptickets[u.tix] = 0u;  // ready for the next launch
                }
                if (!epi_sync()) { ok = false; break; }
                if (*s_last) {
                    __threadfence();
                    const int np = u.nparts;
                    const float *o0 = p.pscratch + (size_t)u.first * 128 * kHeadDim;
                    const float2 *m0 = p.pml + (size_t)u.first * 128;
                    // lane = row of this warp's 32: each piece's weight, normalised
                    const int rr = quad * 32 + lane;
                    float wm[4], M = -INFINITY;
#pragma unroll
                    for (int j = 0; j < 4; ++j) {
                        wm[j] = -INFINITY;
                        if (j < np) {
                            const float2 a = __ldcg(m0 + (size_t)j * 128 + rr);
                            wm[j] = a.x;
                            M = fmaxf(M, a.x);
                        }
                    }
                    float Lr = 0.f;
#pragma unroll
                    for (int j = 0; j < 4; ++j) {
                        const float w = wm[j] == -INFINITY ? 0.f : ex2_approx(wm[j] - M);
                        if (j < np) Lr += __ldcg(m0 + (size_t)j * 128 + rr).y * w;
                        wm[j] = w;
                    }
                    const float il = Lr > 0.f ? 1.0f / Lr : 0.f;
#pragma unroll
                    for (int j = 0; j < 4; ++j) wm[j] *= il;
                    // warp = 32 rows, lanes along the 64 float4 of a row, 2 rows per batch
                    for (int r0 = 0; r0 < 32; r0 += 2) {
                        float4 acc[2][2];
#pragma unroll
                        for (int jr = 0; jr < 2; ++jr)
#pragma unroll
                            for (int h2 = 0; h2 < 2; ++h2) acc[jr][h2] = make_float4(0.f, 0.f, 0.f, 0.f);
#pragma unroll
                        for (int j = 0; j < 4; ++j) {
                            if (j >= np) break;
                            float4 x[2][2];
#pragma unroll
                            for (int jr = 0; jr < 2; ++jr)
#pragma unroll
                                for (int h2 = 0; h2 < 2; ++h2)
                                    x[jr][h2] = __ldcg(reinterpret_cast<const float4 *>(
                                                           o0 + ((size_t)j * 128 + quad * 32 + r0 + jr) * kHeadDim) +
                                                       lane + 32 * h2);
#pragma unroll
                            for (int jr = 0; jr < 2; ++jr) {
                                const float w = __shfl_sync(0xffffffffu, wm[j], r0 + jr);
#pragma unroll
                                for (int h2 = 0; h2 < 2; ++h2) {
                                    acc[jr][h2].x += x[jr][h2].x * w;
                                    acc[jr][h2].y += x[jr][h2].y * w;
                                    acc[jr][h2].z += x[jr][h2].z * w;
                                    acc[jr][h2].w += x[jr][h2].w * w;
                                }
                            }
                        }
#pragma unroll
                        for (int jr = 0; jr < 2; ++jr) {
                            const int r = quad * 32 + r0 + jr;
                            if ((r & 63) >= nvalid) continue;
                            float4 *dst = reinterpret_cast<float4 *>(
                                p.out + ((size_t)(u.t0 + (r & 63)) * kHeads + 2 * u.g + (r >> 6)) * kHeadDim);
#pragma unroll
                            for (int h2 = 0; h2 < 2; ++h2) dst[lane + 32 * h2] = acc[jr][h2];
                        }
                    }
                }
            }
        }
        if (!ok) *s_abort = 1;
    } else {
        // ------------------------------------------------ softmax warps 0-7
        // Warps w and w + 4 share TMEM lanes 32 (w % 4) .. + 31: thread r of
        // one and thread r of the other hold the two halves of a row, and
        // exchange the row maximum through shared memory behind a 64-thread
        // named barrier (id 1 + w % 4).  Every exit from the tile loop goes
        // through that barrier (bar.red.and of both warps' status), so a
        // failed wait in one warp never leaves its partner at the barrier.
        const int row = threadIdx.x & 127;  // TMEM lane == S/O row
        const int half = threadIdx.x >> 7;  // keys [64*half, +64), O cols [128*half, +128)
        const int tr = row & 63;
        const uint32_t pair_bar = 1 + (warp & 3);
        const uint32_t lane_base = tmem + ((uint32_t)((warp & 3) * 32) << 16);
        bool ok = true, fail = false;
        int gi = 0, uk = 0;
        for (int k = 0; ok && k < nitems; ++k) {
            PfUnit u;
            if (!pf_get(p, nunits, k, u)) continue;
            const int ukc = uk++;
            const int qpos = p.start_pos + u.t0 + tr;
            const int lo_ok = p.is_global ? INT_MIN : qpos - (kWindow - 1);
            const int hi_ok = min(qpos, p.kv_end - 1);   // last key of the row: causal, and staged here
            const int hi_unit = min(u.qlo, p.kv_end - 1);  // tiles past it hold some masked key
            float m = -INFINITY;  // reference max of the row, log2 domain
            float l = 0.f;        // this half's share of the row sum
            for (int i = 0; i < u.ntiles; ++i, ++gi) {
                const int b = gi & 1;
                const uint32_t pbuf = lane_base + kTmemP + b * 64;
                // every wait's outcome is made warp-uniform so the warp-collective
                // tcgen05 and vote instructions below never run diverged
                const bool w = !fail && __all_sync(0xffffffffu, !*s_abort && mbar_wait(s_full, gi & 1, p.err));
                float xa[32], xb[32];  // keys 64*half + 0..31, + 32..63
                float mx = -INFINITY;
                if (w) {
                    tc_fence_after();
                    tmem_ld32(lane_base + kTmemS + half * 64, xa);
                    tmem_ld32(lane_base + kTmemS + half * 64 + 32, xb);
                    tc_wait_ld();
                    tc_fence_before();
                    mbar_arrive(s_free);  // the next tile's S MMAs may overwrite it
                    const int tb = p.kv_pos0 + (u.j0 + i) * kPfTK;  // position of the tile's first key
                    const bool edge = (tb + kPfTK - 1 > hi_unit) || (!p.is_global && tb < u.qhi - (kWindow - 1));
                    if (edge) {
                        // valid keys of the row among this half's 64: one bit each
                        const int kb = tb + half * 64;
                        const int lo = lo_ok <= kb ? 0 : min(lo_ok - kb, 64);
                        const int hi = hi_ok >= kb + 63 ? 63 : hi_ok - kb;  // may be < 0
                        const uint64_t vm = (lo > hi) ? 0ull : ((~0ull >> (63 - hi)) & (~0ull << lo));
                        const uint32_t ma = (uint32_t)vm, mb = (uint32_t)(vm >> 32);
#pragma unroll
                        for (int k = 0; k < 32; ++k) {
                            if (!((ma >> k) & 1u)) xa[k] = -INFINITY;
                            if (!((mb >> k) & 1u)) xb[k] = -INFINITY;
                        }
                    }
                    // four independent chains
                    float m4[4];
#pragma unroll
                    for (int c = 0; c < 4; ++c) m4[c] = fmaxf(xa[c], xb[c]);
#pragma unroll
                    for (int k = 4; k < 32; ++k) m4[k & 3] = fmaxf(m4[k & 3], fmaxf(xa[k], xb[k]));
                    mx = fmaxf(fmaxf(m4[0], m4[1]), fmaxf(m4[2], m4[3]));
                }
                // exchanged in bf16 rounded up: both halves then use the same
                // value, not below the true max (P stays <= 2^kRescaleLog2)
                const __nv_bfloat16 mine = __float2bfloat16_ru(mx * kScaleLog2);
                redm[(b * 2 + half) * 128 + row] = mine;
                tc_fence_before();
                if (!named_bar_and(pair_bar, 64, w)) {
                    ok = false;
                    break;
                }
                tc_fence_after();
                mx = fmaxf(__bfloat162float(mine), __bfloat162float(redm[(b * 2 + (half ^ 1)) * 128 + row]));
                const bool raise = mx > m + kRescaleLog2;  // false while the row has no valid key
                const float m_new = raise ? mx : m;
                const float alpha = raise ? ex2_approx(m - m_new) : 1.f;
                // a row without a valid key so far has O = 0 and l = 0: its
                // first real maximum needs no rescale (alpha = 0 leaves l exact);
                // local units' first tile (window edge) leaves many such rows.
                // O is written by PV(gi-1): a rescale waits for it.
                const bool rescale = i >= 1 && __any_sync(0xffffffffu, raise && m != -INFINITY);
                // P buffer b was last read by PV(gi - 2)
                if ((gi >= 2 && !__all_sync(0xffffffffu, mbar_wait(&p_empty[b], ((gi - 2) >> 1) & 1, p.err))) ||
                    (rescale && !__all_sync(0xffffffffu, mbar_wait(&p_empty[b ^ 1], ((gi - 1) >> 1) & 1, p.err)))) {
                    fail = true;  // leaves at the next pair barrier
                    continue;
                }
                if (rescale) {
                    tc_fence_after();
#pragma unroll 1
                    for (int cc = 0; cc < 4; ++cc) {
                        float o[32];
                        const uint32_t ta = lane_base + kTmemO + half * 128 + cc * 32;
                        tmem_ld32(ta, o);
                        tc_wait_ld();
#pragma unroll
                        for (int k = 0; k < 32; k += 2) {
                            const float2 r = fmul2(make_float2(o[k], o[k + 1]), make_float2(alpha, alpha));
                            o[k] = r.x;
                            o[k + 1] = r.y;
                        }
                        tmem_st32(ta, o);
                    }
                }
                float2 r2[2] = {make_float2(0.f, 0.f), make_float2(0.f, 0.f)};
                // a row with no valid key so far (m_new = -inf) gets P = 0: with the
                // subtracted reference at -inf every exponent is -inf, so no
                // per-element select is needed
                const float nm = m_new == -INFINITY ? -INFINITY : -m_new;
                const float2 sc2 = make_float2(kScaleLog2, kScaleLog2), nm2 = make_float2(nm, nm);
                // two chunks of 32 keys, each handed to the PV MMAs as soon
                // as it is in TMEM (the O rescale above is ordered before it)
#pragma unroll
                for (int c = 0; c < 2; ++c) {
                    uint32_t pk[16];
#pragma unroll
                    for (int k = 0; k < 16; ++k) {
                        const float2 a = ffma2(c ? make_float2(xb[2 * k], xb[2 * k + 1])
                                                   : make_float2(xa[2 * k], xa[2 * k + 1]),
                                                 sc2, nm2);
                        const float e0 = ex2_approx(a.x);
                        const float e1 = ex2_approx(a.y);
                        r2[k & 1] = fadd2(r2[k & 1], make_float2(e0, e1));
                        pk[k] = pack_f16x2(e0, e1);
                    }
                    tmem_st16(pbuf + half * 32 + c * 16, pk);
                    tc_wait_st();
                    tc_fence_before();
                    mbar_arrive(&p_full[2 * b + c]);
                }
                l = l * alpha + ((r2[0].x + r2[1].x) + (r2[0].y + r2[1].y));
                m = m_new;
            }
            if (!ok) break;
            // ---- hand the unit to the epilogue warps: this half's row sum.
            // Stay at most one unit ahead of the epilogue: its barriers count
            // phases by parity, and it reads the sums before releasing O.
            if (fail || (ukc >= 1 && !__all_sync(0xffffffffu, mbar_wait(o_free, (ukc - 1) & 1, p.err)))) {
                fail = true;  // leaves at the next unit's first pair barrier
                continue;
            }
            reds[half * 128 + row] = l;  // read by the epilogue before it releases O
            if (half == 0) redmx[row] = m;
            mbar_arrive(fin_bar);
        }
        if (fail) ok = false;
        if (!ok) *s_abort = 1;
    }
    tc_fence_before();
    __syncthreads();
    if (warp == kPfWarpMma) {
        tc_fence_after();
        tmem_dealloc(tmem, kTmemCols);
    }
}

// ------------------------------------------------------------------------
// Self-test of the bounded-wait path: one thread waits on an mbarrier that
// nothing ever arrives on.  The wait gives up after kWaitLimitNs, sets
// kErrWaitTimeout in *err and the kernel returns normally.
// ------------------------------------------------------------------------
__global__ void wait_timeout_probe(unsigned *err) {
    __shared__ uint64_t never;
    if (threadIdx.x == 0) {
        mbar_init(&never, 1);
        fence_mbar_init();
        mbar_wait(&never, 0, err);
    }
}

// ------------------------------------------------------------------------
// Utility kernels: seeded N(0,1) fill, host-layout import/export.
// ------------------------------------------------------------------------
__device__ __forceinline__ uint64_t splitmix64(uint64_t x) {
    x += 0x9E3779B97F4A7C15ull;
    x = (x ^ (x >> 30)) * 0xBF58476D1CE4E5B9ull;
    x = (x ^ (x >> 27)) * 0x94D049BB133111EBull;
    return x ^ (x >> 31);
}

template <typename KVT>
__global__ void fill_normal(KVT *dst, size_t n, uint64_t seed) {
    for (size_t i = (size_t)blockIdx.x * blockDim.x + threadIdx.x; i < n / 2; i += (size_t)gridDim.x * blockDim.x) {
        const uint64_t r = splitmix64(seed ^ (i * 0xD1B54A32D192ED03ull));
        const float u1 = ((uint32_t)(r >> 40) + 0.5f) * (1.0f / 16777216.0f);
        const float u2 = ((uint32_t)(r & 0xFFFFFF)) * (1.0f / 16777216.0f);
        const float rad = sqrtf(-2.0f * logf(u1));
        float sn, cs;
        sincospif(2.0f * u2, &sn, &cs);
        dst[2 * i] = KvType<KVT>::from_f(rad * cs);
        dst[2 * i + 1] = KvType<KVT>::from_f(rad * sn);
    }
}

// host-layout [rows][4][256] fp32  <->  device planes [4][rows][256]
template <typename KVT>
__global__ void import_rows(const float *__restrict__ src, KVT *__restrict__ dst_plane0, size_t plane_stride, int rows) {
    const size_t n = (size_t)rows * kKvHeads * kHeadDim;
    for (size_t i = (size_t)blockIdx.x * blockDim.x + threadIdx.x; i < n; i += (size_t)gridDim.x * blockDim.x) {
        const int d = i % kHeadDim;
        const int h = (i / kHeadDim) % kKvHeads;
        const size_t r = i / (kHeadDim * kKvHeads);
        dst_plane0[h * plane_stride + r * kHeadDim + d] = KvType<KVT>::from_f(src[i]);
    }
}
template <typename KVT>
__global__ void export_rows(const KVT *__restrict__ src_plane0, size_t plane_stride, int rows, float *__restrict__ dst) {
    const size_t n = (size_t)rows * kKvHeads * kHeadDim;
    for (size_t i = (size_t)blockIdx.x * blockDim.x + threadIdx.x; i < n; i += (size_t)gridDim.x * blockDim.x) {
        const int d = i % kHeadDim;
        const int h = (i / kHeadDim) % kKvHeads;
        const size_t r = i / (kHeadDim * kKvHeads);
        dst[i] = KvType<KVT>::to_f(src_plane0[h * plane_stride + r * kHeadDim + d]);
    }
}

}  // namespace g3

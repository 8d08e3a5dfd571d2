// proj_kernels.cuh - BF16 Q/K/V and O projections of the attention layer on
// the tensor cores (sm_100a).  Every kernel here is launched with
// programmatic dependent launch: it begins while the previous kernel of the
// stream drains and calls griddepcontrol.wait before touching memory.
//
// The reference computes every projection as y = W x with W stored BF16
// [out][in] row-major and x fp32 (gemma3_matvec_bf16, gemma3_kernels.c:195-225,
// called from layer_attention, gemma3_transformer.c:290-292 and :355; the
// batched prefill converts W to fp32 and runs cblas_sgemm(NoTrans, Trans),
// gemma3_transformer.c:614-639 and :694-699).  Here W is held as fp16 (the
// BF16 values convert exactly for |w| >= 2^-14; smaller ones keep an absolute
// error below 2^-24) and x is rounded once to fp16, whose 11-bit significand
// keeps a whole layer (two projections around the attention) within 1e-2 of
// the fp32 reference; BF16 activations (8 bits) did not.  A value outside the
// fp16 range raises a status bit instead of saturating.  The products
// accumulate in fp32 in TMEM.
//
// proj_gemm_sm100 computes the transposed product Y^T = W . X^T, so that the
// output features fill the 128-row M dimension of tcgen05.mma and the
// tokens (a decode batch of 1-256, or a prefill block) form N.  One tile =
// 128 features x NT tokens x a K range; tiles are dealt to persistent CTAs.
// When there are too few tiles to keep every SM streaming weights (decode),
// the K range is split and the partial sums are reduced in order by
// proj_splitk_reduce (deterministic).
//
//   warp 0: TMA producer (W box 128 x 64, X box NT x 64 fp16, 128-byte swizzle)
//   warp 1: TMEM owner and MMA issuer (4 MMAs of K=16 per 64-wide K chunk)
//   warps 2-5: epilogue, thread = output feature (TMEM lane), 32 tokens per
//              tcgen05.ld; each store instruction writes 32 consecutive
//              features of one token (coalesced)
// TMEM: two accumulators of 256 columns, so a tile's epilogue overlaps the
// next tile's MMAs.
#pragma once
#include "sm100_ptx.cuh"

namespace g3 {

constexpr int kProjThreads = 192;
constexpr int kProjStages = 4;
constexpr uint32_t kProjWBytes = 128 * 128;        // 128 rows x 64 fp16
constexpr uint32_t kProjXBytesMax = 256 * 128;     // up to 256 tokens x 64 fp16
constexpr uint32_t kProjStageBytes = kProjWBytes + kProjXBytesMax;
constexpr uint32_t kProjSmem = kProjStages * kProjStageBytes + 256;  // + barriers

// Output routing: feature f in [seg_lo[s], seg_lo[s+1]) goes to
// seg_ptr[s][t * seg_ld[s] + f - seg_lo[s]] (Q / K / V of a fused QKV weight).
struct ProjOut {
    float *ptr[3];
    int lo[4];
    int ld[3];
};

struct ProjParams {
    int T;          // tokens
    int N;          // output features (multiple of 128)
    int kchunks;    // K / 64
    int nt;         // tokens per tile (multiple of 32, <= 256)
    int splits;     // K splits; > 1 writes partials
    int ntile_tok;  // ceil(T / nt)
    ProjOut out;
    float *partial;  // [splits][T][N] when splits > 1
    unsigned *err;
};

__device__ __forceinline__ float *proj_dst(const ProjOut &o, int t, int f) {
    if (f < o.lo[1]) return o.ptr[0] + (size_t)t * o.ld[0] + (f - o.lo[0]);
    if (f < o.lo[2]) return o.ptr[1] + (size_t)t * o.ld[1] + (f - o.lo[1]);
    return o.ptr[2] + (size_t)t * o.ld[2] + (f - o.lo[2]);
}

__global__ void __launch_bounds__(kProjThreads, 1)
    proj_gemm_sm100(const __grid_constant__ CUtensorMap tmW, const __grid_constant__ CUtensorMap tmX,
                    const ProjParams p) {
    extern __shared__ __align__(1024) unsigned char smem_raw[];
    if (smem_u32(smem_raw) & 1023u) {
        if (threadIdx.x == 0) raise_status(p.err, kErrBadIndex);
        return;
    }
    unsigned char *sm = smem_raw;
    uint64_t *bars = reinterpret_cast<uint64_t *>(sm + kProjStages * kProjStageBytes);
    uint64_t *full = bars;                 // [4]
    uint64_t *empty = bars + 4;            // [4]
    uint64_t *acc_full = bars + 8;         // [2]
    uint64_t *acc_empty = bars + 10;       // [2], 128 arrivals
    uint64_t *done = bars + 12;
    uint32_t *tmem_slot = reinterpret_cast<uint32_t *>(bars + 13);
    volatile int *s_abort = reinterpret_cast<volatile int *>(bars + 14);

    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const int mtiles = p.N / 128;
    const int ntiles = mtiles * p.ntile_tok * p.splits;
    const int kper = (p.kchunks + p.splits - 1) / p.splits;
    const uint32_t xbytes = (uint32_t)p.nt * 128;

    if (threadIdx.x == 0) {
        for (int i = 0; i < 10; ++i) mbar_init(&bars[i], 1);
        mbar_init(&acc_empty[0], 128);
        mbar_init(&acc_empty[1], 128);
        mbar_init(done, 1);
        *s_abort = 0;
        fence_mbar_init();
    }
    if (warp == 1) tmem_alloc(tmem_slot, 512);
    tc_fence_before();
    __syncthreads();
    tc_fence_after();
    const uint32_t tmem = *tmem_slot;
    pdl_launch_dependents();

    // tile index -> (feature tile, token tile, K split)
    auto tile_of = [&](int idx, int &m, int &n, int &s) {
        s = idx % p.splits;
        const int r = idx / p.splits;
        m = r % mtiles;
        n = r / mtiles;
    };
    auto k_range = [&](int s, int &k0, int &k1) {
        k0 = s * kper;
        k1 = min(p.kchunks, k0 + kper);
    };
    // The weights do not depend on the previous kernel of the stream: warm L2
    // with this CTA's first weight tiles while that kernel drains, then wait
    // for it (programmatic dependent launch) before touching anything else.
    if (warp == 0 && lane == 0 && blockIdx.x < ntiles) {
        prefetch_tmap(&tmW);
        int m, n, s, k0, k1;
        tile_of(blockIdx.x, m, n, s);
        k_range(s, k0, k1);
        for (int kc = k0; kc < min(k1, k0 + 2 * kProjStages); ++kc) tma_prefetch_2d(&tmW, kc * 64, m * 128);
    }
    pdl_wait();

    if (warp == 0) {
        // ---------------------------------------------------- TMA producer
        if (lane == 0) {
            prefetch_tmap(&tmW);
            prefetch_tmap(&tmX);
            int it = 0;
            bool ok = true;
            for (int idx = blockIdx.x; ok && idx < ntiles; idx += gridDim.x) {
                int m, n, s, k0, k1;
                tile_of(idx, m, n, s);
                k_range(s, k0, k1);
                for (int kc = k0; kc < k1; ++kc, ++it) {
                    const int st = it % kProjStages, u = it / kProjStages;
                    if (*s_abort || (u >= 1 && !mbar_wait(&empty[st], (u - 1) & 1, p.err))) { ok = false; break; }
                    unsigned char *sb = sm + st * kProjStageBytes;
                    mbar_expect_tx(&full[st], kProjWBytes + xbytes);
                    tma_load_2d(sb, &tmW, kc * 64, m * 128, &full[st]);
                    tma_load_2d(sb + kProjWBytes, &tmX, kc * 64, n * p.nt, &full[st]);
                }
            }
            if (!ok) {
                *s_abort = 1;
                // let the copies in flight land before the shared memory goes
                for (int j = max(0, it - kProjStages); j < it; ++j)
                    mbar_wait(&full[j % kProjStages], (j / kProjStages) & 1, nullptr);
            }
        }
    } else if (warp == 1) {
        // ---------------------------------------------------- MMA issuer
        if (lane == 0) {
            const uint32_t idesc = idesc_f16_f32(128, p.nt, 0, 0);
            int it = 0, tl = 0;
            bool ok = true;
            for (int idx = blockIdx.x; ok && idx < ntiles; idx += gridDim.x, ++tl) {
                int m, n, s, k0, k1;
                tile_of(idx, m, n, s);
                k_range(s, k0, k1);
                const int b = tl & 1;
                // the epilogue has drained this accumulator (tile tl-2)
                if (tl >= 2 && !mbar_wait(&acc_empty[b], ((tl - 2) >> 1) & 1, p.err)) { ok = false; break; }
                tc_fence_after();
                for (int kc = k0; kc < k1; ++kc, ++it) {
                    const int st = it % kProjStages;
                    if (*s_abort || !mbar_wait(&full[st], (it / kProjStages) & 1, p.err)) { ok = false; break; }
                    tc_fence_after();
                    const uint32_t sa = smem_u32(sm + st * kProjStageBytes);
                    const uint64_t dA = smem_desc_sw128(sa, 16, 1024);
                    const uint64_t dB = smem_desc_sw128(sa + kProjWBytes, 16, 1024);
#pragma unroll
                    for (int kk = 0; kk < 4; ++kk)
                        tc_mma_f16(tmem + b * 256, dA + (uint64_t)((kk * 32) >> 4), dB + (uint64_t)((kk * 32) >> 4),
                                   idesc, (kc > k0 || kk > 0) ? 1u : 0u);
                    tc_commit(&empty[st]);
                }
                if (!ok) break;
                tc_commit(&acc_full[b]);
            }
            if (!ok) *s_abort = 1;
            tc_commit(done);
            mbar_wait(done, 0, nullptr);
        }
    } else {
        // ---------------------------------------------------- epilogue (warps 2-5)
        const int quad = warp & 3;
        const int row = quad * 32 + lane;  // feature within the tile
        const uint32_t lane_base = tmem + ((uint32_t)(quad * 32) << 16);
        int tl = 0;
        bool ok = true;
        for (int idx = blockIdx.x; ok && idx < ntiles; idx += gridDim.x, ++tl) {
            int m, n, s;
            tile_of(idx, m, n, s);
            const int b = tl & 1;
            if (!__all_sync(0xffffffffu, !*s_abort && mbar_wait(&acc_full[b], (tl >> 1) & 1, p.err))) {
                ok = false;
                break;
            }
            tc_fence_after();
            // destination of this tile (a 128-feature tile never straddles the
            // Q / K / V segments): column f of a row-major [T][ld] array
            const int f0 = m * 128;
            float *base;
            int ld;
            if (p.splits > 1) {
                base = p.partial + (size_t)s * p.T * p.N + f0;
                ld = p.N;
            } else if (f0 < p.out.lo[1]) {
                base = p.out.ptr[0] + (f0 - p.out.lo[0]);
                ld = p.out.ld[0];
            } else if (f0 < p.out.lo[2]) {
                base = p.out.ptr[1] + (f0 - p.out.lo[1]);
                ld = p.out.ld[1];
            } else {
                base = p.out.ptr[2] + (f0 - p.out.lo[2]);
                ld = p.out.ld[2];
            }
            float *col = base + row;
            const int t0 = n * p.nt;
            for (int c = 0; c < p.nt / 32; ++c) {
                float v[32];
                tmem_ld32(lane_base + b * 256 + c * 32, v);
                tc_wait_ld();
                const int tc = t0 + c * 32;
#pragma unroll
                for (int j = 0; j < 32; ++j)
                    if (tc + j < p.T) col[(size_t)(tc + j) * ld] = v[j];
            }
            tc_fence_before();
            mbar_arrive(&acc_empty[b]);
        }
        if (!ok) *s_abort = 1;
    }
    tc_fence_before();
    __syncthreads();
    if (warp == 1) {
        tc_fence_after();
        tmem_dealloc(tmem, 512);
    }
}

// out[t][f] = sum over s (in order) of partial[s][t][f], routed as ProjOut.
__global__ void __launch_bounds__(256) proj_splitk_reduce(const float *__restrict__ partial, int splits, int T, int N,
                                                          const ProjOut out) {
    pdl_launch_dependents();
    pdl_wait();
    const size_t n = (size_t)T * N;
    for (size_t i = (size_t)blockIdx.x * blockDim.x + threadIdx.x; i < n; i += (size_t)gridDim.x * blockDim.x) {
        float acc = partial[i];
        for (int s = 1; s < splits; ++s) acc += partial[(size_t)s * n + i];
        *proj_dst(out, (int)(i / N), (int)(i % N)) = acc;
    }
}

// fp32 rows -> fp16 (round to nearest even), 4 elements per thread step; a
// value outside the fp16 range sets kErrRange.
__global__ void __launch_bounds__(256) to_f16_rows(const float *__restrict__ x, __half *__restrict__ y, size_t n4,
                                                   unsigned *err) {
    pdl_launch_dependents();
    pdl_wait();
    for (size_t i = (size_t)blockIdx.x * blockDim.x + threadIdx.x; i < n4; i += (size_t)gridDim.x * blockDim.x) {
        const float4 v = reinterpret_cast<const float4 *>(x)[i];
        const float m = fmaxf(fmaxf(fabsf(v.x), fabsf(v.y)), fmaxf(fabsf(v.z), fabsf(v.w)));
        if (!(m <= 65504.f)) raise_status(err, kErrRange);
        uint2 o;
        o.x = pack_f16x2(v.x, v.y);
        o.y = pack_f16x2(v.z, v.w);
        reinterpret_cast<uint2 *>(y)[i] = o;
    }
}

// BF16 weights (as the reference stores them) -> fp16: exact for |w| >= 2^-14,
// subnormal below (absolute error < 2^-24); a weight beyond the fp16 range
// sets kErrRange.
__global__ void __launch_bounds__(256) bf16_to_f16(const uint16_t *__restrict__ src, __half *__restrict__ dst, size_t n,
                                                   unsigned *err) {
    for (size_t i = (size_t)blockIdx.x * blockDim.x + threadIdx.x; i < n; i += (size_t)gridDim.x * blockDim.x) {
        const float f = __uint_as_float((uint32_t)src[i] << 16);
        if (!(fabsf(f) <= 65504.f)) raise_status(err, kErrRange);
        dst[i] = __float2half_rn(f);
    }
}

}  // namespace g3

// decode_tc.cuh - GQA decode over a BF16 cache on the 5th-generation tensor
// core (gemma3_kernels.c:527-597 for one (sequence, kv head, key range)).
//
// The split-KV decode on CUDA cores spends ~80 instructions per cache row
// (shared loads, bf16 unpacking, dot products, 32-lane shuffle reductions,
// the P.V update) and on a BF16 cache that work, not HBM, sets its rate.
// Here the two contractions go to tcgen05.mma instead, with the cache tiles
// as they are streamed in:
//
//   S^T [128 keys x 16]  = K tile [128 keys x 256] . Qs^T      (M = keys)
//   O^T [256 dims x 16]  = V tile^T [256 x 128 keys] . P^T     (M = dims, two
//                                                               halves of 128)
//
// Qs holds the two query heads of the group, each split into a BF16 high
// part and the BF16 rounding of the remainder (q = hi + lo exactly to ~2^-17
// relative): rows 0,1 = head 2g hi/lo, rows 2,3 = head 2g+1 hi/lo, rows 4-15
// zero.  The cache rows are BF16 already, so S = S_hi + S_lo is the fp32 dot
// product of the BF16 row with q to ~2^-17, and P is split the same way
// before the P.V product.  Accumulation is fp32 throughout; the result
// matches the CUDA-core kernel's precision, not BF16's.
//
// CTA = (split, kv head, sequence) as in decode_splitkv, 192 threads:
//   warps 0-3  thread t = key t of the tile (TMEM lane of S^T) for the
//              online softmax, and dims t / t+128 (TMEM lanes of the two O^T
//              halves) for the running output; the fused q/k/v prologue;
//   warp 4     TMA producer: the K and V tiles of 128 rows, each as four
//              16 KB chunks [128 rows][64 dims] (128-byte swizzle) through a
//              six-chunk ring;
//   warp 5     TMEM owner and MMA issuer (one thread).
// Per tile: S MMAs (16) -> softmax (max over the CTA's 128 threads, P^T hi/lo
// into shared memory) -> P.V MMAs (16, into a fresh O^T) -> the 128 threads
// fold O^T into their registers with the running rescale.  Two CTAs share an
// SM, so one CTA's softmax overlaps the other's MMAs and copies.
//
// TMEM (128 columns): S^T cols 0-15, O^T dims 0-127 cols 32-47, dims 128-255
// cols 48-63.  Every wait is bounded (mbar_wait); a failed wait stops the
// CTA cleanly (copies drained, MMAs completed, TMEM freed) and sets the
// context status word.
#pragma once
#include "attn_kernels.cuh"

namespace g3 {

constexpr int kTcTK = 128;                    // cache rows per tile
constexpr uint32_t kTcChunk = 128 * 128;      // [128 rows][64 dims] bf16
constexpr int kTcSlots = 6;                   // ring of 16 KB chunks
// Shared memory: the ring, then
//   Qs  [4 dim-chunks][16 rows][128 B]   8 KB
//   P^T [2 key-chunks][16 rows][128 B]   4 KB
//   q heads fp32 [2][256] (fused prologue) 2 KB
//   mbarriers, reductions, flags           512 B
// = 113,152 B: two CTAs per SM, so one CTA's softmax and copies overlap the
// other's MMAs.  (A one-CTA-per-SM build with a 12-chunk ring and double-
// buffered S^T / O^T / P^T, overlapping a CTA's own tiles, measured no
// faster at any batch: a lone CTA streamed ~45 GB/s either way.)
constexpr uint32_t kTcOffQ = kTcSlots * kTcChunk;
constexpr uint32_t kTcOffP = kTcOffQ + 8192;
constexpr uint32_t kTcOffQf = kTcOffP + 4096;
constexpr uint32_t kTcOffBar = kTcOffQf + 2048;
constexpr uint32_t kTcSmem = kTcOffBar + 512;
constexpr int kTcThreads = 192;
constexpr uint32_t kTcTmemCols = 128;
constexpr uint32_t kTcTmemS = 0;
constexpr uint32_t kTcTmemO = 32;

// Instruction descriptor, kind::f16 with BF16 A/B (format 1 in bits 7-9 and
// 10-12), fp32 D; a_mn / b_mn select MN-major operands.
__host__ __device__ constexpr uint32_t idesc_bf16_f32(int M, int N, int a_mn, int b_mn) {
    return idesc_f16_f32(M, N, a_mn, b_mn) | (1u << 7) | (1u << 10);
}

// Byte offset of element (row r, column c) in a K-major BF16 tile of
// `rows_per_chunk` rows stored as 64-column chunks [rows][128 B] with the
// 128-byte swizzle (16-byte unit u of a row at u ^ (r & 7)).
__device__ __forceinline__ uint32_t sw128_off(int r, int c, int rows_per_chunk) {
    return (uint32_t)((c >> 6) * rows_per_chunk * 128 + r * 128 + ((((c & 63) >> 3) ^ (r & 7)) << 4) + (c & 7) * 2);
}

__device__ __forceinline__ void tmem_ld4(uint32_t taddr, float (&v)[4]) {
    uint32_t r[4];
    asm volatile("tcgen05.ld.sync.aligned.32x32b.x4.b32 {%0,%1,%2,%3}, [%4];"
                 : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3])
                 : "r"(taddr));
#pragma unroll
    for (int i = 0; i < 4; ++i) v[i] = __uint_as_float(r[i]);
}

// Barrier over the four compute warps only (named barrier 1).
__device__ __forceinline__ void tc_compute_sync() { asm volatile("bar.sync 1, 128;" ::: "memory"); }

__device__ __forceinline__ void fence_proxy_async_global() {
    asm volatile("fence.proxy.async.global;" ::: "memory");
}

__device__ __forceinline__ uint16_t bf16_bits(float x) {
    return __bfloat16_as_ushort(__float2bfloat16_rn(x));
}

// Log-sum-exp merge of n partials [m, l, O[256]] of the two heads of group
// g by 128 threads: thread t writes dims t and t + 128 of both heads.  One
// online pass over the partials (read through L2: other CTAs wrote them),
// 16 partials (48 loads) in flight per thread and head.
__device__ __forceinline__ void tc_merge_group(const float *base, size_t hstride, int n, float *out_g) {
    constexpr int C = 16;
    const int t = threadIdx.x;
#pragma unroll 1
    for (int hh = 0; hh < 2; ++hh) {
        const float *bh = base + hh * hstride;
        float Mx = -INFINITY, Lt = 0.f, At = 0.f, Bt = 0.f;
#pragma unroll 1
        for (int i0 = 0; i0 < n; i0 += C) {
            float2 ml[C];
            float oa[C], ob[C];
#pragma unroll
            for (int j = 0; j < C; ++j) {
                if (i0 + j < n) {
                    const float *pp = bh + (size_t)(i0 + j) * (kHeadDim + 2);
                    ml[j] = __ldcg(reinterpret_cast<const float2 *>(pp));
                    oa[j] = __ldcg(pp + 2 + t);
                    ob[j] = __ldcg(pp + 2 + 128 + t);
                } else {
                    ml[j] = make_float2(-INFINITY, 0.f);
                    oa[j] = ob[j] = 0.f;
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
                At += oa[j] * f;
                Bt += ob[j] * f;
            }
            Mx = cm;
        }
        const float inv = Lt > 0.f ? 1.0f / Lt : 0.f;
        out_g[hh * kHeadDim + t] = At * inv;
        out_g[hh * kHeadDim + 128 + t] = Bt * inv;
    }
}

template <bool kFused, typename Rows = DecodeRows>
__global__ void __launch_bounds__(kTcThreads, 2)
    decode_tc(const __grid_constant__ CUtensorMap tmKV, const DecodeParams p, const __grid_constant__ Rows rows) {
    // All shared state lives in the dynamic buffer (no static shared
    // memory), whose base is then 1024-byte aligned as the swizzled tiles
    // need; checked, since the two-CTAs-per-SM budget leaves no room to
    // realign.
    extern __shared__ __align__(1024) unsigned char sm[];
    if (smem_u32(sm) & 1023u) {
        if (threadIdx.x == 0) raise_status(p.err, kErrBadIndex);
        return;
    }
    unsigned char *ring = sm;
    unsigned char *sQ = sm + kTcOffQ;
    unsigned char *sP = sm + kTcOffP;
    float(*qf)[kHeadDim] = reinterpret_cast<float(*)[kHeadDim]>(sm + kTcOffQf);
    uint64_t *bars = reinterpret_cast<uint64_t *>(sm + kTcOffBar);
    uint64_t *full = bars, *empty = bars + kTcSlots;  // [kTcSlots] each
    uint64_t &q_ready = bars[12], &s_full = bars[13], &p_full = bars[14], &o_full = bars[15], &o_free = bars[16],
             &row_ready = bars[17], &mma_done = bars[18];
    uint32_t &tmem_slot = *reinterpret_cast<uint32_t *>(bars + 19);
    volatile int &s_abort = *reinterpret_cast<volatile int *>(bars + 20);
    volatile int &s_flag = *reinterpret_cast<volatile int *>(bars + 21);  // compute warps: any failed / last split
    float(*red)[4][2] = reinterpret_cast<float(*)[4][2]>(bars + 22);     // [2][4][2] floats = 64 B
    float(*lred)[2] = reinterpret_cast<float(*)[2]>(bars + 30);          // [4][2] = 32 B
    static_assert((kTcSlots % 2) == 0, "V chunk pairs must not wrap the ring");

    const int split = blockIdx.x, g = blockIdx.y, b = blockIdx.z;
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const int seq = rows.seq[b];
    const int n = rows.nrows[b];
    const int r0 = split * p.chunk;
    const int r1 = min(n, r0 + p.chunk);
    const int ntiles = r1 > r0 ? (r1 - r0 + kTcTK - 1) / kTcTK : 0;
    const int plane_k = (seq * 2 + 0) * kKvHeads + g;
    const int plane_v = (seq * 2 + 1) * kKvHeads + g;
    const int slot = kFused ? cache_row(p.L, rows.pos[b]) : -1;  // cache row of the new token
    const bool owner = kFused && slot >= r0 && slot < r1;
    const int own_tile = owner ? (slot - r0) / kTcTK : -1;

    pdl_launch_dependents();
    if (threadIdx.x == 0) {
        for (int s = 0; s < kTcSlots; ++s) {
            mbar_init(&full[s], 1);
            mbar_init(&empty[s], 1);
        }
        mbar_init(&q_ready, 128);
        mbar_init(&s_full, 1);
        mbar_init(&p_full, 128);
        mbar_init(&o_full, 1);
        mbar_init(&o_free, 128);
        mbar_init(&row_ready, 64);
        mbar_init(&mma_done, 1);
        s_abort = 0;
        fence_mbar_init();
    }
    if (warp == 5) tmem_alloc(&tmem_slot, kTcTmemCols);
    tc_fence_before();
    __syncthreads();
    tc_fence_after();
    const uint32_t tmem = tmem_slot;
    pdl_wait();

    if (warp == 4) {
        // ------------------------------------------------ TMA producer
        if (lane == 0 && ntiles > 0) {
            prefetch_tmap(&tmKV);
            const int nq = 8 * ntiles;
            int q = 0;
            for (; q < nq; ++q) {
                const int s = q % kTcSlots, i = q >> 3, c = q & 7;
                if (s_abort) break;
                if (q >= kTcSlots && !mbar_wait(&empty[s], ((q / kTcSlots) - 1) & 1, p.err)) {
                    s_abort = 1;
                    break;
                }
                // the tile holding the new token's row is read only after the
                // prologue has written that row to the cache
                if (kFused && i == own_tile && c == 0 && !mbar_wait(&row_ready, 0, p.err)) {
                    s_abort = 1;
                    break;
                }
                mbar_expect_tx(&full[s], kTcChunk);
                tma_load_4d(ring + s * kTcChunk, &tmKV, 0, r0 + i * kTcTK, c & 3, c < 4 ? plane_k : plane_v,
                            &full[s]);
            }
            // every issued copy has landed before the CTA can exit
            for (int d = max(0, q - kTcSlots); d < q; ++d)
                mbar_wait(&full[d % kTcSlots], (d / kTcSlots) & 1, nullptr);
        }
    } else if (warp == 5) {
        // ------------------------------------------------ MMA issuer
        if (lane == 0 && ntiles > 0) {
            constexpr uint32_t idS = idesc_bf16_f32(128, 16, 0, 0);
            constexpr uint32_t idO = idesc_bf16_f32(128, 16, 1, 0);
            const uint64_t dRing = smem_desc_sw128(smem_u32(ring), 16, 1024);
            const uint64_t dRingMN = smem_desc_sw128(smem_u32(ring), kTcChunk, 1024);
            const uint64_t dQ = smem_desc_sw128(smem_u32(sQ), 16, 1024);
            const uint64_t dP = smem_desc_sw128(smem_u32(sP), 16, 1024);
            bool ok = mbar_wait(&q_ready, 0, p.err);
            // S^T(i) = K(i) . Qs^T, the K tile's four dim-chunks as they land
            auto issue_s = [&](int i) {
                for (int c = 0; c < 4; ++c) {
                    const int q = 8 * i + c, s = q % kTcSlots;
                    if (s_abort || !mbar_wait(&full[s], (q / kTcSlots) & 1, p.err)) return false;
                    tc_fence_after();
#pragma unroll
                    for (int kk = 0; kk < 4; ++kk)
                        tc_mma_f16(tmem + kTcTmemS, dRing + (uint64_t)((s * kTcChunk + kk * 32) >> 4),
                                   dQ + (uint64_t)((c * 2048 + kk * 32) >> 4), idS, (c | kk) ? 1u : 0u);
                    tc_commit(&empty[s]);
                }
                tc_commit(&s_full);
                return true;
            };
            if (ok && ntiles > 0) ok = issue_s(0);
            for (int i = 0; ok && i < ntiles; ++i) {
                // O^T(i) = V(i)^T . P^T(i) once the softmax has written P(i) and
                // the compute warps have read the previous O^T
                if (!mbar_wait(&p_full, i & 1, p.err) || (i >= 1 && !mbar_wait(&o_free, (i - 1) & 1, p.err))) {
                    ok = false;
                    break;
                }
                for (int h = 0; h < 2 && ok; ++h) {
                    const int q0 = 8 * i + 4 + 2 * h, s0 = q0 % kTcSlots;  // s0 even: s0, s0 + 1 adjacent
                    if (s_abort || !mbar_wait(&full[s0], (q0 / kTcSlots) & 1, p.err) ||
                        !mbar_wait(&full[s0 + 1], ((q0 + 1) / kTcSlots) & 1, p.err)) {
                        ok = false;
                        break;
                    }
                    tc_fence_after();
#pragma unroll
                    for (int kk = 0; kk < 8; ++kk)
                        tc_mma_f16(tmem + kTcTmemO + 16 * h, dRingMN + (uint64_t)((s0 * kTcChunk + kk * 2048) >> 4),
                                   dP + (uint64_t)(((kk >> 2) * 2048 + (kk & 3) * 32) >> 4), idO, kk ? 1u : 0u);
                    tc_commit(&empty[s0]);
                    tc_commit(&empty[s0 + 1]);
                }
                if (!ok) break;
                tc_commit(&o_full);
                // the next tile's S overwrites the S^T the softmax has read
                // (P(i) is written only after that read)
                if (i + 1 < ntiles && !(ok = issue_s(i + 1))) break;
            }
            if (!ok) s_abort = 1;
            // drain: every MMA this thread issued has completed
            tc_commit(&mma_done);
            mbar_wait(&mma_done, 0, nullptr);
        }
    } else {
        // ------------------------------------------------ compute warps 0-3
        const int t = threadIdx.x;  // 0..127
        // Fused prologue (gemma3_transformer.c:294-316): warps 0-1 normalise
        // + rotate the group's two query heads; in the CTA holding the new
        // token's cache row, warps 2-3 build that k / v row and append it.
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
                store4<float>(&qf[warp][4 * lane], r.a);
                store4<float>(&qf[warp][128 + 4 * lane], r.b);
            } else if (owner) {
                const int sel = warp - 2;
                load_head_row((sel ? p.vraw : p.kraw) + ((size_t)b * kKvHeads + g) * kHeadDim, lane, r);
                if (!sel) norm_rope_row(r, kn, p.eps, rope_row, lane);
                __nv_bfloat16 *dst = plane<__nv_bfloat16>(p.L, seq, sel, g) + (size_t)slot * kHeadDim;
                store4<__nv_bfloat16>(dst + 4 * lane, r.a);
                store4<__nv_bfloat16>(dst + 128 + 4 * lane, r.b);
                // the row is read back by the TMA (async proxy) of this CTA
                fence_proxy_async_global();
                mbar_arrive(&row_ready);
            }
            tc_compute_sync();
        }
        // Qs rows: 2hh = hi, 2hh + 1 = lo of head 2g + hh; rows 4-15 zero.
        {
            const float *q0 = kFused ? qf[0] : p.q + ((size_t)b * kHeads + 2 * g) * kHeadDim;
#pragma unroll
            for (int hh = 0; hh < 2; ++hh) {
#pragma unroll
                for (int j = 0; j < 2; ++j) {
                    const int d = 2 * t + j;
                    const float x = q0[hh * kHeadDim + d];
                    const uint16_t hi = bf16_bits(x);
                    const uint16_t lo = bf16_bits(x - __uint_as_float((uint32_t)hi << 16));
                    *reinterpret_cast<uint16_t *>(sQ + sw128_off(2 * hh, d, 16)) = hi;
                    *reinterpret_cast<uint16_t *>(sQ + sw128_off(2 * hh + 1, d, 16)) = lo;
                }
            }
            // zero rows 4-15 of Qs and P^T (the MMAs read all 16 rows)
            for (int e = t; e < 12 * 32; e += 128) {  // 12 rows x 32 16-byte units
                const int r = 4 + e / 32, u = e % 32;
                *reinterpret_cast<uint4 *>(sQ + (u >> 3) * 2048 + r * 128 + ((u & 7) << 4)) = make_uint4(0, 0, 0, 0);
            }
            for (int e = t; e < 12 * 16; e += 128) {  // 12 rows x 16 units
                const int r = 4 + e / 16, u = e % 16;
                *reinterpret_cast<uint4 *>(sP + (u >> 3) * 2048 + r * 128 + ((u & 7) << 4)) = make_uint4(0, 0, 0, 0);
            }
            fence_proxy_async_smem();
            mbar_arrive(&q_ready);
        }

        const uint32_t lane_base = tmem + ((uint32_t)(warp * 32) << 16);
        float m0 = -INFINITY, m1 = -INFINITY;  // running maxima (log2 domain)
        float l0 = 0.f, l1 = 0.f;              // this thread's share of the sums
        float a00 = 0.f, a01 = 0.f, a10 = 0.f, a11 = 0.f;  // O[head][dim t / t+128]
        // Every compute thread runs the same sequence of named barriers
        // whatever happens: after a failed wait a warp keeps iterating with
        // its waits and TMEM reads skipped (ok = false), so no barrier is
        // ever left one warp short.
        // Tile i: S^T(i) -> P(i) -> (tensor core: O^T(i)) -> O^T(i) folded in,
        // which releases the O^T accumulator for the next tile's P.V.
        bool ok = true;
        for (int i = 0; i < ntiles; ++i) {
            ok = __all_sync(0xffffffffu, ok && !s_abort && mbar_wait(&s_full, i & 1, p.err));
            float c[4] = {0.f, 0.f, 0.f, 0.f};
            if (ok) {
                tc_fence_after();
                tmem_ld4(lane_base + kTcTmemS, c);
                tc_wait_ld();
            }
            const bool valid = r0 + i * kTcTK + t < r1;
            const float s0 = valid ? c[0] + c[1] : -INFINITY;
            const float s1 = valid ? c[2] + c[3] : -INFINITY;
            float w0 = s0, w1 = s1;
#pragma unroll
            for (int o = 16; o > 0; o >>= 1) {
                w0 = fmaxf(w0, __shfl_xor_sync(0xffffffffu, w0, o));
                w1 = fmaxf(w1, __shfl_xor_sync(0xffffffffu, w1, o));
            }
            if (lane == 0) {
                red[i & 1][warp][0] = w0;
                red[i & 1][warp][1] = w1;
            }
            tc_compute_sync();
            const float M0 = fmaxf(fmaxf(red[i & 1][0][0], red[i & 1][1][0]), fmaxf(red[i & 1][2][0], red[i & 1][3][0]));
            const float M1 = fmaxf(fmaxf(red[i & 1][0][1], red[i & 1][1][1]), fmaxf(red[i & 1][2][1], red[i & 1][3][1]));
            const float n0 = fmaxf(m0, M0), n1 = fmaxf(m1, M1);  // finite: every tile has a valid row
            const float al0 = ex2_approx(m0 - n0), al1 = ex2_approx(m1 - n1);  // 0 on the first tile
            const float p0 = valid ? ex2_approx(s0 - n0) : 0.f;
            const float p1 = valid ? ex2_approx(s1 - n1) : 0.f;
            l0 = l0 * al0 + p0;
            l1 = l1 * al1 + p1;
            m0 = n0;
            m1 = n1;
            {
                unsigned char *pb = sP;
                const uint16_t h0 = bf16_bits(p0), h1 = bf16_bits(p1);
                const uint16_t e0 = bf16_bits(p0 - __uint_as_float((uint32_t)h0 << 16));
                const uint16_t e1 = bf16_bits(p1 - __uint_as_float((uint32_t)h1 << 16));
                *reinterpret_cast<uint16_t *>(pb + sw128_off(0, t, 16)) = h0;
                *reinterpret_cast<uint16_t *>(pb + sw128_off(1, t, 16)) = e0;
                *reinterpret_cast<uint16_t *>(pb + sw128_off(2, t, 16)) = h1;
                *reinterpret_cast<uint16_t *>(pb + sw128_off(3, t, 16)) = e1;
            }
            fence_proxy_async_smem();
            tc_fence_before();  // S read before the next S MMA overwrites it
            mbar_arrive(&p_full);
            ok = __all_sync(0xffffffffu, ok && !s_abort && mbar_wait(&o_full, i & 1, p.err));
            float o0[4] = {0.f, 0.f, 0.f, 0.f}, o1[4] = {0.f, 0.f, 0.f, 0.f};
            if (ok) {
                tc_fence_after();
                tmem_ld4(lane_base + kTcTmemO, o0);
                tmem_ld4(lane_base + kTcTmemO + 16, o1);
                tc_wait_ld();
                tc_fence_before();
            }
            mbar_arrive(&o_free);
            a00 = a00 * al0 + (o0[0] + o0[1]);
            a10 = a10 * al1 + (o0[2] + o0[3]);
            a01 = a01 * al0 + (o1[0] + o1[1]);
            a11 = a11 * al1 + (o1[2] + o1[3]);
        }
        if (t == 0) s_flag = 0;
        tc_compute_sync();
        if (!ok) {
            s_abort = 1;
            s_flag = 1;
        }
        // sums over the 128 threads
#pragma unroll
        for (int o = 16; o > 0; o >>= 1) {
            l0 += __shfl_xor_sync(0xffffffffu, l0, o);
            l1 += __shfl_xor_sync(0xffffffffu, l1, o);
        }
        if (lane == 0) {
            lred[warp][0] = l0;
            lred[warp][1] = l1;
        }
        tc_compute_sync();
        const float L0 = lred[0][0] + lred[1][0] + lred[2][0] + lred[3][0];
        const float L1 = lred[0][1] + lred[1][1] + lred[2][1] + lred[3][1];
        // one decision for all 128 threads (s_abort may still change under
        // them: it is read once, before the barrier that publishes it)
        const bool good = !s_flag;
        tc_compute_sync();
        if (good) {
            if (p.write_partial) {
                float *d0 = p.partial + (((size_t)b * kHeads + 2 * g) * p.nsplit + split) * (kHeadDim + 2);
                float *d1 = d0 + (size_t)p.nsplit * (kHeadDim + 2);
                if (t == 0) {
                    d0[0] = ntiles ? m0 : -INFINITY;
                    d0[1] = L0;
                    d1[0] = ntiles ? m1 : -INFINITY;
                    d1[1] = L1;
                }
                d0[2 + t] = a00;
                d0[2 + 128 + t] = a01;
                d1[2 + t] = a10;
                d1[2 + 128 + t] = a11;
                if (kFused && p.tickets) {
                    // the last split of this (sequence, kv head) to finish
                    // merges the partials; no CTA waits for another
                    tc_compute_sync();
                    if (t == 0)
                        s_flag = atom_add_acqrel_gpu(&p.tickets[b * kKvHeads + g], 1u) == (unsigned)(p.nsplit - 1);
                    tc_compute_sync();
                    if (s_flag) {
                        tc_merge_group(p.partial + ((size_t)b * kHeads + 2 * g) * p.nsplit * (kHeadDim + 2),
                                       (size_t)p.nsplit * (kHeadDim + 2), p.nsplit,
                                       p.out + (size_t)b * kHeads * kHeadDim + 2 * g * kHeadDim);
                        if (t == 0) p.tickets[b * kKvHeads + g] = 0u;
                    }
                }
            } else {
                const float i0 = L0 > 0.f ? 1.0f / L0 : 0.f, i1 = L1 > 0.f ? 1.0f / L1 : 0.f;
                float *o = p.out + (size_t)b * kHeads * kHeadDim + 2 * g * kHeadDim;
                o[t] = a00 * i0;
                o[128 + t] = a01 * i0;
                o[kHeadDim + t] = a10 * i1;
                o[kHeadDim + 128 + t] = a11 * i1;
            }
        }
    }
    tc_fence_before();
    __syncthreads();
    tc_fence_after();
    if (warp == 5) tmem_dealloc(tmem, kTcTmemCols);
}

}  // namespace g3

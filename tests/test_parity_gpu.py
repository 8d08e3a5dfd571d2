"""Parity of the CUDA path (through the C-ABI) against the reference's own CPU
attention (oracle/_ref, falling back to the C restatement) on seeded inputs.

Tolerance (from the task statement): max |err| <= 1e-2 x RMS(reference
output), fp32 accumulation.  Cache indexing is checked bit-exactly: the V
rows (stored without transformation) of an fp32 cache must equal the
reference's cache row for row, ring slots included.
"""
import numpy as np
import pytest

import gemma3_cuda as gc
import synth
from oracles import best_oracle, bf16_round, exact_attention, rel_err

pytestmark = pytest.mark.gpu
TOL = 1e-2


@pytest.fixture(scope="module")
def oracle():
    return best_oracle()


@pytest.fixture(scope="module")
def ropes(oracle):
    # the integration uploads the host's own tables (gemma3_transformer.c:870-883)
    return oracle.rope_table(8192, 10000.0), oracle.rope_table(8192, 1000000.0)


def make_ctx(ropes, kv_dtype=gc.KV_F32, max_batch=1, max_context=8192, max_prefill=4096):
    ctx = gc.Context(max_context=max_context, max_batch=max_batch, kv_dtype=kv_dtype, max_prefill=max_prefill)
    ctx.upload_rope(ropes[0][:max_context], ropes[1][:max_context])
    return ctx


def qkv(seed, T):
    return (synth.normal(seed, (T, gc.Q_SIZE)), synth.normal(seed + 1, (T, gc.KV_SIZE)),
            synth.normal(seed + 2, (T, gc.KV_SIZE)))


@pytest.mark.parametrize("layer,T,kv", [(0, 200, gc.KV_F32), (5, 300, gc.KV_F32), (0, 200, gc.KV_BF16),
                                        (5, 300, gc.KV_BF16), (1, 1, gc.KV_F32), (11, 65, gc.KV_BF16)])
def test_prefill_from_zero(oracle, ropes, layer, T, kv):
    glob = gc.is_global_layer(layer)
    rope = ropes[1] if glob else ropes[0]
    qn, kn = synth.qk_norm_gains(100 + layer)
    Q, K, V = qkv(7 * layer + T, T)
    c = oracle.new_cache(glob, 8192)
    want = oracle.attn_core_tokens(c, Q, K, V, qn, kn, rope, 0)
    Qn, Kn = oracle.last_qk
    ctx = make_ctx(ropes, kv)
    ctx.set_qk_norm(layer, qn, kn)
    got = ctx.attn_prefill(layer, 0, Q, K, V, 0)
    assert np.isfinite(got).all()
    if kv == gc.KV_F32:
        assert rel_err(got, want) <= TOL, rel_err(got, want)
    # reference semantics on a cache of this dtype, evaluated exactly
    exact = exact_attention(Qn, Kn, V, 0, glob, "bf16" if kv == gc.KV_BF16 else None)
    assert rel_err(got, exact) <= TOL, rel_err(got, exact)
    # cache contents
    kr, vr = oracle.cache_arrays(c)
    kd, vd = ctx.export_cache(layer, 0)
    rows = min(T, kd.shape[0])
    if kv == gc.KV_F32:
        assert np.array_equal(vd[:rows], vr[:rows])
        assert rel_err(kd[:rows], kr[:rows]) < 1e-5
    else:  # a bf16 cache holds the round-to-nearest-even value of each row
        assert np.array_equal(vd[:rows], bf16_round(vr[:rows]))
        # K is recomputed in fp32 on both sides, so the rounding may land one
        # bf16 ulp (<= 2^-7 relative) apart
        assert np.all(np.abs(kd[:rows] - kr[:rows]) <= 2.0 ** -7 * np.abs(kr[:rows]) + 1e-6)
    oracle.free_cache(c)
    ctx.close()


def test_prefill_local_window_wrap(oracle, ropes):
    """T=1500 on a local layer: the window slides past 1024 and the ring wraps."""
    layer, T = 2, 1500
    qn, kn = synth.qk_norm_gains(5)
    Q, K, V = qkv(11, T)
    c = oracle.new_cache(False, 8192)
    want = oracle.attn_core_tokens(c, Q, K, V, qn, kn, ropes[0], 0)
    Qn, Kn = oracle.last_qk
    ctx = make_ctx(ropes)
    ctx.set_qk_norm(layer, qn, kn)
    got = ctx.attn_prefill(layer, 0, Q, K, V, 0)
    assert rel_err(got, want) <= TOL
    # ring slots bit-exact: slot s holds the last position p with p % 1024 == s
    kr, vr = oracle.cache_arrays(c)
    kd, vd = ctx.export_cache(layer, 0)
    assert np.array_equal(vd, vr)
    oracle.free_cache(c)


@pytest.mark.parametrize("layer,kv", [(3, gc.KV_F32), (5, gc.KV_F32), (3, gc.KV_BF16), (17, gc.KV_BF16)])
def test_prefill_chunked(oracle, ropes, layer, kv):
    """Two prefill calls (start_pos > 0) crossing the 1024 window edge."""
    glob = gc.is_global_layer(layer)
    rope = ropes[1] if glob else ropes[0]
    qn, kn = synth.qk_norm_gains(9)
    Q, K, V = qkv(21, 1300)
    c = oracle.new_cache(glob, 8192)
    want = oracle.attn_core_tokens(c, Q, K, V, qn, kn, rope, 0)
    if kv == gc.KV_BF16:
        Qn, Kn = oracle.last_qk
        want = exact_attention(Qn, Kn, V, 0, glob, "bf16")
    ctx = make_ctx(ropes, kv)
    ctx.set_qk_norm(layer, qn, kn)
    a = ctx.attn_prefill(layer, 0, Q[:700], K[:700], V[:700], 0)
    b = ctx.attn_prefill(layer, 0, Q[700:], K[700:], V[700:], 700)
    got = np.concatenate([a, b])
    assert rel_err(got, want) <= TOL
    oracle.free_cache(c)


@pytest.mark.parametrize("kv", [gc.KV_F32, gc.KV_BF16])
def test_decode_global_8192(oracle, ropes, kv):
    """Config 1: one token at position 8191 over an 8192-row global cache."""
    layer, pos = 5, 8191
    c = oracle.new_cache(True, 8192)
    kr, vr = oracle.cache_arrays(c)
    kr[:pos] = synth.normal(31, (pos, 4, 256))
    vr[:pos] = synth.normal(32, (pos, 4, 256))
    if kv == gc.KV_BF16:  # the reference sees the same (rounded) cache contents
        import torch
        kr[:pos] = torch.from_numpy(kr[:pos]).bfloat16().float().numpy()
        vr[:pos] = torch.from_numpy(vr[:pos]).bfloat16().float().numpy()
    qn, kn = synth.qk_norm_gains(33)
    Q, K, V = qkv(34, 1)
    ctx = make_ctx(ropes, kv)
    ctx.set_qk_norm(layer, qn, kn)
    ctx.import_cache(layer, 0, kr[:pos].copy(), vr[:pos].copy())
    want = oracle.attn_core_tokens(c, Q, K, V, qn, kn, ropes[1], pos)
    got = ctx.attn_decode(layer, [0], [pos], Q, K, V)
    assert rel_err(got, want) <= TOL
    kd, vd = ctx.export_cache(layer, 0)
    if kv == gc.KV_F32:
        assert np.array_equal(vd[pos], vr[pos])
    oracle.free_cache(c)


def test_decode_batch_mixed(oracle, ropes):
    """B=4 sequences at different positions on local and global layers; the
    decode path follows a prefill, the way generation does."""
    rng = [(0, 40), (1, 1030), (2, 2100), (3, 5)]
    for layer in (4, 5):
        glob = gc.is_global_layer(layer)
        rope = ropes[1] if glob else ropes[0]
        qn, kn = synth.qk_norm_gains(40 + layer)
        ctx = make_ctx(ropes, gc.KV_F32, max_batch=4)
        ctx.set_qk_norm(layer, qn, kn)
        caches, Qd, Kd, Vd, wants = [], [], [], [], []
        for s, n in rng:
            Q, K, V = qkv(1000 + 10 * s + layer, n + 1)
            c = oracle.new_cache(glob, 8192)
            full = oracle.attn_core_tokens(c, Q, K, V, qn, kn, rope, 0)
            ctx.attn_prefill(layer, s, Q[:n], K[:n], V[:n], 0)
            Qd.append(Q[n]); Kd.append(K[n]); Vd.append(V[n]); wants.append(full[n])
            caches.append(c)
        got = ctx.attn_decode(layer, [s for s, _ in rng], [n for _, n in rng], np.stack(Qd), np.stack(Kd),
                              np.stack(Vd))
        for b in range(len(rng)):
            assert rel_err(got[b], wants[b]) <= TOL, (layer, b, rel_err(got[b], wants[b]))
        for c in caches:
            oracle.free_cache(c)
        ctx.close()


def test_decode_steps_local_ring(oracle, ropes):
    """Token-by-token decode across the ring wrap on a local layer."""
    layer = 0
    qn, kn = synth.qk_norm_gains(77)
    n0, steps = 1018, 12
    Q, K, V = qkv(55, n0 + steps)
    c = oracle.new_cache(False, 8192)
    want = oracle.attn_core_tokens(c, Q, K, V, qn, kn, ropes[0], 0)
    ctx = make_ctx(ropes)
    ctx.set_qk_norm(layer, qn, kn)
    ctx.attn_prefill(layer, 0, Q[:n0], K[:n0], V[:n0], 0)
    for i in range(n0, n0 + steps):
        got = ctx.attn_decode(layer, [0], [i], Q[i:i + 1], K[i:i + 1], V[i:i + 1])
        assert rel_err(got[0], want[i]) <= TOL, i
    kr, vr = oracle.cache_arrays(c)
    kd, vd = ctx.export_cache(layer, 0)
    assert np.array_equal(vd, vr)
    oracle.free_cache(c)


def test_no_qk_norm(oracle, ropes):
    """Null gains disable QK-norm, as `if (q_norm && k_norm)` does."""
    layer, T = 0, 70
    Q, K, V = qkv(88, T)
    c = oracle.new_cache(False, 8192)
    want = oracle.attn_core_tokens(c, Q, K, V, None, None, ropes[0], 0)
    ctx = make_ctx(ropes)
    ctx.set_qk_norm(layer, None, None)
    got = ctx.attn_prefill(layer, 0, Q, K, V, 0)
    assert rel_err(got, want) <= TOL
    oracle.free_cache(c)


def test_errors_are_reported(ropes):
    ctx = make_ctx(ropes, max_context=2048, max_prefill=512)
    Q, K, V = qkv(1, 1)
    with pytest.raises(gc.Gemma3CudaError) as e:
        ctx.attn_decode(0, [0], [2048], Q, K, V)
    assert e.value.code == gc.ERR_CONTEXT_OVERFLOW
    with pytest.raises(gc.Gemma3CudaError) as e:
        ctx.attn_decode(0, [1], [3], Q, K, V)
    assert e.value.code == gc.ERR_INVALID_ARG
    with pytest.raises(gc.Gemma3CudaError) as e:
        ctx.attn_decode(40, [0], [3], Q, K, V)
    assert e.value.code == gc.ERR_INVALID_ARG
    Q, K, V = qkv(1, 600)
    with pytest.raises(gc.Gemma3CudaError) as e:
        ctx.attn_prefill(0, 0, Q, K, V, 0)
    assert e.value.code == gc.ERR_INVALID_ARG
    ctx.synchronize()


def _norm_rope_np(X, heads, w, rope, start_pos):
    """numpy restatement of per-head RMSNorm with (1+w) gain
    (gemma3_kernels.c:289-304) and rotate-half RoPE from the table
    (gemma3_kernels.c:470-484), for T tokens at positions start_pos..."""
    T = X.shape[0]
    x = X.reshape(T, heads, 256).astype(np.float64)
    if w is not None:
        g = 1.0 + synth.bf16_to_f32(np.asarray(w)).astype(np.float64)
        x = x / np.sqrt((x * x).mean(-1, keepdims=True) + 1e-6) * g
    tab = rope[start_pos:start_pos + T].astype(np.float64)  # [T][128][2]
    c, s = tab[:, None, :, 0], tab[:, None, :, 1]
    a, b = x[..., :128], x[..., 128:]
    return np.concatenate([a * c - b * s, a * s + b * c], -1).reshape(T, heads * 256).astype(np.float32)


@pytest.mark.parametrize("layer", [0, 5])
def test_prefill_8192_many_units_per_cta(ropes, layer):
    """T=8192: 512 (block, kv head) units on at most one CTA per SM, so every
    CTA carries Q, S, P and O across several units.  Checked against exact
    fp32 attention (torch, GPU) of the reference's semantics on the bf16
    cache contents."""
    import torch
    T = 8192
    glob = gc.is_global_layer(layer)
    rope = ropes[1] if glob else ropes[0]
    qn, kn = synth.qk_norm_gains(321)
    Q, K, V = qkv(4242, T)
    ctx = make_ctx(ropes, gc.KV_BF16, max_context=T, max_prefill=T)
    ctx.set_qk_norm(layer, qn, kn)
    got = ctx.attn_prefill(layer, 0, Q, K, V, 0)
    ctx.close()
    Qn = torch.from_numpy(_norm_rope_np(Q, 8, qn, rope, 0)).cuda().view(T, 8, 256)
    Kn = torch.from_numpy(bf16_round(_norm_rope_np(K, 4, kn, rope, 0))).cuda().view(T, 4, 256)
    Vb = torch.from_numpy(bf16_round(V)).cuda().view(T, 4, 256)
    pos = torch.arange(T, device="cuda")
    ok = pos[None, :] <= pos[:, None]
    if not glob:
        ok &= pos[None, :] > pos[:, None] - 1024
    want = torch.empty(T, 8, 256, device="cuda")
    for h in range(8):
        s = (Qn[:, h] @ Kn[:, h // 2].T) / 16.0
        want[:, h] = torch.softmax(s.masked_fill(~ok, float("-inf")), dim=1) @ Vb[:, h // 2]
    want = want.view(T, 2048).cpu().numpy()
    assert np.isfinite(got).all()
    assert rel_err(got, want) <= TOL, rel_err(got, want)


@pytest.mark.parametrize("layer", [0, 5])
def test_prefill_8192_against_reference(oracle, ropes, layer):
    """configs[2]'s prompt length on one layer, T=8192 from position 0, the
    reference's fp32 cache: the whole prompt against the reference compiled
    from its own sources (its per-token prefill attention,
    gemma3_transformer.c:641-692 over gemma3_gqa, gemma3_kernels.c:527-597),
    every output row within TOL x RMS, and the cache rows as the reference
    stores them."""
    T = 8192
    glob = gc.is_global_layer(layer)
    rope = ropes[1] if glob else ropes[0]
    qn, kn = synth.qk_norm_gains(700 + layer)
    Q, K, V = qkv(9100 + layer, T)
    c = oracle.new_cache(glob, T)
    want = oracle.attn_core_tokens(c, Q, K, V, qn, kn, rope, 0)
    ctx = make_ctx(ropes, gc.KV_F32, max_context=T, max_prefill=T)
    ctx.set_qk_norm(layer, qn, kn)
    got = ctx.attn_prefill(layer, 0, Q, K, V, 0)
    assert np.isfinite(got).all()
    assert rel_err(got, want) <= TOL, rel_err(got, want)
    kr, vr = oracle.cache_arrays(c)
    kd, vd = ctx.export_cache(layer, 0)
    rows = kd.shape[0]
    if glob:
        assert np.array_equal(vd[:rows], vr[:rows])
        assert rel_err(kd[:rows], kr[:rows]) < 1e-5
    else:
        # the ring holds the last 1024 positions, at slot pos % 1024, on both sides
        assert np.array_equal(vd, vr[:rows])
        assert rel_err(kd, kr[:rows]) < 1e-5
    oracle.free_cache(c)
    ctx.close()


def test_bounded_wait_times_out_and_context_survives(ropes):
    """A device wait that can never complete gives up after its limit, the
    call reports GENERATION_FAILED with the timeout text, and the same
    context then runs a normal decode correctly."""
    import time
    ctx = make_ctx(ropes, max_context=1024, max_prefill=64)
    t0 = time.time()
    rc = ctx.selftest_wait_timeout()
    dt = time.time() - t0
    assert rc == gc.ERR_GENERATION_FAILED
    assert "timed out" in ctx.last_error()
    assert 1.0 < dt < 30.0
    Q, K, V = qkv(5, 1)
    out = ctx.attn_decode(0, [0], [0], Q, K, V)  # position 0 attends only itself: out == v
    assert np.allclose(out.reshape(8, 256), V.reshape(4, 256)[np.arange(8) // 2], atol=1e-5)
    ctx.close()


def _bf16_cache(kr, vr, rows):
    import torch
    kr[:rows] = torch.from_numpy(kr[:rows]).bfloat16().float().numpy()
    vr[:rows] = torch.from_numpy(vr[:rows]).bfloat16().float().numpy()


@pytest.mark.parametrize("kv", [gc.KV_F32, gc.KV_BF16])
@pytest.mark.parametrize("layer,positions", [
    # local: units of 172..1024 rows, runs of ~167 rows straddling units
    (0, [170, 171, 255, 300, 511, 700, 1022, 1023, 1024, 1500, 2047, 2048, 3000, 4000, 5000, 8190]),
    # local: one 128-row unit per run (a segment is the whole unit)
    (0, [127]),
    # global: long units, many runs per unit
    (5, [600, 700, 1000, 1500, 2000, 3000, 4095, 8190]),
])
def test_decode_streamk_runs(oracle, ropes, kv, layer, positions):
    """Short decode calls run as equal row runs over (seq, kv head) units
    (stream-K), the last run of a unit merging its partials: two consecutive
    steps per sequence (the second reads the row the first appended) against
    the reference, for mixed lengths, runs covering two units and units
    covered by a single run."""
    glob = gc.is_global_layer(layer)
    rope = ropes[1] if glob else ropes[0]
    qn, kn = synth.qk_norm_gains(500 + layer)
    B = len(positions)
    ctx = make_ctx(ropes, kv, max_batch=B)
    ctx.set_qk_norm(layer, qn, kn)
    caches, toks, wants = [], [], []
    for s, p in enumerate(positions):
        c = oracle.new_cache(glob, 8192)
        kr, vr = oracle.cache_arrays(c)
        rows = p if glob else min(p, 1024)
        kr[:rows] = synth.normal(600 + 3 * s, (rows, 4, 256))
        vr[:rows] = synth.normal(601 + 3 * s, (rows, 4, 256))
        if kv == gc.KV_BF16:
            _bf16_cache(kr, vr, rows)
        ctx.import_cache(layer, s, kr[:rows].copy(), vr[:rows].copy())
        Q, K, V = qkv(700 + 5 * s, 2)
        wants.append(oracle.attn_core_tokens(c, Q, K, V, qn, kn, rope, p))
        toks.append((Q, K, V))
        caches.append(c)
    seqs = list(range(B))
    for step in range(2):
        got = ctx.attn_decode(layer, seqs, [p + step for p in positions], np.stack([t[0][step] for t in toks]),
                              np.stack([t[1][step] for t in toks]), np.stack([t[2][step] for t in toks]))
        for b in range(B):
            assert rel_err(got[b], wants[b][step]) <= TOL, (step, b, rel_err(got[b], wants[b][step]))
    if kv == gc.KV_F32:
        for s, p in enumerate(positions):
            kd, vd = ctx.export_cache(layer, s)
            _, vr = oracle.cache_arrays(caches[s])
            for q in (p, p + 1):
                slot = q if glob else q % 1024
                assert np.array_equal(vd[slot], vr[slot]), (s, q)
    for c in caches:
        oracle.free_cache(c)
    ctx.close()


def test_prefill_local_balanced_chunked(ropes):
    """Local layer, second prefill chunk (positions 2048..7167 over keys from
    1025): 320 units of 17 tiles on 148 CTAs, two full rounds and 24 units
    left over, which the kernel runs first as 4 key-range pieces each on
    different CTAs and merges.  Checked against exact fp32 attention (torch,
    GPU) of the reference's semantics on the bf16 cache contents."""
    import torch
    layer, T0, T1 = 2, 2048, 5120
    T = T0 + T1
    rope = ropes[0]
    qn, kn = synth.qk_norm_gains(77)
    Q, K, V = qkv(999, T)
    ctx = make_ctx(ropes, gc.KV_BF16, max_context=8192, max_prefill=T1)
    ctx.set_qk_norm(layer, qn, kn)
    ctx.attn_prefill(layer, 0, Q[:T0], K[:T0], V[:T0], 0)
    got = ctx.attn_prefill(layer, 0, Q[T0:], K[T0:], V[T0:], T0)
    ctx.close()
    Qn = torch.from_numpy(_norm_rope_np(Q[T0:], 8, qn, rope, T0)).cuda().view(T1, 8, 256)
    Kn = torch.from_numpy(bf16_round(_norm_rope_np(K, 4, kn, rope, 0))).cuda().view(T, 4, 256)
    Vb = torch.from_numpy(bf16_round(V)).cuda().view(T, 4, 256)
    qp = torch.arange(T0, T, device="cuda")[:, None]
    kp = torch.arange(T, device="cuda")[None, :]
    ok = (kp <= qp) & (kp > qp - 1024)
    want = torch.empty(T1, 8, 256, device="cuda")
    for h in range(8):
        s = (Qn[:, h] @ Kn[:, h // 2].T) / 16.0
        want[:, h] = torch.softmax(s.masked_fill(~ok, float("-inf")), dim=1) @ Vb[:, h // 2]
    want = want.view(T1, 2048).cpu().numpy()
    assert np.isfinite(got).all()
    assert rel_err(got, want) <= TOL, rel_err(got, want)


@pytest.mark.parametrize("layer,B,pos,ctxlen", [
    (0, 64, 1100, 2048),     # local layer, fused kernel, one split per (seq, kv head): in place
    (5, 64, 16384, 16385),   # global layer, long-range form (prologue + split + merge): in place
    (0, 4, 1100, 2048),      # fused kernel with several splits, each reading its q in place
])
def test_decode_pinned_host_buffers(ropes, layer, B, pos, ctxlen):
    """gemma3_cuda_attn_decode with page-locked host buffers (used in place
    by the kernels) gives bit-identical results to pageable buffers (staged
    through device copies).  Decoding the same token twice at the same
    position rewrites the same cache row, so both calls see the same cache."""
    import torch
    rope_l = gc.rope_table(ctxlen, 1e4)
    rope_g = gc.rope_table(ctxlen, 1e6)
    ctx = gc.Context(max_context=ctxlen, max_batch=B, kv_dtype=gc.KV_BF16, max_prefill=64, num_layers=6)
    ctx.upload_rope(rope_l, rope_g)
    qn, kn = synth.qk_norm_gains(61)
    ctx.set_qk_norm(layer, qn, kn)
    for s in range(B):
        ctx.fill_cache_random(layer, s, pos if gc.is_global_layer(layer) else 1024, 4000 + s)
    Q, K, V = (synth.normal(62, (B, gc.Q_SIZE)), synth.normal(63, (B, gc.KV_SIZE)),
               synth.normal(64, (B, gc.KV_SIZE)))
    seqs, poss = list(range(B)), [pos] * B
    want = ctx.attn_decode(layer, seqs, poss, Q, K, V)
    pin = [torch.from_numpy(a).pin_memory() for a in (Q, K, V)]
    out = torch.full((B, gc.Q_SIZE), float("nan")).pin_memory()
    for _ in range(2):
        got = ctx.attn_decode(layer, seqs, poss, pin[0].numpy(), pin[1].numpy(), pin[2].numpy(), out=out.numpy())
        assert np.array_equal(got, want)
    ctx.close()

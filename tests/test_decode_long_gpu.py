"""The long-range decode form against the reference's own attention.

When a CTA of the split-KV decode streams 2048 or more cache rows (the
configs[3] headline: 64 sequences x 32,769 rows of a global layer; here also
B=8, whose 9-way split has the same row counts), the library runs three
kernels: prologue_decode (QK-norm, RoPE, append), decode_splitkv in its plain
form, and merge_partials.  These tests take that form on global layers with
32,768 cached rows, in the reference's fp32 cache dtype and in bf16, and
check four sequences per batch against the reference compiled from its own
sources (oracle/_ref: gemma3_transformer.c:294-352 driving
gemma3_kernels.c:527-597), two consecutive steps each, plus the appended
cache rows.

Tolerance: max |err| <= 1e-2 x RMS of the reference output per token
(gemma3_gqa's unit of output); the appended V rows are bit-exact (fp32 cache)
or the round-to-nearest-even of the reference row (bf16 cache).
"""
import numpy as np
import pytest

import gemma3_cuda as gc
import synth
from oracles import bf16_round, best_oracle, rel_err

pytestmark = pytest.mark.gpu
TOL = 1e-2
CTX = 32770          # rows 0..32767 cached; new tokens at positions 32768 and 32769
LAYER = 5            # the only global layer of a 6-layer context
LAUNCHES_LONG = 3    # prologue_decode + decode_splitkv<plain> + merge_partials


@pytest.fixture(scope="module")
def oracle():
    return best_oracle()


@pytest.fixture(scope="module")
def rope_global(oracle):
    return oracle.rope_table(CTX, 1000000.0)


@pytest.mark.parametrize("kv", [gc.KV_F32, gc.KV_BF16])
@pytest.mark.parametrize("B", [8, 64])
def test_long_range_decode_matches_reference(oracle, rope_global, kv, B):
    # positions: the headline's 32768 for most sequences, a few shorter ones
    # (fewer splits than the longest, so some of their splits are empty)
    positions = [32768] * B
    positions[1], positions[B // 2] = 20000, 4097
    if B > 8:
        positions[3] = 100
    checked = [0, 1, B // 2, B - 1]
    qn, kn = synth.qk_norm_gains(901)
    ctx = gc.Context(max_context=CTX, max_batch=B, kv_dtype=kv, max_prefill=64, num_layers=6)
    ident = np.zeros((CTX, 128, 2), dtype=np.float32)
    ident[..., 0] = 1.0
    ctx.upload_rope(ident, rope_global)
    ctx.set_qk_norm(LAYER, qn, kn)
    for s, p in enumerate(positions):
        ctx.fill_cache_random(LAYER, s, p, 5000 + s)
    ctx.synchronize()

    Q = synth.normal(910, (2, B, gc.Q_SIZE))
    K = synth.normal(911, (2, B, gc.KV_SIZE))
    V = synth.normal(912, (2, B, gc.KV_SIZE))
    wants, caches = {}, {}
    for s in checked:
        p = positions[s]
        kd, vd = ctx.export_cache(LAYER, s)          # the rows the device holds, as fp32
        c = oracle.new_cache(True, CTX)
        kr, vr = oracle.cache_arrays(c)
        kr[:p] = kd[:p]
        vr[:p] = vd[:p]
        del kd, vd
        wants[s] = oracle.attn_core_tokens(c, Q[:, s], K[:, s], V[:, s], qn, kn, rope_global, p)
        caches[s] = c

    seqs = list(range(B))
    for step in range(2):
        n0 = ctx.launch_count()
        got = ctx.attn_decode(LAYER, seqs, [p + step for p in positions], Q[step], K[step], V[step])
        assert ctx.launch_count() - n0 == LAUNCHES_LONG, "the long-range form did not run"
        assert np.isfinite(got).all()
        for s in checked:
            e = rel_err(got[s], wants[s][step])
            assert e <= TOL, (step, s, positions[s], e)

    for s in checked:
        p = positions[s]
        kd, vd = ctx.export_cache(LAYER, s)
        kr, vr = oracle.cache_arrays(caches[s])
        rows = slice(p, p + 2)
        if kv == gc.KV_F32:
            assert np.array_equal(vd[rows], vr[rows])
            assert rel_err(kd[rows], kr[rows]) < 1e-5
        else:
            assert np.array_equal(vd[rows], bf16_round(vr[rows]))
            assert np.all(np.abs(kd[rows] - kr[rows]) <= 2.0 ** -7 * np.abs(kr[rows]) + 1e-6)
        oracle.free_cache(caches[s])
    ctx.close()

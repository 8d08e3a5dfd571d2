"""The no-allocation decode entry point (gemma3_cuda_gqa_decode_noalloc),
called through the C-ABI, against the context path gemma3_cuda_attn_decode.

This entry point serves callers that cannot allocate device memory (serving
loops that may not stall on cudaMalloc's device synchronisation, fixed-budget
processes, embedders owning all buffers); its scratch is a static device array.  The test drives the
existing entry point with QK-norm off and identity RoPE tables, so the raw Q
is exactly the query both paths attend with, exports the cache the existing
path built, and checks two consecutive no-allocation calls against it within
the parity tolerance; both are also checked against the reference's own
gemma3_gqa (oracle/_ref) on the same cache rows.  The file is named to be
collected last.
"""
import numpy as np
import pytest

import gemma3_cuda as gc
import synth
from oracles import best_oracle, rel_err

pytestmark = pytest.mark.gpu
TOL = 1e-2
MAXCTX = 4096
LAYER = 5  # a global layer: rows = MAXCTX per sequence


def _kv_device(torch, ctx, seqs, dtype):
    planes = []
    for s in seqs:
        k, v = ctx.export_cache(LAYER, s)                       # [rows][4][256] fp32
        planes.append(np.stack([k.transpose(1, 0, 2), v.transpose(1, 0, 2)]))  # [2][4][rows][256]
    t = torch.from_numpy(np.ascontiguousarray(np.stack(planes))).cuda()
    return t.to(torch.bfloat16) if dtype == gc.KV_BF16 else t


@pytest.mark.parametrize("kv_dtype", [gc.KV_F32, gc.KV_BF16])
def test_noalloc_matches_context_path(kv_dtype):
    import torch
    oracle = best_oracle()
    ident = np.zeros((MAXCTX, 128, 2), dtype=np.float32)
    ident[..., 0] = 1.0
    ctx = gc.Context(max_context=MAXCTX, max_batch=2, kv_dtype=kv_dtype, max_prefill=64)
    ctx.upload_rope(ident, ident)
    ctx.set_qk_norm(LAYER, None, None)
    ctx.fill_cache_random(LAYER, 0, 3500, 21)
    ctx.fill_cache_random(LAYER, 1, 1200, 22)
    ctx.synchronize()
    positions = [3000, 1100]
    for call in range(2):  # two calls in a row, each against a fresh reference
        Q = synth.normal(300 + call, (2, gc.Q_SIZE))
        K = synth.normal(310 + call, (2, gc.KV_SIZE))
        V = synth.normal(320 + call, (2, gc.KV_SIZE))
        want = ctx.attn_decode(LAYER, [0, 1], positions, Q, K, V)
        # the reference's gemma3_gqa on the same cache rows (what both paths
        # attend: QK-norm is off and the RoPE table is the identity)
        for b, s in enumerate((0, 1)):
            k, v = ctx.export_cache(LAYER, s)
            ref = oracle.gqa(Q[b], k, v, positions[b] + 1)
            assert rel_err(want[b], ref) <= TOL
        kv = _kv_device(torch, ctx, [0, 1], kv_dtype)
        q = torch.from_numpy(Q).cuda()
        out = torch.full((2, gc.Q_SIZE), float("nan"), device="cuda")
        gc.gqa_decode_noalloc(q.data_ptr(), kv.data_ptr(), kv_dtype, MAXCTX, [p + 1 for p in positions],
                              out.data_ptr())
        torch.cuda.synchronize()
        got = out.cpu().numpy()
        assert np.isfinite(got).all()
        assert rel_err(got, want) <= TOL, (call, rel_err(got, want))
        for b in range(2):
            k, v = ctx.export_cache(LAYER, b)
            assert rel_err(got[b], oracle.gqa(Q[b], k, v, positions[b] + 1)) <= TOL
        positions = [p + 1 for p in positions]
    ctx.close()


def test_noalloc_rejects_oversize_batch():
    import torch
    q = torch.zeros(65, gc.Q_SIZE, device="cuda")
    kv = torch.zeros(1, device="cuda")
    out = torch.zeros(65, gc.Q_SIZE, device="cuda")
    with pytest.raises(gc.Gemma3CudaError) as e:
        gc.gqa_decode_noalloc(q.data_ptr(), kv.data_ptr(), gc.KV_F32, 16, [1] * 65, out.data_ptr())
    assert e.value.code == gc.ERR_INVALID_ARG


def test_noalloc_rejects_misaligned_cache():
    """The cache is streamed with 16-byte bulk copies: a pointer off that
    boundary is refused before any launch (nothing runs on the GPU)."""
    import torch
    q = torch.zeros(1, gc.Q_SIZE, device="cuda")
    kv = torch.zeros(2 * 4 * 16 * 256 + 4, device="cuda")
    out = torch.zeros(1, gc.Q_SIZE, device="cuda")
    with pytest.raises(gc.Gemma3CudaError) as e:
        gc.gqa_decode_noalloc(q.data_ptr(), kv.data_ptr() + 4, gc.KV_F32, 16, [16], out.data_ptr())
    assert e.value.code == gc.ERR_INVALID_ARG
    assert "aligned" in str(e.value)

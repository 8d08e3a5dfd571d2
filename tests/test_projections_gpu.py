"""Parity of the tensor-core Q/K/V and O projections and of the whole-layer
attention calls (gemma3_cuda_layer_prefill / gemma3_cuda_layer_decode)
against the reference.

Projections: the reference multiplies BF16 weights by fp32 activations in
fp32 (gemma3_matvec_bf16, gemma3_kernels.c:195-225; cblas_sgemm in the
batched prefill).  The device holds the weights as fp16 (exact for these
values) and rounds the activations to fp16 once, accumulating in fp32, so
each output row is checked against the fp64 product of the reference's
operands with max |err| <= 1e-2 x RMS(row), and against the fp64 product of
the fp16-rounded operands with max |err| <= 1e-4 x RMS(row) (the GEMM itself
adds only accumulation-order error).

Whole layer: the reference's own layer_attention (gemma3_transformer.c:258-
356, compiled into oracle/_ref) run token by token, compared per token with
max |err| <= 1e-2 x RMS.
"""
import numpy as np
import pytest
import torch

import gemma3_cuda as gc
import synth
from oracles import RefOracle

pytestmark = pytest.mark.gpu
TOL = 1e-2


def _weights(seed):
    """Seeded BF16 projection weights ~ N(0, 0.02), truncated as the
    reference converts to BF16."""
    wq = synth.bf16_trunc(synth.normal(seed, (gc.Q_SIZE, gc.HIDDEN), 0.02))
    wk = synth.bf16_trunc(synth.normal(seed + 1, (gc.KV_SIZE, gc.HIDDEN), 0.02))
    wv = synth.bf16_trunc(synth.normal(seed + 2, (gc.KV_SIZE, gc.HIDDEN), 0.02))
    wo = synth.bf16_trunc(synth.normal(seed + 3, (gc.HIDDEN, gc.Q_SIZE), 0.02))
    return wq, wk, wv, wo


def _row_err(got, want):
    """max |err| / RMS per row, worst row."""
    got = np.asarray(got, dtype=np.float64)
    want = np.asarray(want, dtype=np.float64)
    rms = np.sqrt(np.mean(want * want, axis=1)) + 1e-30
    return float(np.max(np.max(np.abs(got - want), axis=1) / rms))


@pytest.fixture(scope="module")
def weights():
    return _weights(900)


@pytest.fixture(scope="module")
def ctx(weights):
    c = gc.Context(max_context=2048, max_batch=64, kv_dtype=gc.KV_F32, max_prefill=1024, num_layers=6)
    c.upload_rope(gc.rope_table(2048, 1e4), gc.rope_table(2048, 1e6))
    for layer in range(6):
        c.set_proj_weights(layer, *weights)
    yield c
    c.close()


@pytest.mark.parametrize("T", [1, 7, 64, 200, 300, 1024])
def test_projections_match_reference_product(ctx, weights, T):
    wq, wk, wv, wo = weights
    x = synth.normal(40 + T, (T, gc.HIDDEN))
    a = synth.normal(41 + T, (T, gc.Q_SIZE))
    dev = torch.device("cuda")
    xd = torch.from_numpy(x).to(dev)
    ad = torch.from_numpy(a).to(dev)
    q = torch.empty(T, gc.Q_SIZE, device=dev)
    k = torch.empty(T, gc.KV_SIZE, device=dev)
    v = torch.empty(T, gc.KV_SIZE, device=dev)
    o = torch.empty(T, gc.HIDDEN, device=dev)
    ctx.project_qkv_dev(0, T, xd.data_ptr(), q.data_ptr(), k.data_ptr(), v.data_ptr())
    ctx.project_o_dev(0, T, ad.data_ptr(), o.data_ptr())
    ctx.synchronize()
    w32 = [synth.bf16_to_f32(w) for w in (wq, wk, wv, wo)]
    h = lambda arr: arr.astype(np.float16).astype(np.float64)  # what the device multiplies
    for got, w, inp in ((q, w32[0], x), (k, w32[1], x), (v, w32[2], x), (o, w32[3], a)):
        g = got.cpu().numpy()
        assert _row_err(g, inp.astype(np.float64) @ w.astype(np.float64).T) <= TOL
        assert _row_err(g, h(inp) @ h(w).T) <= 1e-4


def test_projection_bad_arguments(ctx):
    dev = torch.device("cuda")
    x = torch.zeros(4, gc.HIDDEN, device=dev)
    with pytest.raises(gc.Gemma3CudaError) as e:
        ctx.project_qkv_dev(6, 4, x.data_ptr(), x.data_ptr(), x.data_ptr(), x.data_ptr())
    assert e.value.code == gc.ERR_INVALID_ARG
    with pytest.raises(gc.Gemma3CudaError):
        ctx.project_qkv_dev(0, 0, x.data_ptr(), x.data_ptr(), x.data_ptr(), x.data_ptr())
    other = gc.Context(max_context=256, max_batch=4, num_layers=2)
    try:
        with pytest.raises(gc.Gemma3CudaError) as e:  # weights never set
            other.project_o_dev(0, 4, x.data_ptr(), x.data_ptr())
        assert e.value.code == gc.ERR_INVALID_ARG
    finally:
        other.close()


@pytest.mark.parametrize("layer", [0, 5])
def test_layer_prefill_then_decode_match_reference_layer_attention(ctx, weights, layer):
    """Prefill 96 tokens through gemma3_cuda_layer_prefill, then 3 decode
    steps through gemma3_cuda_layer_decode, against the reference's
    layer_attention run on the same x token by token."""
    ref = RefOracle()
    glob = gc.is_global_layer(layer)
    rope = gc.rope_table(2048, 1e6 if glob else 1e4)
    qn, kn = synth.qk_norm_gains(300 + layer)
    ctx.reset()
    ctx.set_qk_norm(layer, qn, kn)
    T, steps = 96, 3
    x = synth.normal(500 + layer, (T + steps, gc.HIDDEN))
    c = ref.new_cache(glob, 2048)
    want, *_ = ref.layer_attention_tokens(c, x, *weights, qn, kn, rope, layer, 0)
    got = ctx.layer_prefill(layer, 0, x[:T], 0)
    assert _row_err(got, want[:T]) <= TOL
    for s in range(steps):
        out = ctx.layer_decode(layer, [0], [T + s], x[T + s:T + s + 1])
        assert _row_err(out, want[T + s:T + s + 1]) <= TOL


def test_layer_decode_batch_matches_single(ctx, weights):
    """A batch of 4 sequences decoded in one call equals 4 single calls."""
    layer = 0
    qn, kn = synth.qk_norm_gains(77)
    ctx.set_qk_norm(layer, qn, kn)
    x0 = synth.normal(600, (4, 40, gc.HIDDEN))
    ctx.reset()
    for s in range(4):
        ctx.layer_prefill(layer, s, x0[s], 0)
    xb = synth.normal(601, (4, gc.HIDDEN))
    batch = ctx.layer_decode(layer, [0, 1, 2, 3], [40] * 4, xb)
    ctx.reset()
    for s in range(4):
        ctx.layer_prefill(layer, s, x0[s], 0)
    single = np.stack([ctx.layer_decode(layer, [s], [40], xb[s:s + 1])[0] for s in range(4)])
    # the split-KV plan may differ with the batch size: summation order only
    assert _row_err(batch, single) <= 1e-3

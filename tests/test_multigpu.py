"""Context-parallel (split-KV) decode across GPUs: BASELINE configs[4].

A global layer's KV range is split contiguously over R ranks; each rank emits a
log-sum-exp partial (m, l, O) per (sequence, q head) for its shard, the
partials are all-gathered and merged.

  * test_lse_exchange_gloo   - CPU, two gloo processes: the exchange step with
                               real collectives, partials computed in numpy;
  * test_split_emulated_*    - one GPU: R contexts with kv_rank/kv_ranks set,
                               partial + merge through the C-ABI, against an
                               unsplit context;
  * test_split_configs4_full_size_emulated - the same at configs[4]'s own
                               size (B=4 x 131,072 keys), also against the
                               reference;
  * test_split_nccl_2gpu     - two GPUs: NCCL all-gather, then the peer-memory exchange, inside
                               gemma3_cuda_attn_decode_dev (skipped with fewer).
"""
import os
import socket
import subprocess
import sys

import numpy as np
import pytest

import synth
from oracles import rel_err

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
LOG2E = 1.4426950408889634


def _partial(q, k, v):
    """numpy (m, l, O) of one shard, log2 domain, q [8][256], k/v [rows][4][256]."""
    out = np.zeros((8, 258))
    for h in range(8):
        s = (k[:, h // 2] @ q[h]) / 16.0 * LOG2E
        if s.size == 0:
            out[h, 0], out[h, 1] = -np.inf, 0.0
            continue
        m = s.max()
        p = np.exp2(s - m)
        out[h, 0], out[h, 1], out[h, 2:] = m, p.sum(), p @ v[:, h // 2]
    return out


def _merge(parts):
    """parts [R][8][258] -> [8][256]."""
    M = parts[:, :, 0].max(axis=0)
    f = np.where(np.isfinite(parts[:, :, 0]), np.exp2(parts[:, :, 0] - M), 0.0)
    L = (parts[:, :, 1] * f).sum(0)
    O = (parts[:, :, 2:] * f[:, :, None]).sum(0)
    return O / L[:, None]


def _gloo_worker(rank, world, port, rows, result):
    import torch
    import torch.distributed as dist
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
    dist.init_process_group("gloo", rank=rank, world_size=world)
    q = synth.normal(1, (8, 256)).astype(np.float64)
    k = synth.normal(2, (rows, 4, 256)).astype(np.float64)
    v = synth.normal(3, (rows, 4, 256)).astype(np.float64)
    S = -(-rows // world)  # the library's shard: ceil(max_context / kv_ranks)
    lo, hi = min(rows, rank * S), min(rows, rank * S + S)
    mine = torch.from_numpy(_partial(q, k[lo:hi], v[lo:hi]))
    gathered = [torch.zeros_like(mine) for _ in range(world)]
    dist.all_gather(gathered, mine)
    got = _merge(np.stack([g.numpy() for g in gathered]))
    sys.path.insert(0, ROOT)
    import bench
    d = bench.Dist()
    d.pg, d.world, d.rank = dist, world, rank
    mx, sm = d.max(float(rank + 1)), d.sum(1.0)
    if rank == 0:
        want = _merge(_partial(q, k, v)[None])
        result.put((float(np.max(np.abs(got - want))), mx, sm))
    dist.destroy_process_group()


def _free_port():
    s = socket.socket()
    s.bind(("127.0.0.1", 0))
    p = s.getsockname()[1]
    s.close()
    return p


@pytest.mark.parametrize("world,rows", [(2, 1000), (2, 3), (3, 777)])
def test_lse_exchange_gloo(world, rows):
    import torch.multiprocessing as mp
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=_gloo_worker, args=(r, world, port, rows, q)) for r in range(world)]
    for p in procs:
        p.start()
    for p in procs:
        p.join(120)
        assert p.exitcode == 0
    err, mx, sm = q.get(timeout=5)
    assert err < 1e-9
    assert mx == world and sm == world


# ---------------------------------------------------------------- GPU
def _setup(gc, ctx, layer, seqs, ctxlen, full_k, full_v):
    ctx.upload_rope(gc.rope_table(ctxlen, 1e4), gc.rope_table(ctxlen, 1e6))
    qn, kn = synth.qk_norm_gains(4)
    ctx.set_qk_norm(layer, qn, kn)
    S = -(-ctxlen // ctx.cfg.kv_ranks)
    lo = min(ctxlen, ctx.cfg.kv_rank * S)
    hi = min(ctxlen, lo + S)
    for s in range(seqs):
        if hi > lo:
            ctx.import_cache(layer, s, full_k[s][lo:hi], full_v[s][lo:hi])


@pytest.mark.gpu
@pytest.mark.parametrize("R,kv", [(2, 0), (3, 1), (4, 1)])
def test_split_emulated_one_gpu(R, kv):
    import torch
    import gemma3_cuda as gc
    layer, ctxlen, B = 5, 4096, 3
    pos = [4095, 2500, 700]
    full_k = [synth.normal(10 + s, (ctxlen, 4, 256)) for s in range(B)]
    full_v = [synth.normal(20 + s, (ctxlen, 4, 256)) for s in range(B)]
    Q, K, V = synth.normal(30, (B, 2048)), synth.normal(31, (B, 1024)), synth.normal(32, (B, 1024))
    ref = gc.Context(max_context=ctxlen, max_batch=B, kv_dtype=kv, max_prefill=64)
    _setup(gc, ref, layer, B, ctxlen, full_k, full_v)
    want = ref.attn_decode(layer, list(range(B)), pos, Q, K, V)
    ref.close()
    q, k, v = (torch.from_numpy(a).cuda() for a in (Q, K, V))
    parts = torch.empty(R, B, 8, 258, device="cuda")
    ctxs = []
    for r in range(R):
        c = gc.Context(max_context=ctxlen, max_batch=B, kv_dtype=kv, max_prefill=64, kv_rank=r, kv_ranks=R)
        _setup(gc, c, layer, B, ctxlen, full_k, full_v)
        c.attn_decode_partial_dev(layer, list(range(B)), pos, q.data_ptr(), k.data_ptr(), v.data_ptr(),
                                  parts[r].data_ptr())
        c.synchronize()
        ctxs.append(c)
    out = torch.empty(B, 2048, device="cuda")
    ctxs[0].merge_partials_dev(R, B, parts.data_ptr(), out.data_ptr())
    ctxs[0].synchronize()
    assert rel_err(out.cpu().numpy(), want) <= 1e-3
    # the new row landed only on the rank owning its position
    S = -(-ctxlen // R)
    for b, p in enumerate(pos):
        owner = p // S
        kd, vd = ctxs[owner].export_cache(layer, b)
        assert np.allclose(vd[p - owner * S], V[b].reshape(4, 256), atol=1e-2)
    for c in ctxs:
        c.close()


@pytest.mark.gpu
@pytest.mark.parametrize("R", [2, 4])
def test_split_configs4_full_size_emulated(R):
    """configs[4] at its own size: B=4 sequences, 131,072-key global layer
    (new token at position 131071), BF16 cache, the KV range split over R
    contexts on one GPU (partials + merge through the C-ABI).  Checked
    against the unsplit context on all four sequences (<= 1e-3 x RMS) and
    against the reference compiled from its own sources
    (gemma3_transformer.c:294-352 driving gemma3_kernels.c:527-597) on two
    of them (<= 1e-2 x RMS); the new row lands on the last rank only."""
    import torch
    import gemma3_cuda as gc
    from oracles import best_oracle
    layer, ctxlen, B = 5, 131072, 4
    pos = [ctxlen - 1] * B
    qn, kn = synth.qk_norm_gains(44)
    ident = np.zeros((ctxlen, 128, 2), dtype=np.float32)
    ident[..., 0] = 1.0
    oracle = best_oracle()
    rope_g = oracle.rope_table(ctxlen, 1e6)
    Q, K, V = synth.normal(60, (B, 2048)), synth.normal(61, (B, 1024)), synth.normal(62, (B, 1024))

    def setup(c):
        c.upload_rope(ident, rope_g)
        c.set_qk_norm(layer, qn, kn)

    full = gc.Context(max_context=ctxlen, max_batch=B, kv_dtype=gc.KV_BF16, max_prefill=64, num_layers=6)
    setup(full)
    for s in range(B):
        full.fill_cache_random(layer, s, ctxlen - 1, 9000 + s)
    full.synchronize()
    rows = [full.export_cache(layer, s) for s in range(B)]  # fp32 copies of the BF16 rows
    want = full.attn_decode(layer, list(range(B)), pos, Q, K, V)
    full.close()

    q, k, v = (torch.from_numpy(a).cuda() for a in (Q, K, V))
    parts = torch.empty(R, B, 8, 258, device="cuda")
    S = -(-ctxlen // R)
    ctxs = []
    for r in range(R):
        c = gc.Context(max_context=ctxlen, max_batch=B, kv_dtype=gc.KV_BF16, max_prefill=64, num_layers=6,
                       kv_rank=r, kv_ranks=R)
        setup(c)
        lo, hi = r * S, min(ctxlen - 1, (r + 1) * S)
        for s in range(B):
            c.import_cache(layer, s, rows[s][0][lo:hi], rows[s][1][lo:hi])
        c.attn_decode_partial_dev(layer, list(range(B)), pos, q.data_ptr(), k.data_ptr(), v.data_ptr(),
                                  parts[r].data_ptr())
        c.synchronize()
        ctxs.append(c)
    out = torch.empty(B, 2048, device="cuda")
    ctxs[0].merge_partials_dev(R, B, parts.data_ptr(), out.data_ptr())
    ctxs[0].synchronize()
    got = out.cpu().numpy()
    assert np.isfinite(got).all()
    assert rel_err(got, want) <= 1e-3
    # the new token's row (position 131071) belongs to the last rank
    kd, vd = ctxs[R - 1].export_cache(layer, 0)
    assert np.array_equal(vd[pos[0] - (R - 1) * S], oracle_bf16(V[0]).reshape(4, 256))
    for c in ctxs:
        c.close()
    for s in (0, B - 1):
        cache = oracle.new_cache(True, ctxlen)
        kr, vr = oracle.cache_arrays(cache)
        kr[:ctxlen - 1] = rows[s][0][:ctxlen - 1]
        vr[:ctxlen - 1] = rows[s][1][:ctxlen - 1]
        ref = oracle.attn_core_tokens(cache, Q[None, s], K[None, s], V[None, s], qn, kn, rope_g, pos[s])
        oracle.free_cache(cache)
        assert rel_err(got[s], ref[0]) <= 1e-2, s


def oracle_bf16(x):
    from oracles import bf16_round
    return bf16_round(np.asarray(x, dtype=np.float32))


NCCL_CHILD = r'''
import os, sys, json
sys.path[:0] = [os.path.join(sys.argv[1], "gemma3.c_b200"), os.path.join(sys.argv[1], "oracle")]
import numpy as np, torch, torch.distributed as dist
import gemma3_cuda as gc, synth
rank, world = int(os.environ["RANK"]), int(os.environ["WORLD_SIZE"])
torch.cuda.set_device(rank)
dist.init_process_group("gloo")
layer, ctxlen, B, pos = 5, 4096, 2, [4095, 1500]
full_k = [synth.normal(10 + s, (ctxlen, 4, 256)) for s in range(B)]
full_v = [synth.normal(20 + s, (ctxlen, 4, 256)) for s in range(B)]
Q, K, V = synth.normal(30, (B, 2048)), synth.normal(31, (B, 1024)), synth.normal(32, (B, 1024))
def setup(c):
    c.upload_rope(gc.rope_table(ctxlen, 1e4), gc.rope_table(ctxlen, 1e6))
    qn, kn = synth.qk_norm_gains(4); c.set_qk_norm(layer, qn, kn)
    S = -(-ctxlen // c.cfg.kv_ranks); lo = min(ctxlen, c.cfg.kv_rank * S); hi = min(ctxlen, lo + S)
    for s in range(B):
        c.import_cache(layer, s, full_k[s][lo:hi], full_v[s][lo:hi])
uid = [gc.Context.comm_unique_id() if rank == 0 else None]
dist.broadcast_object_list(uid, src=0)
c = gc.Context(max_context=ctxlen, max_batch=B, kv_dtype=gc.KV_BF16, device=rank, max_prefill=64,
               kv_rank=rank, kv_ranks=world)
setup(c)
c.comm_init(uid[0])
q, k, v = (torch.from_numpy(a).cuda() for a in (Q, K, V))
out = torch.empty(B, 2048, device="cuda")
c.attn_decode_dev(layer, [0, 1], pos, q.data_ptr(), k.data_ptr(), v.data_ptr(), out.data_ptr())
c.synchronize()
got = out.cpu().numpy()
# the same call through the peer-memory exchange, three times in a row (both
# buffer parities, and a parity reused), then once more through NCCL
c.peer_init()
peer = []
for _ in range(3):
    out.zero_()
    c.attn_decode_dev(layer, [0, 1], pos, q.data_ptr(), k.data_ptr(), v.data_ptr(), out.data_ptr())
    c.synchronize()
    peer.append(out.cpu().numpy())
c.set_exchange(gc.XCHG_NCCL)
out.zero_()
c.attn_decode_dev(layer, [0, 1], pos, q.data_ptr(), k.data_ptr(), v.data_ptr(), out.data_ptr())
c.synchronize()
again = out.cpu().numpy()
if rank == 0:
    ref = gc.Context(max_context=ctxlen, max_batch=B, kv_dtype=gc.KV_BF16, device=0, max_prefill=64)
    setup(ref)
    want = ref.attn_decode(layer, [0, 1], pos, Q, K, V)
    rms = np.sqrt(np.mean(want ** 2))
    e = np.max(np.abs(got - want)) / rms
    ep = max(float(np.max(np.abs(p_ - got)) / rms) for p_ in peer)
    ea = float(np.max(np.abs(again - got)) / rms)
    print(json.dumps({"err": float(e), "peer_vs_nccl": ep, "nccl_again": ea}))
c.close()
dist.destroy_process_group()
'''


@pytest.mark.gpu
def test_split_nccl_2gpu(tmp_path):
    import torch
    if torch.cuda.device_count() < 2:
        pytest.skip("needs 2 GPUs")
    script = tmp_path / "child.py"
    script.write_text(NCCL_CHILD)
    env = dict(os.environ, NCCL_NVLS_ENABLE="0")
    r = subprocess.run([sys.executable, "-m", "torch.distributed.run", "--nnodes=1", "--nproc-per-node=2",
                        "--master-addr", "127.0.0.1", "--master-port", str(_free_port()), str(script), ROOT],
                       capture_output=True, text=True, timeout=300, env=env)
    assert r.returncode == 0, r.stderr[-3000:]
    line = [l for l in r.stdout.splitlines() if l.startswith("{")][-1]
    import json
    res = json.loads(line)
    assert res["err"] <= 1e-3
    # the peer exchange merges the same partials in the same order as the
    # all-gather path: identical up to float rounding of the merge
    assert res["peer_vs_nccl"] <= 1e-6
    assert res["nccl_again"] <= 1e-6


# ---------------------------------------------------------------- prefill
def _prefill_partial(q, k, v, lo, hi):
    """numpy: queries q [T][8][256] at positions 0..T-1, keys [lo, hi) of k/v
    [T][4][256], causal.  Returns (O normalised over those keys [T][8][256],
    m [T][8] log2-domain reference max, l [T][8]); rows with no key: 0, 0, 0."""
    T = q.shape[0]
    O = np.zeros((T, 8, 256))
    m = np.zeros((T, 8))
    l = np.zeros((T, 8))
    for t in range(T):
        kh = min(hi, t + 1)
        if kh <= lo:
            continue
        for h in range(8):
            s = (k[lo:kh, h // 2] @ q[t, h]) / 16.0 * LOG2E
            mm = s.max()
            p = np.exp2(s - mm)
            m[t, h], l[t, h] = mm, p.sum()
            O[t, h] = p @ v[lo:kh, h // 2] / p.sum()
    return O, m, l


def _prefill_merge(Os, ms, ls):
    """The log-sum-exp merge of merge_prefill_partials: w_r = l_r 2^(m_r - M)."""
    M = np.where(ls > 0, ms, -np.inf).max(axis=0)
    w = np.where(ls > 0, ls * np.exp2(ms - np.where(np.isfinite(M), M, 0.0)), 0.0)
    W = w.sum(0)
    return (Os * w[..., None]).sum(0) / np.where(W > 0, W, 1.0)[..., None]


def _gloo_prefill_worker(rank, world, port, T, result):
    import torch
    import torch.distributed as dist
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
    dist.init_process_group("gloo", rank=rank, world_size=world)
    q = synth.normal(41, (T, 8, 256)).astype(np.float64)
    k = synth.normal(42, (T, 4, 256)).astype(np.float64)
    v = synth.normal(43, (T, 4, 256)).astype(np.float64)
    S = -(-T // world)
    lo, hi = min(T, rank * S), min(T, rank * S + S)
    O, m, l = _prefill_partial(q, k, v, lo, hi)
    mine = torch.from_numpy(np.concatenate([O.reshape(T, -1), m, l], axis=1))
    gathered = [torch.zeros_like(mine) for _ in range(world)]
    dist.all_gather(gathered, mine)
    g = np.stack([x.numpy() for x in gathered])
    got = _prefill_merge(g[:, :, :2048].reshape(world, T, 8, 256), g[:, :, 2048:2056], g[:, :, 2056:2064])
    if rank == 0:
        O1, _, _ = _prefill_partial(q, k, v, 0, T)
        result.put(float(np.max(np.abs(got - O1))))
    dist.destroy_process_group()


@pytest.mark.parametrize("world,T", [(2, 40), (3, 37)])
def test_prefill_lse_exchange_gloo(world, T):
    """The context-parallel prefill's exchange with real collectives (gloo):
    each rank's outputs over its key shard with (m, l), all-gathered and
    merged as merge_prefill_partials does, equal attention over all keys."""
    import torch.multiprocessing as mp
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=_gloo_prefill_worker, args=(r, world, port, T, q)) for r in range(world)]
    for p in procs:
        p.start()
    for p in procs:
        p.join(120)
        assert p.exitcode == 0
    assert q.get(timeout=5) < 1e-9


@pytest.mark.gpu
@pytest.mark.parametrize("R,kv", [(2, 1), (3, 0), (4, 1)])
def test_prefill_split_emulated_one_gpu(R, kv):
    """Prefill into a context-parallel global layer, R ranks as R contexts on
    one GPU: a 1,500-token prompt then a 700-token chunk, each rank's partial
    through gemma3_cuda_attn_prefill_partial_dev, merged by
    gemma3_cuda_merge_prefill_partials_dev, against the unsplit context and
    against the reference's own attention (oracle/_ref); every rank's cache
    holds exactly its positions' rows."""
    import torch
    import gemma3_cuda as gc
    from oracles import best_oracle, exact_attention
    layer, ctxlen, T0, T1 = 5, 4096, 1500, 700
    T = T0 + T1
    Q, K, V = synth.normal(50, (T, 2048)), synth.normal(51, (T, 1024)), synth.normal(52, (T, 1024))
    qn, kn = synth.qk_norm_gains(53)
    rope_l, rope_g = gc.rope_table(ctxlen, 1e4), gc.rope_table(ctxlen, 1e6)

    def make(**kw):
        c = gc.Context(max_context=ctxlen, max_batch=1, kv_dtype=kv, max_prefill=T0, num_layers=6, **kw)
        c.upload_rope(rope_l, rope_g)
        c.set_qk_norm(layer, qn, kn)
        return c

    ref = make()
    want = np.concatenate([ref.attn_prefill(layer, 0, Q[:T0], K[:T0], V[:T0], 0),
                           ref.attn_prefill(layer, 0, Q[T0:], K[T0:], V[T0:], T0)])
    kref, vref = ref.export_cache(layer, 0)
    ref.close()
    oracle = best_oracle()
    c0 = oracle.new_cache(True, ctxlen)
    exact = oracle.attn_core_tokens(c0, Q, K, V, qn, kn, oracle.rope_table(ctxlen, 1e6), 0)
    oracle.free_cache(c0)
    if kv == gc.KV_BF16:  # the reference's semantics on the rows a BF16 cache holds
        Qn, Kn = oracle.last_qk
        exact = exact_attention(Qn, Kn, V, 0, True, "bf16")

    q, k, v = (torch.from_numpy(a).cuda() for a in (Q, K, V))
    ctxs = [make(kv_rank=r, kv_ranks=R) for r in range(R)]
    got = []
    for t0, n in ((0, T0), (T0, T1)):
        outs = torch.empty(R, n, 2048, device="cuda")
        mls = torch.empty(R, n, 8, 2, device="cuda")
        for r, c in enumerate(ctxs):
            c.attn_prefill_partial_dev(layer, 0, q[t0:].data_ptr(), k[t0:].data_ptr(), v[t0:].data_ptr(), n, t0,
                                       outs[r].data_ptr(), mls[r].data_ptr())
            c.synchronize()
        out = torch.empty(n, 2048, device="cuda")
        ctxs[0].merge_prefill_partials_dev(R, n, outs.data_ptr(), mls.data_ptr(), out.data_ptr())
        ctxs[0].synchronize()
        got.append(out.cpu().numpy())
    got = np.concatenate(got)
    assert np.isfinite(got).all()
    assert rel_err(got, want) <= 2e-3, rel_err(got, want)
    assert rel_err(got, exact) <= 1e-2, rel_err(got, exact)
    S = -(-ctxlen // R)
    for r, c in enumerate(ctxs):
        lo, hi = min(ctxlen, r * S), min(T, r * S + S)
        kd, vd = c.export_cache(layer, 0)
        if hi > lo:
            assert np.array_equal(vd[:hi - lo], vref[lo:hi]), r
            assert np.array_equal(kd[:hi - lo], kref[lo:hi]), r
        c.close()


NCCL_PREFILL_CHILD = r'''
import os, sys, json
sys.path[:0] = [os.path.join(sys.argv[1], "gemma3.c_b200"), os.path.join(sys.argv[1], "oracle")]
import numpy as np, torch, torch.distributed as dist
import gemma3_cuda as gc, synth
rank, world = int(os.environ["RANK"]), int(os.environ["WORLD_SIZE"])
torch.cuda.set_device(rank)
dist.init_process_group("gloo")
layer, ctxlen, T = 5, 4096, 3000
Q, K, V = synth.normal(60, (T, 2048)), synth.normal(61, (T, 1024)), synth.normal(62, (T, 1024))
qn, kn = synth.qk_norm_gains(63)
def make(**kw):
    c = gc.Context(max_context=ctxlen, max_batch=1, kv_dtype=gc.KV_BF16, max_prefill=T, num_layers=6, **kw)
    c.upload_rope(gc.rope_table(ctxlen, 1e4), gc.rope_table(ctxlen, 1e6)); c.set_qk_norm(layer, qn, kn)
    return c
uid = [gc.Context.comm_unique_id() if rank == 0 else None]
dist.broadcast_object_list(uid, src=0)
c = make(device=rank, kv_rank=rank, kv_ranks=world)
c.comm_init(uid[0])
q, k, v = (torch.from_numpy(a).cuda() for a in (Q, K, V))
out = torch.empty(T, 2048, device="cuda")
c.attn_prefill_dev(layer, 0, q.data_ptr(), k.data_ptr(), v.data_ptr(), T, 0, out.data_ptr())
c.synchronize()
got = out.cpu().numpy()
if rank == 0:
    ref = make(device=0)
    want = ref.attn_prefill(layer, 0, Q, K, V, 0)
    print(json.dumps({"err": float(np.max(np.abs(got - want)) / np.sqrt(np.mean(want ** 2)))}))
    ref.close()
c.close()
dist.destroy_process_group()
'''


@pytest.mark.gpu
def test_prefill_split_nccl_2gpu(tmp_path):
    """gemma3_cuda_attn_prefill_dev on a context-parallel global layer over
    two GPUs (partial, NCCL all-gather, merge inside the call) against the
    unsplit prefill."""
    import torch
    if torch.cuda.device_count() < 2:
        pytest.skip("needs 2 GPUs")
    script = tmp_path / "child.py"
    script.write_text(NCCL_PREFILL_CHILD)
    env = dict(os.environ, NCCL_NVLS_ENABLE="0")
    r = subprocess.run([sys.executable, "-m", "torch.distributed.run", "--nnodes=1", "--nproc-per-node=2",
                        "--master-addr", "127.0.0.1", "--master-port", str(_free_port()), str(script), ROOT],
                       capture_output=True, text=True, timeout=300, env=env)
    assert r.returncode == 0, r.stderr[-3000:]
    import json
    res = json.loads([l for l in r.stdout.splitlines() if l.startswith("{")][-1])
    assert res["err"] <= 2e-3


NCCL_SKIP_CHILD = r'''
import os, sys, json, time
sys.path[:0] = [os.path.join(sys.argv[1], "gemma3.c_b200"), os.path.join(sys.argv[1], "oracle")]
import numpy as np, torch, torch.distributed as dist
import gemma3_cuda as gc, synth
rank, world = int(os.environ["RANK"]), int(os.environ["WORLD_SIZE"])
torch.cuda.set_device(rank)
dist.init_process_group("gloo")
layer, ctxlen, B, pos = 5, 4096, 2, [4095, 1500]
full_k = [synth.normal(10 + s, (ctxlen, 4, 256)) for s in range(B)]
full_v = [synth.normal(20 + s, (ctxlen, 4, 256)) for s in range(B)]
Q, K, V = synth.normal(30, (B, 2048)), synth.normal(31, (B, 1024)), synth.normal(32, (B, 1024))
def setup(c):
    c.upload_rope(gc.rope_table(ctxlen, 1e4), gc.rope_table(ctxlen, 1e6))
    qn, kn = synth.qk_norm_gains(4); c.set_qk_norm(layer, qn, kn)
    S = -(-ctxlen // c.cfg.kv_ranks); lo = min(ctxlen, c.cfg.kv_rank * S); hi = min(ctxlen, lo + S)
    for s in range(B):
        c.import_cache(layer, s, full_k[s][lo:hi], full_v[s][lo:hi])
uid = [gc.Context.comm_unique_id() if rank == 0 else None]
dist.broadcast_object_list(uid, src=0)
c = gc.Context(max_context=ctxlen, max_batch=B, kv_dtype=gc.KV_BF16, device=rank, max_prefill=64,
               kv_rank=rank, kv_ranks=world)
setup(c)
c.comm_init(uid[0])
c.peer_init()
q, k, v = (torch.from_numpy(a).cuda() for a in (Q, K, V))
out = torch.empty(B, 2048, device="cuda")
def step():
    c.attn_decode_dev(layer, [0, 1], pos, q.data_ptr(), k.data_ptr(), v.data_ptr(), out.data_ptr())
    c.synchronize()
    return out.cpu().numpy()
first = step()
dist.barrier()
# rank 1 skips one exchange: rank 0's bounded wait for its flag gives up
res = {}
if rank == 0:
    t0 = time.time()
    try:
        step()
        res["skipped_rc"] = 0
    except gc.Gemma3CudaError as e:
        res["skipped_rc"] = e.code
        res["msg"] = str(e)
    res["wait_s"] = time.time() - t0
dist.barrier()
# recovery: every rank resets (caches, exchange epochs and flags), then the caches are rebuilt
c.reset()
setup(c)
dist.barrier()
again = step()
if rank == 0:
    res["recovered_err"] = float(np.max(np.abs(again - first)) / np.sqrt(np.mean(first ** 2)))
    print(json.dumps(res))
c.close()
dist.destroy_process_group()
'''


@pytest.mark.gpu
def test_peer_exchange_skipped_rank_recovers_2gpu(tmp_path):
    """A rank that skips one peer-memory exchange: the other rank's bounded
    flag wait gives up (GENERATION_FAILED, about 2 s, no trap), both ranks
    call gemma3_cuda_reset, and the next exchange is correct again."""
    import torch
    import gemma3_cuda as gc
    if torch.cuda.device_count() < 2:
        pytest.skip("needs 2 GPUs")
    script = tmp_path / "child.py"
    script.write_text(NCCL_SKIP_CHILD)
    env = dict(os.environ, NCCL_NVLS_ENABLE="0")
    r = subprocess.run([sys.executable, "-m", "torch.distributed.run", "--nnodes=1", "--nproc-per-node=2",
                        "--master-addr", "127.0.0.1", "--master-port", str(_free_port()), str(script), ROOT],
                       capture_output=True, text=True, timeout=300, env=env)
    assert r.returncode == 0, r.stderr[-3000:]
    import json
    res = json.loads([l for l in r.stdout.splitlines() if l.startswith("{")][-1])
    assert res["skipped_rc"] == gc.ERR_GENERATION_FAILED, res
    assert "timed out" in res.get("msg", ""), res
    assert 1.0 < res["wait_s"] < 30.0, res
    assert res["recovered_err"] <= 1e-6, res

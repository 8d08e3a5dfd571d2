"""SafeTensors checkpoint loading (gemma3_cuda_safetensors_check /
gemma3_cuda_load_safetensors), which reads checkpoints the way the reference's
gemma3_load_weights does (gemma3_safetensors.c:393-486, :651-713): every
*.safetensors file of the directory, tensor names
"language_model.model.layers.<l>.<...>.weight", BF16.

The host-only check runs on sparse synthetic checkpoints (real headers, data
regions left as holes), so these tests need no GPU and little disk; the GPU
test loads a small real checkpoint and compares the model's output with the
same weights uploaded directly.
"""
import json
import os

import numpy as np
import pytest

import gemma3_cuda as gc

H, QS, KS, I, HD = 2560, 2048, 1024, 10240, 256
LAYER_TENSORS = [
    ("input_layernorm.weight", (H,)),
    ("self_attn.q_proj.weight", (QS, H)),
    ("self_attn.k_proj.weight", (KS, H)),
    ("self_attn.v_proj.weight", (KS, H)),
    ("self_attn.o_proj.weight", (H, QS)),
    ("self_attn.q_norm.weight", (HD,)),
    ("self_attn.k_norm.weight", (HD,)),
    ("post_attention_layernorm.weight", (H,)),
    ("mlp.gate_proj.weight", (I, H)),
    ("mlp.up_proj.weight", (I, H)),
    ("mlp.down_proj.weight", (H, I)),
    ("pre_feedforward_layernorm.weight", (H,)),
    ("post_feedforward_layernorm.weight", (H,)),
]


def model_tensors(n_layers, vocab, prefix="language_model.model."):
    t = [(prefix + "embed_tokens.weight", (vocab, H)), (prefix + "norm.weight", (H,))]
    for l in range(n_layers):
        t += [(f"{prefix}layers.{l}.{n}", s) for n, s in LAYER_TENSORS]
    return t


def write_shard(path, tensors, data=None, dtype="BF16", header_extra=None):
    """tensors: [(name, shape)]; data: {name: uint16 array} or None (sparse)."""
    header, off = {"__metadata__": {"format": "pt"}}, 0
    for name, shape in tensors:
        n = int(np.prod(shape)) * 2
        header[name] = {"dtype": dtype, "shape": list(shape), "data_offsets": [off, off + n]}
        off += n
    if header_extra:
        header.update(header_extra)
    h = json.dumps(header).encode()
    h += b" " * (-len(h) % 8)
    with open(path, "wb") as f:
        f.write(len(h).to_bytes(8, "little"))
        f.write(h)
        if data is None:
            f.truncate(8 + len(h) + off)
        else:
            for name, shape in tensors:
                f.write(np.ascontiguousarray(data[name], dtype=np.uint16).tobytes())


def write_model(d, n_layers, vocab, data=None, prefix="language_model.model.", **kw):
    t = model_tensors(n_layers, vocab, prefix)
    half = len(t) // 2
    write_shard(os.path.join(d, "model-00001-of-00002.safetensors"), t[:half], data, **kw)
    write_shard(os.path.join(d, "model-00002-of-00002.safetensors"), t[half:], data, **kw)


def test_check_accepts_a_two_shard_checkpoint(tmp_path):
    write_model(str(tmp_path), 2, 1000)
    assert gc.safetensors_check(str(tmp_path), 2) == 1000


def test_check_accepts_text_only_names(tmp_path):
    write_model(str(tmp_path), 1, 64, prefix="model.")
    assert gc.safetensors_check(str(tmp_path), 1) == 64


def test_check_accepts_missing_optional_norms(tmp_path):
    t = [x for x in model_tensors(1, 64) if "feedforward_layernorm" not in x[0]]
    write_shard(str(tmp_path / "a.safetensors"), t)
    assert gc.safetensors_check(str(tmp_path), 1) == 64


@pytest.mark.parametrize("case,needle", [
    ("missing", "not found"), ("dtype", "not BF16"), ("shape", "has shape"), ("layers", "not found"),
    ("offsets", "outside the file"), ("json", "malformed"), ("empty", "no .safetensors"),
])
def test_check_rejects_bad_checkpoints(tmp_path, case, needle):
    d = str(tmp_path)
    if case == "missing":
        t = [x for x in model_tensors(1, 64) if not x[0].endswith("mlp.up_proj.weight")]
        write_shard(os.path.join(d, "a.safetensors"), t)
    elif case == "dtype":
        write_model(d, 1, 64, dtype="F16")
    elif case == "shape":
        t = [(n, (QS, 2048) if n.endswith("q_proj.weight") else s) for n, s in model_tensors(1, 64)]
        write_shard(os.path.join(d, "a.safetensors"), t)
    elif case == "layers":
        write_model(d, 1, 64)  # asked for 2 layers below
    elif case == "offsets":
        write_model(d, 1, 64, header_extra={"extra": {"dtype": "BF16", "shape": [4], "data_offsets": [0, 1 << 40]}})
    elif case == "json":
        with open(os.path.join(d, "a.safetensors"), "wb") as f:
            h = b'{"x": {"dtype": "BF16", "shape": [2, '
            f.write(len(h).to_bytes(8, "little") + h)
    with pytest.raises(gc.Gemma3CudaError) as e:
        gc.safetensors_check(d, 2 if case == "layers" else 1)
    assert needle in str(e.value)


SLOT_NAMES = [n for n, _ in LAYER_TENSORS]  # gemma3_weights_t order of a layer's 13 weights
REF_LAYERS = 34                              # gemma3_load_weights always walks GEMMA3_NUM_LAYERS


def _ref_oracle():
    from oracles import RefOracle
    try:
        return RefOracle()
    except (FileNotFoundError, OSError):
        pytest.skip("reference build (oracle/_ref) not available")


def _random_checkpoint(d, L, V, seed):
    """L layers, vocab V, BF16 ~N(0, 0.02) matrices and ~N(0, 0.1) norms, two shards."""
    import synth
    rng = np.random.default_rng(seed)

    def w(shape, std=0.02):
        return synth.bf16_trunc((rng.standard_normal(shape, dtype=np.float32) * std).astype(np.float32))

    pre = "language_model.model."
    data = {pre + "embed_tokens.weight": w((V, H)), pre + "norm.weight": w((H,), 0.1)}
    for l in range(L):
        for n, shp in LAYER_TENSORS:
            data[f"{pre}layers.{l}.{n}"] = w(shp, 0.1 if len(shp) == 1 else 0.02)
    write_model(d, L, V, data)
    return data


def _slot_shapes(L, V):
    shapes = {0: (V, H), 1 + 13 * REF_LAYERS: (H,)}
    for l in range(L):
        for j, (_, shp) in enumerate(LAYER_TENSORS):
            shapes[1 + 13 * l + j] = shp
    return shapes


def test_reference_loader_reads_the_fixture(tmp_path):
    """The reference's own loader (st_load + gemma3_load_weights, compiled
    from its sources into oracle/_ref) resolves every weight of the two-shard
    fixture to the bytes written, and leaves the absent layers NULL: the
    fixture is a checkpoint in the reference's sense."""
    ref = _ref_oracle()
    L, V = 2, 96
    data = _random_checkpoint(str(tmp_path), L, V, 7100)
    got, missing = ref.load_weights(str(tmp_path), _slot_shapes(L, V))
    pre = "language_model.model."
    assert np.array_equal(got[0], data[pre + "embed_tokens.weight"])
    assert np.array_equal(got[1 + 13 * REF_LAYERS], data[pre + "norm.weight"])
    for l in range(L):
        for j, n in enumerate(SLOT_NAMES):
            assert np.array_equal(got[1 + 13 * l + j], data[f"{pre}layers.{l}.{n}"]), (l, n)
    assert missing == list(range(1 + 13 * L, 1 + 13 * REF_LAYERS))


@pytest.mark.gpu
def test_load_matches_reference_loader(tmp_path):
    """gemma3_cuda_load_safetensors against the reference's loader: the
    weights the reference's gemma3_load_weights resolves (read through its
    own pointers) are uploaded directly into one context, the checkpoint is
    loaded by this library into another, and a prompt plus one greedy step
    give identical tokens and top-1 logits."""
    ref = _ref_oracle()
    L, V = 2, 512
    _random_checkpoint(str(tmp_path), L, V, 7200)
    got, _ = ref.load_weights(str(tmp_path), _slot_shapes(L, V))

    def run(ctx):
        ctx.upload_rope(gc.rope_table(256, 1e4), gc.rope_table(256, 1e6))
        nxt, top = ctx.prefill_greedy(0, [3, 1, 4, 1, 5, 9, 2, 6], 0)
        n2, t2 = ctx.greedy_step([0], [8], [nxt])
        return nxt, top, int(n2[0]), float(t2[0])

    a = gc.Context(max_context=256, max_batch=1, max_prefill=8, num_layers=L)
    try:
        a.load_safetensors(str(tmp_path))
        mine = run(a)
    finally:
        a.close()
    b = gc.Context(max_context=256, max_batch=1, max_prefill=8, num_layers=L)
    try:
        for l in range(L):
            lw = {n.replace(".weight", "").replace("self_attn.", "").replace("mlp.", ""): got[1 + 13 * l + j]
                  for j, n in enumerate(SLOT_NAMES)}
            b.set_layer_weights(l, **lw)
        b.set_embeddings(got[0], got[1 + 13 * REF_LAYERS])
        theirs = run(b)
    finally:
        b.close()
    assert mine == theirs


@pytest.mark.gpu
def test_load_matches_direct_upload(tmp_path):
    """2 layers, vocab 512: a prompt and one greedy step give the same tokens
    and top-1 logits whether the weights come from the checkpoint files or
    from gemma3_cuda_set_layer_weights / gemma3_cuda_set_embeddings."""
    import synth
    L, V = 2, 512
    rng = np.random.default_rng(7000)

    def w(shape, std=0.02):
        return synth.bf16_trunc((rng.standard_normal(shape, dtype=np.float32) * std).astype(np.float32))

    data, per_layer = {}, []
    pre = "language_model.model."
    data[pre + "embed_tokens.weight"] = w((V, H))
    data[pre + "norm.weight"] = w((H,), 0.1)
    for l in range(L):
        lw = {}
        for n, s in LAYER_TENSORS:
            a = w(s, 0.1 if len(s) == 1 else 0.02)
            data[f"{pre}layers.{l}.{n}"] = a
            lw[n.replace(".weight", "").replace("self_attn.", "").replace("mlp.", "")] = a
        per_layer.append(lw)
    write_model(str(tmp_path), L, V, data)

    def run(ctx):
        ctx.upload_rope(gc.rope_table(256, 1e4), gc.rope_table(256, 1e6))
        nxt, top = ctx.prefill_greedy(0, [3, 1, 4, 1, 5, 9, 2, 6], 0)
        n2, t2 = ctx.greedy_step([0], [8], [nxt])
        return nxt, top, int(n2[0]), float(t2[0])

    a = gc.Context(max_context=256, max_batch=1, max_prefill=8, num_layers=L)
    try:
        a.load_safetensors(str(tmp_path))
        got = run(a)
    finally:
        a.close()
    b = gc.Context(max_context=256, max_batch=1, max_prefill=8, num_layers=L)
    try:
        for l, lw in enumerate(per_layer):
            b.set_layer_weights(l, **lw)
        b.set_embeddings(data[pre + "embed_tokens.weight"], data[pre + "norm.weight"])
        want = run(b)
    finally:
        b.close()
    assert got == want

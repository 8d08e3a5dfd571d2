"""End-to-end greedy decoding on the random-init 34-layer Gemma-3-4B: the
reference's own forward pass vs the same model with the attention core on the
B200 (prompt through gemma3_cuda_attn_prefill, 32 generated tokens through
gemma3_cuda_attn_decode), and with every transformer block on the B200.  The
first 32 tokens must match; the top-1 logits of every step must agree within
1e-2 relative (the margins are logged).  The reference arm runs the prompt
through the reference's own prefill (gemma3_transformer_prefill, as
gemma3_generate does) and each generated token through
gemma3_transformer_forward.  Two prompt lengths: 8 tokens, and 1,100 tokens,
where the local layers' 1024-row ring wraps during the prompt and keeps
wrapping while the 32 tokens are generated, so local and global layers attend
to different keys (gemma3_transformer.c:330-346).
Harness: oracle/e2e_harness.c (test infrastructure)."""
import ctypes
import os

import numpy as np
import pytest

pytestmark = pytest.mark.gpu
ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
SO = os.path.join(ROOT, "oracle", "_ref", "libgemma3_e2e.so")
N_PROMPT, N_STEPS = 8, 32


def _arm(lib, use_cuda, kv_dtype=0, n_prompt=N_PROMPT):
    if use_cuda == 0 and n_prompt in _REF:
        return _REF[n_prompt]
    toks = np.zeros(N_STEPS, np.int32)
    marg = np.zeros(N_STEPS, np.float32)
    top = np.zeros(N_STEPS, np.float32)
    rc = lib.e2e_greedy(n_prompt, N_STEPS, 20241, use_cuda, kv_dtype, toks.ctypes.data, marg.ctypes.data,
                        top.ctypes.data)
    assert rc == 0
    if use_cuda == 0:
        _REF[n_prompt] = (toks, marg, top)
    return toks, marg, top


_REF = {}  # the reference arm's result per prompt length (it is the slow arm)


def _lib():
    if not os.path.exists(SO):
        pytest.skip("e2e harness not built (needs the reference sources at build time)")
    os.environ.setdefault("OPENBLAS_NUM_THREADS", "1")
    lib = ctypes.CDLL(SO)
    lib.e2e_greedy.argtypes = [ctypes.c_int, ctypes.c_int, ctypes.c_uint64, ctypes.c_int, ctypes.c_int,
                               ctypes.c_void_p, ctypes.c_void_p, ctypes.c_void_p]
    return lib


def test_greedy_32_steps_match():
    if not os.path.exists(SO):
        pytest.skip("e2e harness not built (needs the reference sources at build time)")
    os.environ.setdefault("OPENBLAS_NUM_THREADS", "1")
    lib = ctypes.CDLL(SO)
    lib.e2e_greedy.argtypes = [ctypes.c_int, ctypes.c_int, ctypes.c_uint64, ctypes.c_int, ctypes.c_int,
                               ctypes.c_void_p, ctypes.c_void_p, ctypes.c_void_p]
    ref_t, ref_m, ref_top = _arm(lib, 0)
    dev_t, dev_m, dev_top = _arm(lib, 1, 0)
    print("reference tokens", ref_t.tolist())
    print("device tokens   ", dev_t.tolist())
    print("min margin", float(ref_m.min()))
    assert np.array_equal(ref_t, dev_t)
    assert np.max(np.abs(dev_top - ref_top) / np.abs(ref_top)) <= 1e-2


def test_greedy_32_steps_all_blocks_on_device():
    """The same 32 steps with every transformer block on the device
    (gemma3_cuda_prefill_forward / gemma3_cuda_forward: projections, norms,
    residuals, GELU MLP and attention), the host keeping only the embedding
    lookup, the final norm and the logits."""
    if not os.path.exists(SO):
        pytest.skip("e2e harness not built (needs the reference sources at build time)")
    os.environ.setdefault("OPENBLAS_NUM_THREADS", "1")
    lib = ctypes.CDLL(SO)
    lib.e2e_greedy.argtypes = [ctypes.c_int, ctypes.c_int, ctypes.c_uint64, ctypes.c_int, ctypes.c_int,
                               ctypes.c_void_p, ctypes.c_void_p, ctypes.c_void_p]
    ref_t, ref_m, ref_top = _arm(lib, 0)
    dev_t, dev_m, dev_top = _arm(lib, 2, 0)
    print("reference tokens", ref_t.tolist())
    print("device tokens   ", dev_t.tolist())
    print("min margin", float(ref_m.min()), "max top-1 rel diff",
          float(np.max(np.abs(dev_top - ref_top) / np.abs(ref_top))))
    assert np.array_equal(ref_t, dev_t)
    assert np.max(np.abs(dev_top - ref_top) / np.abs(ref_top)) <= 1e-2


def test_greedy_32_steps_token_ids_on_device():
    """Token ids in, token ids out: embedding lookup, all blocks, final norm,
    the tied-embedding logits and the greedy argmax on the device
    (gemma3_cuda_prefill_greedy / gemma3_cuda_greedy_step)."""
    if not os.path.exists(SO):
        pytest.skip("e2e harness not built (needs the reference sources at build time)")
    os.environ.setdefault("OPENBLAS_NUM_THREADS", "1")
    lib = ctypes.CDLL(SO)
    lib.e2e_greedy.argtypes = [ctypes.c_int, ctypes.c_int, ctypes.c_uint64, ctypes.c_int, ctypes.c_int,
                               ctypes.c_void_p, ctypes.c_void_p, ctypes.c_void_p]
    ref_t, ref_m, ref_top = _arm(lib, 0)
    dev_t, _, dev_top = _arm(lib, 3, 0)
    print("reference tokens", ref_t.tolist())
    print("device tokens   ", dev_t.tolist())
    print("max top-1 rel diff", float(np.max(np.abs(dev_top - ref_top) / np.abs(ref_top))))
    assert np.array_equal(ref_t, dev_t)
    assert np.max(np.abs(dev_top - ref_top) / np.abs(ref_top)) <= 1e-2


N_LONG = 1100  # > the 1024-row window: the local rings wrap


@pytest.mark.parametrize("arm", [2, 3])
def test_greedy_past_the_window(arm):
    """A 1,100-token prompt, then 32 greedy tokens, with every block on the
    device (arm 2: host embedding / final norm / logits; arm 3: token ids in
    and out).  The prompt runs through one prefill of 1,100 tokens per layer
    (local layers: 1024-row ring already wrapped by 76 rows), each generated
    token through the decode path at positions 1100..1131."""
    lib = _lib()
    ref_t, ref_m, ref_top = _arm(lib, 0, n_prompt=N_LONG)
    dev_t, _, dev_top = _arm(lib, arm, 0, n_prompt=N_LONG)
    print("reference tokens", ref_t.tolist())
    print("device tokens   ", dev_t.tolist())
    print("min margin", float(ref_m.min()), "max top-1 rel diff",
          float(np.max(np.abs(dev_top - ref_top) / np.abs(ref_top))))
    assert np.array_equal(ref_t, dev_t)
    assert np.max(np.abs(dev_top - ref_top) / np.abs(ref_top)) <= 1e-2

"""End-to-end greedy decoding on the random-init 34-layer Gemma-3-4B: the
reference's own forward pass vs the same model with the attention core on the
B200 (prompt through gemma3_cuda_attn_prefill, 32 generated tokens through
gemma3_cuda_attn_decode), and with every transformer block on the B200.  The
first 32 tokens must match; the top-1 logits of every step must agree within
1e-2 relative (the margins are logged).
Harness: oracle/e2e_harness.c (test infrastructure)."""
import ctypes
import os

import numpy as np
import pytest

pytestmark = pytest.mark.gpu
ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
SO = os.path.join(ROOT, "oracle", "_ref", "libgemma3_e2e.so")
N_PROMPT, N_STEPS = 8, 32


def _arm(lib, use_cuda, kv_dtype=0):
    toks = np.zeros(N_STEPS, np.int32)
    marg = np.zeros(N_STEPS, np.float32)
    top = np.zeros(N_STEPS, np.float32)
    rc = lib.e2e_greedy(N_PROMPT, N_STEPS, 20241, use_cuda, kv_dtype, toks.ctypes.data, marg.ctypes.data,
                        top.ctypes.data)
    assert rc == 0
    return toks, marg, top


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

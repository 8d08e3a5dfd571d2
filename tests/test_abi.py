"""The C-ABI library loads, exports exactly what include/gemma3_cuda.h
declares, and fails loudly (no fallback) where no usable GPU exists.  CPU."""
import ctypes
import subprocess

import pytest

import gemma3_cuda as gc


def test_header_symbols_exported():
    lib = gc.load_library()
    names = gc.header_functions()
    assert len(names) >= 20
    for n in names:
        assert hasattr(lib, n), n
    # the binding covers the whole header
    assert set(names) == set(gc.SIGNATURES), set(names) ^ set(gc.SIGNATURES)


def test_exported_dynamic_symbols_are_the_header():
    out = subprocess.run(["nm", "-D", "--defined-only", gc.LIB_PATH], capture_output=True, text=True).stdout
    exported = {l.split()[-1] for l in out.splitlines() if " T gemma3_cuda" in l}
    assert exported == set(gc.header_functions())


def test_config_default_and_rejection():
    lib = gc.load_library()
    cfg = gc.Config()
    lib.gemma3_cuda_config_default(ctypes.byref(cfg))
    assert (cfg.num_layers, cfg.num_heads, cfg.num_kv_heads, cfg.head_dim, cfg.sliding_window) == (34, 8, 4, 256, 1024)
    cfg.num_heads = 16  # unsupported geometry is rejected before touching a device
    assert not lib.gemma3_cuda_init(ctypes.byref(cfg))
    assert b"unsupported" in lib.gemma3_cuda_last_error()


def test_rope_helper_formula():
    import numpy as np
    t = gc.rope_table(64, 10000.0)
    i = np.arange(128)
    freq = 1.0 / np.power(10000.0, 2 * i / 256)
    ang = 63 * freq
    assert np.allclose(t[63, :, 0], np.cos(ang), atol=2e-6)
    assert np.allclose(t[63, :, 1], np.sin(ang), atol=2e-6)


def test_no_device_fails_loudly():
    try:
        import torch
        if torch.cuda.is_available():
            pytest.skip("a GPU is present")
    except ImportError:
        pass
    with pytest.raises(gc.Gemma3CudaError):
        gc.Context(max_context=128)

"""The C restatement (oracle/attn_oracle.c) pinned against the reference's
own code compiled from its sources (oracle/_ref) and against the golden
vectors in tests/golden/.  CPU only."""
import os

import numpy as np
import pytest

import synth
from oracles import PortOracle, RefOracle, rel_err, REF_SO, build_oracles

build_oracles()
have_ref = os.path.exists(REF_SO)


@pytest.fixture(scope="module")
def port():
    return PortOracle()


@pytest.fixture(scope="module")
def ref():
    if not have_ref:
        pytest.skip("reference not compiled here (oracle/_ref absent)")
    return RefOracle()


def test_slot_and_rows_semantics(port):
    L = port.lib
    assert [L.oracle_is_global_layer(i) for i in range(34)].count(1) == 5
    assert [i for i in range(34) if L.oracle_is_global_layer(i)] == [5, 11, 17, 23, 29]
    assert L.oracle_cache_slot(1, 5000) == 5000
    assert L.oracle_cache_slot(0, 5000) == 5000 % 1024
    assert L.oracle_attn_rows(0, 10) == 11 and L.oracle_attn_rows(0, 5000) == 1024
    assert L.oracle_attn_rows(1, 5000) == 5001


def test_rope_table_matches_reference(port, ref):
    """The reference's table is built under -ffast-math (Makefile:62), whose
    vectorised cosf/sinf differ from libm by up to ~2.5e-4 at large angles;
    this is why the device path uploads the host's own table bit-for-bit
    instead of computing one (gemma3_metal.h:36-38 does the same)."""
    for theta in (10000.0, 1000000.0):
        a = port.rope_table(4096, theta)
        b = ref.rope_table(4096, theta)
        assert np.max(np.abs(a - b)) < 5e-4


@pytest.mark.parametrize("is_global,T,start", [(False, 64, 0), (True, 96, 0), (False, 1100, 0)])
def test_port_matches_reference(port, ref, is_global, T, start):
    theta = 1e6 if is_global else 1e4
    rope = ref.rope_table(2048, theta)
    qn, kn = synth.qk_norm_gains(3)
    Q, K, V = synth.normal(1, (T, 2048)), synth.normal(2, (T, 1024)), synth.normal(3, (T, 1024))
    cr, cp = ref.new_cache(is_global, 2048), port.new_cache(is_global, 2048)
    a = ref.attn_core_tokens(cr, Q, K, V, qn, kn, rope, start)
    b = port.attn_core_tokens(cp, Q, K, V, qn, kn, rope, start)
    assert rel_err(b, a) < 1e-4
    kr, vr = ref.cache_arrays(cr)
    assert np.array_equal(vr, cp.v)
    assert rel_err(cp.k, kr) < 1e-5
    ref.free_cache(cr)

"""Generates tests/golden/golden.npz from the reference's own code.

Run from the repository root with the reference compiled (make -C oracle):
    python tests/golden/make_golden.py
The inputs are not stored: they are regenerated from the seeds below with
gemma3.c_b200/synth.py; only the reference's outputs are.

Cases (attention core of gemma3_transformer.c:641-692 through ref_harness.c):
  local_prefill   layer kind local,  theta 1e4, T=24 from position 0, QK-norm on
  global_decode   layer kind global, theta 1e6, 300 tokens, output of token 299 only
  local_wrap      layer kind local,  theta 1e4, 1030 tokens (ring wraps), outputs of
                  the last 6 tokens and ring slots 0..7 of V
  rope_*          rows 0, 1, 100, 1000, 8191 of gemma3_rope_precompute's table
"""
import os
import sys

import numpy as np

ROOT = os.path.dirname(os.path.dirname(os.path.dirname(os.path.abspath(__file__))))
sys.path[:0] = [os.path.join(ROOT, "gemma3.c_b200"), os.path.join(ROOT, "oracle")]
import synth  # noqa: E402
from oracles import RefOracle  # noqa: E402

CASES = {
    "local_prefill": dict(is_global=False, theta=1e4, T=24, seed=1000, gains=7, keep="all"),
    "global_decode": dict(is_global=True, theta=1e6, T=300, seed=2000, gains=8, keep="last1"),
    "local_wrap": dict(is_global=False, theta=1e4, T=1030, seed=3000, gains=9, keep="last6"),
}
ROPE_ROWS = [0, 1, 100, 1000, 8191]


def inputs(case):
    c = CASES[case]
    T, s = c["T"], c["seed"]
    Q = synth.normal(s, (T, 2048))
    K = synth.normal(s + 1, (T, 1024))
    V = synth.normal(s + 2, (T, 1024))
    qn, kn = synth.qk_norm_gains(c["gains"])
    return Q, K, V, qn, kn


def main():
    ref = RefOracle()
    out = {}
    for theta, name in ((1e4, "rope_local"), (1e6, "rope_global")):
        out[name] = ref.rope_table(8192, theta)[ROPE_ROWS]
    for case, c in CASES.items():
        Q, K, V, qn, kn = inputs(case)
        rope = ref.rope_table(2048, c["theta"])
        cache = ref.new_cache(c["is_global"], 2048)
        o = ref.attn_core_tokens(cache, Q, K, V, qn, kn, rope, 0)
        keep = {"all": o, "last1": o[-1:], "last6": o[-6:]}[c["keep"]]
        out[case] = keep.astype(np.float32)
        if case == "local_wrap":
            out[case + "_vslots"] = ref.cache_arrays(cache)[1][:8].copy()
        ref.free_cache(cache)
    np.savez_compressed(os.path.join(os.path.dirname(os.path.abspath(__file__)), "golden.npz"), **out)
    print({k: v.shape for k, v in out.items()})


if __name__ == "__main__":
    main()

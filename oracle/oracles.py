"""ctypes front-ends of the CPU checkers.

TEST INFRASTRUCTURE ONLY: imported by tests/, __graft_entry__.smoke() and
bench.py's CPU-baseline / reference legs, never by the shipped library.

  RefOracle  - the reference's own code (gemma3_kernels.c +
               gemma3_transformer.c statics), compiled by oracle/Makefile into
               oracle/_ref/libgemma3_ref.so;
  PortOracle - this repository's C restatement oracle/attn_oracle.c.

Both expose the same methods so a test can run either against the device.
"""
from __future__ import annotations

import ctypes
import os
import subprocess

import numpy as np

ORACLE = os.path.dirname(os.path.abspath(__file__))
REF_SO = os.path.join(ORACLE, "_ref", "libgemma3_ref.so")
PORT_SO = os.path.join(ORACLE, "libattn_oracle.so")

_F = ctypes.POINTER(ctypes.c_float)
_U16 = ctypes.POINTER(ctypes.c_uint16)
_P = ctypes.c_void_p
_I = ctypes.c_int

NH, NKV, HD, WINDOW = 8, 4, 256, 1024


def _fp(a):
    if a is None:
        return None
    assert a.dtype == np.float32 and a.flags["C_CONTIGUOUS"], (a.dtype, a.flags)
    return a.ctypes.data_as(_F)


def _u16(a):
    if a is None:
        return None
    return np.ascontiguousarray(a, dtype=np.uint16).ctypes.data_as(_U16)


def ref_dir():
    """The reference checkout the oracle is compiled from: $GEMMA3_REF_DIR, else
    the checkout this build was made against when it is present, else None
    (the GPU box has no reference sources; it uses the prebuilt oracle/_ref)."""
    d = os.environ.get("GEMMA3_REF_DIR") or "/root/reference"
    return d if os.path.isfile(os.path.join(d, "gemma3_kernels.c")) else None


def build_oracles():
    """Builds whatever oracle/Makefile can build here (no-op when up to date)."""
    cmd = ["make", "-s", "-C", ORACLE]
    if ref_dir():
        cmd.append("REF_DIR=" + ref_dir())
    subprocess.run(cmd, check=False, capture_output=True)


class _Cache:
    def __init__(self, is_global, max_seq):
        self.is_global = bool(is_global)
        self.rows = max_seq if is_global else WINDOW


class RefOracle:
    name = "reference"

    def __init__(self):
        if not os.path.exists(REF_SO):
            build_oracles()
        if not os.path.exists(REF_SO):
            raise FileNotFoundError(REF_SO)
        lib = ctypes.CDLL(REF_SO)
        lib.ref_layer_cache_new.restype = _P
        lib.ref_layer_cache_new.argtypes = [_I, _I]
        lib.ref_layer_cache_free.argtypes = [_P]
        lib.ref_layer_cache_k.restype = _F
        lib.ref_layer_cache_k.argtypes = [_P]
        lib.ref_layer_cache_v.restype = _F
        lib.ref_layer_cache_v.argtypes = [_P]
        lib.ref_attn_core_tokens.argtypes = [_P, _F, _F, _F, _U16, _U16, _F, _I, _I, _I, _I, _F]
        lib.ref_gqa.argtypes = [_F, _F, _F, _F, _I]
        lib.ref_layer_attention_tokens.argtypes = [_F, _F, _U16, _U16, _U16, _U16, _U16, _U16, _P, _F, _I, _I, _I, _I,
                                                   _F, _F, _F, _F]
        lib.gemma3_rope_precompute.argtypes = [_F, _I, _I, ctypes.c_float]
        lib.ref_st_num_slots.restype = _I
        lib.ref_st_load_slots.restype = _P
        lib.ref_st_load_slots.argtypes = [ctypes.c_char_p, ctypes.POINTER(_P)]
        lib.ref_st_free.argtypes = [_P]
        self.lib = lib

    def rope_table(self, max_pos, theta):
        t = np.empty((max_pos, HD // 2, 2), dtype=np.float32)
        self.lib.gemma3_rope_precompute(_fp(t), max_pos, HD, ctypes.c_float(theta))
        return t

    def new_cache(self, is_global, max_seq):
        c = _Cache(is_global, max_seq)
        c.h = self.lib.ref_layer_cache_new(int(is_global), max_seq)
        c.max_seq = max_seq
        return c

    def free_cache(self, c):
        self.lib.ref_layer_cache_free(c.h)

    def cache_arrays(self, c):
        n = c.rows * NKV * HD
        k = np.ctypeslib.as_array(self.lib.ref_layer_cache_k(c.h), shape=(n,)).reshape(c.rows, NKV, HD)
        v = np.ctypeslib.as_array(self.lib.ref_layer_cache_v(c.h), shape=(n,)).reshape(c.rows, NKV, HD)
        return k, v

    def attn_core_tokens(self, c, Q, K, V, q_norm, k_norm, rope, start_pos):
        Q = np.array(Q, dtype=np.float32, copy=True, order="C")
        K = np.array(K, dtype=np.float32, copy=True, order="C")
        V = np.array(V, dtype=np.float32, copy=True, order="C")
        T = Q.shape[0]
        out = np.zeros((T, NH * HD), dtype=np.float32)
        self.lib.ref_attn_core_tokens(c.h, _fp(Q), _fp(K), _fp(V), _u16(q_norm), _u16(k_norm), _fp(rope),
                                      int(c.is_global), T, start_pos, c.max_seq, _fp(out))
        self.last_qk = (Q, K)  # the reference normalises/rotates Q and K in place
        return out

    def load_weights(self, model_dir, shapes):
        """The reference's st_load + gemma3_load_weights on `model_dir`.
        shapes: {slot: shape} of the slots to copy out (slot numbering of
        ref_st_load_slots: 0 embed, 1 + 13 l + j layer l's j-th weight,
        1 + 13 * 34 final norm).  Returns ({slot: uint16 array}, [slots the
        loader left NULL])."""
        n = self.lib.ref_st_num_slots()
        slots = (_P * n)()
        h = self.lib.ref_st_load_slots(model_dir.encode(), slots)
        if not h:
            raise RuntimeError("reference loader failed")
        try:
            got = {}
            for i, shape in shapes.items():
                if slots[i]:
                    cnt = int(np.prod(shape))
                    buf = (ctypes.c_uint16 * cnt).from_address(slots[i])
                    got[i] = np.frombuffer(buf, dtype=np.uint16).reshape(shape).copy()
            missing = [i for i in range(n) if not slots[i]]
        finally:
            self.lib.ref_st_free(h)
        return got, missing

    def gqa(self, q, kc, vc, seq_len):
        out = np.zeros(NH * HD, dtype=np.float32)
        self.lib.ref_gqa(_fp(out), _fp(np.ascontiguousarray(q, dtype=np.float32)), _fp(kc), _fp(vc), seq_len)
        return out

    def layer_attention_tokens(self, c, x, wq, wk, wv, wo, qn, kn, rope, layer, start_pos):
        x = np.ascontiguousarray(x, dtype=np.float32)
        T = x.shape[0]
        out = np.zeros((T, 2560), dtype=np.float32)
        q = np.zeros((T, NH * HD), dtype=np.float32)
        k = np.zeros((T, NKV * HD), dtype=np.float32)
        v = np.zeros((T, NKV * HD), dtype=np.float32)
        attn = np.zeros((T, NH * HD), dtype=np.float32)
        self.lib.ref_layer_attention_tokens(_fp(out), _fp(x), _u16(wq), _u16(wk), _u16(wv), _u16(wo), _u16(qn),
                                            _u16(kn), c.h, _fp(rope), layer, T, start_pos, c.max_seq, _fp(q), _fp(k),
                                            _fp(v), _fp(attn))
        return out, q, k, v, attn


class PortOracle:
    name = "port"

    def __init__(self):
        if not os.path.exists(PORT_SO):
            build_oracles()
        lib = ctypes.CDLL(PORT_SO)
        lib.oracle_rope_table.argtypes = [_F, _I, _I, ctypes.c_float]
        lib.oracle_attn_core_tokens.argtypes = [_F, _F, _F, _F, _F, _U16, _U16, _F, _I, _I, _I, _I, _F]
        lib.oracle_gqa.argtypes = [_F, _F, _F, _F, _I, ctypes.c_float, _F]
        lib.oracle_cache_slot.argtypes = [_I, _I]
        lib.oracle_attn_rows.argtypes = [_I, _I]
        lib.oracle_is_global_layer.argtypes = [_I]
        self.lib = lib

    def rope_table(self, max_pos, theta):
        t = np.empty((max_pos, HD // 2, 2), dtype=np.float32)
        self.lib.oracle_rope_table(_fp(t), max_pos, HD, ctypes.c_float(theta))
        return t

    def new_cache(self, is_global, max_seq):
        c = _Cache(is_global, max_seq)
        c.max_seq = max_seq
        c.k = np.zeros((c.rows, NKV, HD), dtype=np.float32)
        c.v = np.zeros((c.rows, NKV, HD), dtype=np.float32)
        return c

    def free_cache(self, c):
        pass

    def cache_arrays(self, c):
        return c.k, c.v

    def attn_core_tokens(self, c, Q, K, V, q_norm, k_norm, rope, start_pos):
        Q = np.array(Q, dtype=np.float32, copy=True, order="C")
        K = np.array(K, dtype=np.float32, copy=True, order="C")
        V = np.array(V, dtype=np.float32, copy=True, order="C")
        T = Q.shape[0]
        out = np.zeros((T, NH * HD), dtype=np.float32)
        self.lib.oracle_attn_core_tokens(_fp(c.k), _fp(c.v), _fp(Q), _fp(K), _fp(V), _u16(q_norm), _u16(k_norm),
                                         _fp(rope), int(c.is_global), T, start_pos, c.max_seq, _fp(out))
        self.last_qk = (Q, K)
        return out

    def gqa(self, q, kc, vc, seq_len):
        out = np.zeros(NH * HD, dtype=np.float32)
        scores = np.zeros(seq_len, dtype=np.float32)
        self.lib.oracle_gqa(_fp(out), _fp(np.ascontiguousarray(q, dtype=np.float32)), _fp(kc), _fp(vc), seq_len,
                            ctypes.c_float(1.0 / 16.0), _fp(scores))
        return out


def best_oracle():
    """The reference's own build when present, else the restatement."""
    try:
        return RefOracle()
    except (FileNotFoundError, OSError):
        return PortOracle()


def rel_err(got, want):
    """max over tokens of  max|err| / RMS(reference output of that token).

    The unit is one row of [T][2048]: what one gemma3_gqa call of the
    reference returns (gemma3_transformer.c:689-691).  A 1-D input is one
    token.  Tolerance in the tests: 1e-2."""
    got = np.asarray(got, dtype=np.float64)
    want = np.asarray(want, dtype=np.float64)
    if want.ndim == 1:
        got, want = got[None], want[None]
    got = got.reshape(want.shape[0], -1)
    want = want.reshape(want.shape[0], -1)
    rms = np.sqrt(np.mean(want * want, axis=1))
    err = np.max(np.abs(got - want), axis=1)
    return float(np.max(err / np.maximum(rms, 1e-30)))


def bf16_round(x):
    """fp32 -> nearest-even bf16 -> fp32 (what the device stores)."""
    x = np.ascontiguousarray(x, dtype=np.float32)
    u = x.view(np.uint32).astype(np.uint64)
    u = ((u + 0x7FFF + ((u >> 16) & 1)) >> 16) << 16
    return u.astype(np.uint32).view(np.float32)


def exact_attention(Qn, Kn, V, start_pos, is_global, kv_round=None, kv_prefix=None):
    """float64 torch attention of the reference's semantics (causal, 1024
    window on local layers, scale 1/16) over the normalised+rotated Qn/Kn
    the reference produced.  kv_round='bf16' stores K/V rows as a bf16 cache
    holds them (round-to-nearest-even): the reference's semantics on a BF16
    cache.  kv_prefix = (K, V) rows for positions [0, start_pos) or None."""
    import torch
    T = Qn.shape[0]
    Kall, Vall = Kn, V
    if kv_prefix is not None:
        Kall = np.concatenate([kv_prefix[0], Kn])
        Vall = np.concatenate([kv_prefix[1], V])
    if kv_round == "bf16":
        Kall, Vall = bf16_round(Kall), bf16_round(Vall)
    q = torch.from_numpy(np.ascontiguousarray(Qn, dtype=np.float32).reshape(T, NH, HD)).double()
    k = torch.from_numpy(np.ascontiguousarray(Kall, dtype=np.float32).reshape(-1, NKV, HD)).double()
    v = torch.from_numpy(np.ascontiguousarray(Vall, dtype=np.float32).reshape(-1, NKV, HD)).double()
    L = k.shape[0]
    qpos = torch.arange(start_pos, start_pos + T)[:, None]
    kpos = torch.arange(0, L)[None, :]
    ok = kpos <= qpos
    if not is_global:
        ok &= kpos > qpos - WINDOW
    out = torch.empty(T, NH, HD, dtype=torch.float64)
    for h in range(NH):
        s = (q[:, h] @ k[:, h // 2].T) / 16.0
        s = s.masked_fill(~ok, float("-inf"))
        out[:, h] = torch.softmax(s, dim=1) @ v[:, h // 2]
    return out.reshape(T, NH * HD).float().numpy()

"""ctypes binding of libgemma3_cuda.so (the C-ABI in include/gemma3_cuda.h).

This is the same binding a Python caller of gemma3.c would add; the C host
(gemma3_transformer.c under USE_CUDA) calls the identical entry points
directly.  Every method maps 1:1 onto one C entry point and raises
Gemma3CudaError (carrying the C return code, whose values are the
reference's gemma3_error codes, gemma3.h:57-67) when it fails.  There is no
fallback of any kind: if the shared library is missing, importing the
binding's loader raises.
"""
from __future__ import annotations

import ctypes
import os
import re

import numpy as np

HERE = os.path.dirname(os.path.abspath(__file__))
LIB_PATH = os.path.join(HERE, "libgemma3_cuda.so")
HEADER_PATH = os.path.join(os.path.dirname(HERE), "include", "gemma3_cuda.h")

OK = 0
ERR_INVALID_ARG = -1
ERR_OUT_OF_MEMORY = -4
ERR_GENERATION_FAILED = -7
ERR_CONTEXT_OVERFLOW = -8

KV_F32 = 0
KV_BF16 = 1
XCHG_NCCL = 0
XCHG_PEER = 1

N_LAYERS = 34
N_HEADS = 8
N_KV = 4
HEAD_DIM = 256
WINDOW = 1024
Q_SIZE = N_HEADS * HEAD_DIM
KV_SIZE = N_KV * HEAD_DIM
HIDDEN = 2560  # Gemma 3 4B hidden size (gemma3.h)
PARTIAL_STRIDE = HEAD_DIM + 2


def is_global_layer(layer: int) -> bool:
    """gemma3.h:347-350: layers 5, 11, 17, 23, 29 are global."""
    return (layer + 1) % 6 == 0


class Gemma3CudaError(RuntimeError):
    def __init__(self, code: int, msg: str):
        super().__init__(f"gemma3_cuda error {code}: {msg}")
        self.code = code


class Config(ctypes.Structure):
    _fields_ = [
        ("num_layers", ctypes.c_int),
        ("num_heads", ctypes.c_int),
        ("num_kv_heads", ctypes.c_int),
        ("head_dim", ctypes.c_int),
        ("sliding_window", ctypes.c_int),
        ("rmsnorm_eps", ctypes.c_float),
        ("max_context", ctypes.c_int),
        ("max_batch", ctypes.c_int),
        ("kv_dtype", ctypes.c_int),
        ("device", ctypes.c_int),
        ("max_prefill", ctypes.c_int),
        ("kv_rank", ctypes.c_int),
        ("kv_ranks", ctypes.c_int),
    ]


_P = ctypes.c_void_p
_I = ctypes.c_int
_FP = ctypes.POINTER(ctypes.c_float)
_IP = ctypes.POINTER(ctypes.c_int)
_U16P = ctypes.POINTER(ctypes.c_uint16)

# name -> (restype, argtypes); must cover every function in the header.
class LayerWeights(ctypes.Structure):
    """gemma3_cuda_layer_weights: BF16 (uint16) arrays as gemma3_layer_weights holds them."""
    _fields_ = [(n, ctypes.c_void_p) for n in (
        "input_layernorm", "q_proj", "k_proj", "v_proj", "o_proj", "q_norm", "k_norm",
        "post_attention_layernorm", "gate_proj", "up_proj", "down_proj",
        "pre_feedforward_layernorm", "post_feedforward_layernorm")]


SIGNATURES = {
    "gemma3_cuda_config_default": (None, [ctypes.POINTER(Config)]),
    "gemma3_cuda_init": (_P, [ctypes.POINTER(Config)]),
    "gemma3_cuda_free": (None, [_P]),
    "gemma3_cuda_upload_rope": (_I, [_P, _FP, _FP, _I, _I]),
    "gemma3_cuda_rope_precompute": (None, [_FP, _I, _I, ctypes.c_float]),
    "gemma3_cuda_set_qk_norm": (_I, [_P, _I, _U16P, _U16P]),
    "gemma3_cuda_attn_prefill": (_I, [_P, _I, _I, _FP, _FP, _FP, _I, _I, _FP]),
    "gemma3_cuda_attn_prefill_dev": (_I, [_P, _I, _I, _P, _P, _P, _I, _I, _P]),
    "gemma3_cuda_attn_decode": (_I, [_P, _I, _I, _IP, _IP, _FP, _FP, _FP, _FP]),
    "gemma3_cuda_peer_init": (_I, [_P]),
    "gemma3_cuda_set_exchange": (_I, [_P, _I]),
    "gemma3_cuda_attn_decode_dev": (_I, [_P, _I, _I, _IP, _IP, _P, _P, _P, _P]),
    "gemma3_cuda_attn_decode_partial_dev": (_I, [_P, _I, _I, _IP, _IP, _P, _P, _P, _P]),
    "gemma3_cuda_merge_partials_dev": (_I, [_P, _I, _I, _P, _P]),
    "gemma3_cuda_attn_prefill_partial_dev": (_I, [_P, _I, _I, _P, _P, _P, _I, _I, _P, _P]),
    "gemma3_cuda_merge_prefill_partials_dev": (_I, [_P, _I, _I, _P, _P, _P]),
    "gemma3_cuda_comm_unique_id": (_I, [ctypes.c_char_p]),
    "gemma3_cuda_comm_init": (_I, [_P, ctypes.c_char_p]),
    "gemma3_cuda_reset": (_I, [_P]),
    "gemma3_cuda_export_cache": (_I, [_P, _I, _I, _FP, _FP]),
    "gemma3_cuda_import_cache": (_I, [_P, _I, _I, _FP, _FP, _I]),
    "gemma3_cuda_fill_cache_random": (_I, [_P, _I, _I, _I, ctypes.c_uint64]),
    "gemma3_cuda_stream": (_P, [_P]),
    "gemma3_cuda_synchronize": (_I, [_P]),
    "gemma3_cuda_launch_count": (ctypes.c_longlong, [_P]),
    "gemma3_cuda_profile": (_I, [_P, _I]),
    "gemma3_cuda_profile_read": (_I, [_P, _I, ctypes.POINTER(ctypes.c_longlong), ctypes.POINTER(ctypes.c_double),
                                      ctypes.POINTER(ctypes.c_double)]),
    "gemma3_cuda_gqa_decode_noalloc": (_I, [_P, _P, _I, _I, _I, _IP, _P, _P]),
    "gemma3_cuda_selftest_wait_timeout": (_I, [_P]),
    "gemma3_cuda_set_proj_weights": (_I, [_P, _I, _U16P, _U16P, _U16P, _U16P]),
    "gemma3_cuda_project_qkv_dev": (_I, [_P, _I, _I, _P, _P, _P, _P]),
    "gemma3_cuda_project_o_dev": (_I, [_P, _I, _I, _P, _P]),
    "gemma3_cuda_layer_decode": (_I, [_P, _I, _I, _IP, _IP, _FP, _FP]),
    "gemma3_cuda_layer_decode_dev": (_I, [_P, _I, _I, _IP, _IP, _P, _P]),
    "gemma3_cuda_layer_prefill": (_I, [_P, _I, _I, _FP, _I, _I, _FP]),
    "gemma3_cuda_layer_prefill_dev": (_I, [_P, _I, _I, _P, _I, _I, _P]),
    "gemma3_cuda_set_layer_weights": (_I, [_P, _I, ctypes.POINTER(LayerWeights)]),
    "gemma3_cuda_forward": (_I, [_P, _I, _IP, _IP, _FP]),
    "gemma3_cuda_forward_dev": (_I, [_P, _I, _IP, _IP, _P]),
    "gemma3_cuda_prefill_forward": (_I, [_P, _I, _FP, _I, _I]),
    "gemma3_cuda_prefill_forward_dev": (_I, [_P, _I, _P, _I, _I]),
    "gemma3_cuda_set_embeddings": (_I, [_P, _U16P, _I, _U16P]),
    "gemma3_cuda_prefill_greedy": (_I, [_P, _I, _IP, _I, _I, _IP, _FP]),
    "gemma3_cuda_greedy_step": (_I, [_P, _I, _IP, _IP, _IP, _IP, _FP]),
    "gemma3_cuda_safetensors_check": (_I, [ctypes.c_char_p, _I, _IP]),
    "gemma3_cuda_load_safetensors": (_I, [_P, ctypes.c_char_p]),
    "gemma3_cuda_last_error": (ctypes.c_char_p, []),
}

_lib = None


def header_functions(path: str = HEADER_PATH) -> list[str]:
    """Names of every function the C header declares."""
    text = open(path).read()
    return sorted(set(re.findall(r"\b(gemma3_cuda_[a-z0-9_]+)\s*\(", text)))


def load_library(path: str = LIB_PATH):
    """Loads libgemma3_cuda.so; raises if it is absent (no fallback)."""
    global _lib
    if _lib is not None:
        return _lib
    if not os.path.exists(path):
        raise OSError(f"{path} not built: run `make -C gemma3.c_b200 cuda` (no CPU fallback exists)")
    lib = ctypes.CDLL(path)
    for name, (res, args) in SIGNATURES.items():
        fn = getattr(lib, name)
        fn.restype = res
        fn.argtypes = args
    _lib = lib
    return lib


def _fptr(a: np.ndarray):
    assert a.dtype == np.float32 and a.flags["C_CONTIGUOUS"]
    return a.ctypes.data_as(_FP)


def _iarr(xs):
    a = np.ascontiguousarray(np.asarray(xs, dtype=np.int32))
    return a, a.ctypes.data_as(_IP)


def safetensors_check(model_dir: str, num_layers: int = N_LAYERS) -> int:
    """Host-only check of a checkpoint directory; returns the vocabulary size,
    raises Gemma3CudaError with the reason otherwise."""
    lib = load_library()
    v = np.zeros(1, np.int32)
    rc = lib.gemma3_cuda_safetensors_check(model_dir.encode(), num_layers, v.ctypes.data_as(_IP))
    if rc != 0:
        raise Gemma3CudaError(rc, (lib.gemma3_cuda_last_error() or b"").decode())
    return int(v[0])


def rope_table(max_pos: int, theta: float) -> np.ndarray:
    """RoPE cos/sin table [max_pos][128][2] built by the library's host helper
    (formula of gemma3_rope_precompute, gemma3_kernels.c:455-468)."""
    lib = load_library()
    t = np.empty((max_pos, HEAD_DIM // 2, 2), dtype=np.float32)
    lib.gemma3_cuda_rope_precompute(_fptr(t), max_pos, HEAD_DIM, ctypes.c_float(theta))
    return t


def gqa_decode_noalloc(q_ptr: int, kv_ptr: int, kv_dtype: int, rows: int, nrows, out_ptr: int, stream: int = 0):
    """gemma3_cuda_gqa_decode_noalloc: decode over a caller-owned device cache
    [B][K,V][4][rows][256] with no device allocation (scratch is a static
    device array).  Enqueues on `stream`."""
    lib = load_library()
    a, ap = _iarr(nrows)
    rc = lib.gemma3_cuda_gqa_decode_noalloc(q_ptr, kv_ptr, kv_dtype, rows, len(a), ap, out_ptr, stream or None)
    if rc != 0:
        raise Gemma3CudaError(rc, (lib.gemma3_cuda_last_error() or b"").decode())


class Context:
    """One device context (one GPU, one stream, the device KV cache)."""

    def __init__(self, max_context=8192, max_batch=1, kv_dtype=KV_F32, device=0, max_prefill=None,
                 kv_rank=0, kv_ranks=1, num_layers=N_LAYERS):
        lib = load_library()
        self.lib = lib
        cfg = Config()
        lib.gemma3_cuda_config_default(ctypes.byref(cfg))
        cfg.num_layers = num_layers
        cfg.max_context = max_context
        cfg.max_batch = max_batch
        cfg.kv_dtype = kv_dtype
        cfg.device = device
        cfg.max_prefill = max_prefill if max_prefill is not None else min(max_context, 8192)
        cfg.kv_rank = kv_rank
        cfg.kv_ranks = kv_ranks
        self.cfg = cfg
        h = lib.gemma3_cuda_init(ctypes.byref(cfg))
        if not h:
            raise Gemma3CudaError(ERR_GENERATION_FAILED, self.last_error())
        self.h = h

    # -- plumbing ---------------------------------------------------------
    def last_error(self) -> str:
        return (self.lib.gemma3_cuda_last_error() or b"").decode()

    def _chk(self, rc):
        if rc != 0:
            raise Gemma3CudaError(rc, self.last_error())

    def close(self):
        if getattr(self, "h", None):
            self.lib.gemma3_cuda_free(self.h)
            self.h = None

    def __del__(self):
        try:
            self.close()
        except Exception:
            pass

    @property
    def stream(self) -> int:
        return self.lib.gemma3_cuda_stream(self.h) or 0

    def synchronize(self):
        self._chk(self.lib.gemma3_cuda_synchronize(self.h))

    def launch_count(self) -> int:
        return int(self.lib.gemma3_cuda_launch_count(self.h))

    def selftest_wait_timeout(self) -> int:
        """Runs the bounded-wait failure path; returns the C return code."""
        return self.lib.gemma3_cuda_selftest_wait_timeout(self.h)

    def profile(self, enable: bool):
        self._chk(self.lib.gemma3_cuda_profile(self.h, int(enable)))

    def profile_read(self, kernel: int):
        """(launches, device ms, algorithmic work) of kernel 0 (decode) / 1 (prefill)."""
        n, ms, w = ctypes.c_longlong(), ctypes.c_double(), ctypes.c_double()
        self._chk(self.lib.gemma3_cuda_profile_read(self.h, kernel, ctypes.byref(n), ctypes.byref(ms), ctypes.byref(w)))
        return n.value, ms.value, w.value

    # -- model set-up -----------------------------------------------------
    def upload_rope(self, rope_local: np.ndarray, rope_global: np.ndarray):
        rl = np.ascontiguousarray(rope_local, dtype=np.float32)
        rg = np.ascontiguousarray(rope_global, dtype=np.float32)
        self._chk(self.lib.gemma3_cuda_upload_rope(self.h, _fptr(rl), _fptr(rg), rl.shape[0], HEAD_DIM))

    def set_qk_norm(self, layer: int, q_norm, k_norm):
        if q_norm is None or k_norm is None:
            self._chk(self.lib.gemma3_cuda_set_qk_norm(self.h, layer, None, None))
            return
        qn = np.ascontiguousarray(q_norm, dtype=np.uint16)
        kn = np.ascontiguousarray(k_norm, dtype=np.uint16)
        self._chk(self.lib.gemma3_cuda_set_qk_norm(self.h, layer, qn.ctypes.data_as(_U16P), kn.ctypes.data_as(_U16P)))

    # -- hot path (host buffers) ------------------------------------------
    def attn_prefill(self, layer, seq, Q, K, V, start_pos, out=None):
        Q = np.ascontiguousarray(Q, dtype=np.float32)
        K = np.ascontiguousarray(K, dtype=np.float32)
        V = np.ascontiguousarray(V, dtype=np.float32)
        T = Q.shape[0]
        if out is None:
            out = np.empty((T, Q_SIZE), dtype=np.float32)
        self._chk(self.lib.gemma3_cuda_attn_prefill(self.h, layer, seq, _fptr(Q), _fptr(K), _fptr(V), T, start_pos,
                                                    _fptr(out)))
        return out

    def attn_decode(self, layer, seq_ids, pos, Q, K, V, out=None):
        Q = np.ascontiguousarray(Q, dtype=np.float32)
        K = np.ascontiguousarray(K, dtype=np.float32)
        V = np.ascontiguousarray(V, dtype=np.float32)
        B = len(seq_ids)
        s, sp = _iarr(seq_ids)
        p, pp = _iarr(pos)
        if out is None:
            out = np.empty((B, Q_SIZE), dtype=np.float32)
        self._chk(self.lib.gemma3_cuda_attn_decode(self.h, layer, B, sp, pp, _fptr(Q), _fptr(K), _fptr(V), _fptr(out)))
        return out

    # -- projections and whole-layer attention ----------------------------
    def set_proj_weights(self, layer: int, wq, wk, wv, wo):
        """BF16 (uint16) [2048][2560], [1024][2560], [1024][2560], [2560][2048]."""
        ws = [np.ascontiguousarray(w, dtype=np.uint16) for w in (wq, wk, wv, wo)]
        shapes = [(Q_SIZE, HIDDEN), (KV_SIZE, HIDDEN), (KV_SIZE, HIDDEN), (HIDDEN, Q_SIZE)]
        for w, shp in zip(ws, shapes):
            if w.shape != shp:
                raise ValueError(f"weight shape {w.shape}, expected {shp}")
        self._chk(self.lib.gemma3_cuda_set_proj_weights(self.h, layer, *[w.ctypes.data_as(_U16P) for w in ws]))

    def project_qkv_dev(self, layer, T, x_ptr, q_ptr, k_ptr, v_ptr):
        self._chk(self.lib.gemma3_cuda_project_qkv_dev(self.h, layer, T, x_ptr, q_ptr, k_ptr, v_ptr))

    def project_o_dev(self, layer, T, attn_ptr, out_ptr):
        self._chk(self.lib.gemma3_cuda_project_o_dev(self.h, layer, T, attn_ptr, out_ptr))

    def layer_decode(self, layer, seq_ids, pos, x, out=None):
        x = np.ascontiguousarray(x, dtype=np.float32)
        B = len(seq_ids)
        s, sp = _iarr(seq_ids)
        p, pp = _iarr(pos)
        if out is None:
            out = np.empty((B, HIDDEN), dtype=np.float32)
        self._chk(self.lib.gemma3_cuda_layer_decode(self.h, layer, B, sp, pp, _fptr(x), _fptr(out)))
        return out

    def layer_decode_dev(self, layer, seq_ids, pos, x_ptr, out_ptr):
        s, sp = _iarr(seq_ids)
        p, pp = _iarr(pos)
        self._chk(self.lib.gemma3_cuda_layer_decode_dev(self.h, layer, len(s), sp, pp, x_ptr, out_ptr))

    def layer_prefill(self, layer, seq, x, start_pos, out=None):
        x = np.ascontiguousarray(x, dtype=np.float32)
        T = x.shape[0]
        if out is None:
            out = np.empty((T, HIDDEN), dtype=np.float32)
        self._chk(self.lib.gemma3_cuda_layer_prefill(self.h, layer, seq, _fptr(x), T, start_pos, _fptr(out)))
        return out

    def layer_prefill_dev(self, layer, seq, x_ptr, T, start_pos, out_ptr):
        self._chk(self.lib.gemma3_cuda_layer_prefill_dev(self.h, layer, seq, x_ptr, T, start_pos, out_ptr))

    # -- whole transformer blocks ---------------------------------------------
    def set_layer_weights(self, layer: int, **w):
        """BF16 (uint16) arrays keyed by LayerWeights field name; the three
        optional norms may be omitted or None."""
        keep = {k: np.ascontiguousarray(v, dtype=np.uint16) for k, v in w.items() if v is not None}
        lw = LayerWeights(**{k: v.ctypes.data for k, v in keep.items()})
        self._chk(self.lib.gemma3_cuda_set_layer_weights(self.h, layer, ctypes.byref(lw)))

    def forward(self, seq_ids, pos, x):
        """x [B][2560] fp32 residual stream, updated in place (returned)."""
        x = np.ascontiguousarray(x, dtype=np.float32)
        s, sp = _iarr(seq_ids)
        p, pp = _iarr(pos)
        self._chk(self.lib.gemma3_cuda_forward(self.h, len(s), sp, pp, _fptr(x)))
        return x

    def prefill_forward(self, seq, x, start_pos):
        x = np.ascontiguousarray(x, dtype=np.float32)
        self._chk(self.lib.gemma3_cuda_prefill_forward(self.h, seq, _fptr(x), x.shape[0], start_pos))
        return x

    def forward_dev(self, seq_ids, pos, x_ptr):
        s, sp = _iarr(seq_ids)
        p, pp = _iarr(pos)
        self._chk(self.lib.gemma3_cuda_forward_dev(self.h, len(s), sp, pp, x_ptr))

    def prefill_forward_dev(self, seq, x_ptr, T, start_pos):
        self._chk(self.lib.gemma3_cuda_prefill_forward_dev(self.h, seq, x_ptr, T, start_pos))

    # -- checkpoints -----------------------------------------------------------
    def load_safetensors(self, model_dir: str):
        self._chk(self.lib.gemma3_cuda_load_safetensors(self.h, model_dir.encode()))

    # -- greedy decoding ------------------------------------------------------
    def set_embeddings(self, embed, final_norm):
        e = np.ascontiguousarray(embed, dtype=np.uint16)
        n = np.ascontiguousarray(final_norm, dtype=np.uint16)
        self._chk(self.lib.gemma3_cuda_set_embeddings(self.h, e.ctypes.data_as(_U16P), e.shape[0],
                                                      n.ctypes.data_as(_U16P)))

    def prefill_greedy(self, seq, tokens, start_pos):
        t, tp = _iarr(tokens)
        nxt = np.zeros(1, np.int32)
        top = np.zeros(1, np.float32)
        self._chk(self.lib.gemma3_cuda_prefill_greedy(self.h, seq, tp, len(t), start_pos,
                                                      nxt.ctypes.data_as(_IP), _fptr(top)))
        return int(nxt[0]), float(top[0])

    def greedy_step(self, seq_ids, pos, tokens):
        s, sp = _iarr(seq_ids)
        p, pp = _iarr(pos)
        t, tp = _iarr(tokens)
        nxt = np.zeros(len(s), np.int32)
        top = np.zeros(len(s), np.float32)
        self._chk(self.lib.gemma3_cuda_greedy_step(self.h, len(s), sp, pp, tp, nxt.ctypes.data_as(_IP), _fptr(top)))
        return nxt, top

    # -- hot path (device pointers, enqueue only) -------------------------
    def attn_prefill_dev(self, layer, seq, q_ptr, k_ptr, v_ptr, T, start_pos, out_ptr):
        self._chk(self.lib.gemma3_cuda_attn_prefill_dev(self.h, layer, seq, q_ptr, k_ptr, v_ptr, T, start_pos, out_ptr))

    def attn_decode_dev(self, layer, seq_ids, pos, q_ptr, k_ptr, v_ptr, out_ptr):
        s, sp = _iarr(seq_ids)
        p, pp = _iarr(pos)
        self._chk(self.lib.gemma3_cuda_attn_decode_dev(self.h, layer, len(s), sp, pp, q_ptr, k_ptr, v_ptr, out_ptr))

    def attn_decode_partial_dev(self, layer, seq_ids, pos, q_ptr, k_ptr, v_ptr, partial_ptr):
        s, sp = _iarr(seq_ids)
        p, pp = _iarr(pos)
        self._chk(self.lib.gemma3_cuda_attn_decode_partial_dev(self.h, layer, len(s), sp, pp, q_ptr, k_ptr, v_ptr,
                                                               partial_ptr))

    def attn_prefill_partial_dev(self, layer, seq, q_ptr, k_ptr, v_ptr, T, start_pos, out_ptr, ml_ptr):
        """This rank's share of a context-parallel global-layer prefill:
        out [T][2048] over its keys, ml [T][8][2] (m, l) per row."""
        self._chk(self.lib.gemma3_cuda_attn_prefill_partial_dev(self.h, layer, seq, q_ptr, k_ptr, v_ptr, T, start_pos,
                                                                out_ptr, ml_ptr))

    def merge_prefill_partials_dev(self, n_parts, T, outs_ptr, mls_ptr, out_ptr):
        self._chk(self.lib.gemma3_cuda_merge_prefill_partials_dev(self.h, n_parts, T, outs_ptr, mls_ptr, out_ptr))

    def merge_partials_dev(self, n_parts, B, partials_ptr, out_ptr):
        self._chk(self.lib.gemma3_cuda_merge_partials_dev(self.h, n_parts, B, partials_ptr, out_ptr))

    # -- multi-GPU ----------------------------------------------------------
    @staticmethod
    def comm_unique_id() -> bytes:
        lib = load_library()
        buf = ctypes.create_string_buffer(128)
        rc = lib.gemma3_cuda_comm_unique_id(buf)
        if rc != 0:
            raise Gemma3CudaError(rc, (lib.gemma3_cuda_last_error() or b"").decode())
        return buf.raw

    def comm_init(self, uid: bytes):
        assert len(uid) == 128
        self._chk(self.lib.gemma3_cuda_comm_init(self.h, ctypes.create_string_buffer(uid, 128)))

    def peer_init(self):
        """Maps every rank's receive buffer for the peer-memory exchange
        (collective over the kv_ranks contexts, after comm_init)."""
        self._chk(self.lib.gemma3_cuda_peer_init(self.h))

    def set_exchange(self, mode: int):
        """XCHG_NCCL (all-gather) or XCHG_PEER (NVLink stores + flags)."""
        self._chk(self.lib.gemma3_cuda_set_exchange(self.h, mode))

    # -- cache utilities ----------------------------------------------------
    def cache_rows(self, layer: int) -> int:
        if is_global_layer(layer):
            S = -(-self.cfg.max_context // self.cfg.kv_ranks)
            lo = min(self.cfg.max_context, self.cfg.kv_rank * S)
            return max(1, min(self.cfg.max_context, lo + S) - lo)
        return WINDOW

    def reset(self):
        self._chk(self.lib.gemma3_cuda_reset(self.h))

    def export_cache(self, layer, seq):
        rows = self.cache_rows(layer)
        k = np.empty((rows, N_KV, HEAD_DIM), dtype=np.float32)
        v = np.empty_like(k)
        self._chk(self.lib.gemma3_cuda_export_cache(self.h, layer, seq, _fptr(k), _fptr(v)))
        return k, v

    def import_cache(self, layer, seq, k, v):
        k = np.ascontiguousarray(k, dtype=np.float32)
        v = np.ascontiguousarray(v, dtype=np.float32)
        self._chk(self.lib.gemma3_cuda_import_cache(self.h, layer, seq, _fptr(k), _fptr(v), k.shape[0]))

    def fill_cache_random(self, layer, seq, rows, seed):
        self._chk(self.lib.gemma3_cuda_fill_cache_random(self.h, layer, seq, rows, ctypes.c_uint64(seed)))

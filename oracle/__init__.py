"""ctypes front end of the CPU oracle -- TEST INFRASTRUCTURE ONLY.

Loaded by tests/, __graft_entry__.smoke() and bench.py's CPU baseline, never by
the product. See oracle.h for what is restated from which reference file:line.
"""
from __future__ import annotations

import ctypes
import os
import subprocess
from typing import Optional

import numpy as np

HERE = os.path.dirname(os.path.abspath(__file__))
LIB_PATH = os.path.join(HERE, "liboracle.so")
REF_LIB_PATH = os.path.join(HERE, "_ref", "libref_host.so")

MODE_FP32 = 0
MODE_BF16 = 1
MODE_BF16_REORDERED = 2
MODE_FP32_KV_BF16 = 3


def json_include() -> str:
    """A directory holding nlohmann/json.hpp (the single-header library the
    reference pins, v3.11): the copy vendored with cudnn_frontend in this
    Python environment."""
    import sysconfig

    return os.path.join(sysconfig.get_paths()["purelib"], "include", "cudnn_frontend", "thirdparty")


def build(ref_dir: Optional[str] = None) -> None:
    """Builds liblcr oracle; with `ref_dir` (a reference checkout) also the
    reference's own host code into _ref/."""
    subprocess.run(["make", "-s", "-C", HERE], check=True)
    if ref_dir and os.path.isdir(os.path.join(ref_dir, "src")):
        subprocess.run(["make", "-s", "-C", HERE, "ref", f"REF={ref_dir}", f"JSON_INC={json_include()}"],
                       check=True)


class _Config(ctypes.Structure):
    _fields_ = [
        ("hidden", ctypes.c_int), ("ffn", ctypes.c_int), ("layers", ctypes.c_int),
        ("heads", ctypes.c_int), ("kv_heads", ctypes.c_int), ("head_dim", ctypes.c_int),
        ("vocab", ctypes.c_int), ("eps", ctypes.c_float), ("theta", ctypes.c_float),
        ("rope_scaling", ctypes.c_int), ("rope_factor", ctypes.c_float),
        ("rope_low", ctypes.c_float), ("rope_high", ctypes.c_float),
        ("rope_orig_ctx", ctypes.c_int),
    ]


_P = ctypes.POINTER
_u16p = _P(ctypes.c_uint16)
_f32p = _P(ctypes.c_float)


class _Weights(ctypes.Structure):
    _fields_ = [
        ("embed", _u16p), ("final_norm", _u16p), ("lm_head", _u16p),
        ("input_norm", _P(_u16p)), ("qkv", _P(_u16p)), ("o", _P(_u16p)),
        ("post_norm", _P(_u16p)), ("gate_up", _P(_u16p)), ("down", _P(_u16p)),
    ]


_lib: Optional[ctypes.CDLL] = None


def lib() -> ctypes.CDLL:
    global _lib
    if _lib is None:
        if not os.path.exists(LIB_PATH):
            build()
        L = ctypes.CDLL(LIB_PATH)
        L.orc_state_new.restype = ctypes.c_void_p
        L.orc_state_new.argtypes = [_P(_Config), ctypes.c_int]
        L.orc_state_free.argtypes = [ctypes.c_void_p]
        L.orc_state_reset.argtypes = [ctypes.c_void_p]
        L.orc_decode.restype = ctypes.c_int
        L.orc_decode.argtypes = [_P(_Config), _P(_Weights), ctypes.c_void_p, ctypes.c_int,
                                 ctypes.c_int, ctypes.c_int, _f32p, _f32p]
        L.orc_rope_inv_freq.argtypes = [_P(_Config), _f32p]
        L.orc_weight_bytes_per_token.restype = ctypes.c_size_t
        L.orc_weight_bytes_per_token.argtypes = [_P(_Config)]
        L.orc_argmax.restype = ctypes.c_int
        L.orc_argmax.argtypes = [_f32p, ctypes.c_int]
        L.orc_det_expf.restype = ctypes.c_float
        L.orc_det_expf.argtypes = [ctypes.c_float]
        L.orc_philox4x32_10.argtypes = [_P(ctypes.c_uint32), _P(ctypes.c_uint32), _P(ctypes.c_uint32)]
        L.orc_philox_uniform.restype = ctypes.c_float
        L.orc_philox_uniform.argtypes = [ctypes.c_uint64, ctypes.c_uint64, ctypes.c_uint32]
        L.orc_tree_sum_1024.restype = ctypes.c_float
        L.orc_tree_sum_1024.argtypes = [_f32p, ctypes.c_int]
        L.orc_sample.restype = ctypes.c_int
        L.orc_sample.argtypes = [_f32p, ctypes.c_int, ctypes.c_float, ctypes.c_int,
                                 ctypes.c_float, ctypes.c_float]
        L.orc_paged_reserve.restype = ctypes.c_int
        L.orc_paged_reserve.argtypes = [_P(ctypes.c_int32), ctypes.c_int, ctypes.c_int, ctypes.c_int,
                                        ctypes.c_int, ctypes.c_int, ctypes.c_int, ctypes.c_int,
                                        _P(ctypes.c_int32)]
        L.orc_page_permutation.argtypes = [_P(ctypes.c_int32), ctypes.c_int, ctypes.c_uint64]
        L.orc_rmsnorm.argtypes = [_f32p, _u16p, _u16p, ctypes.c_int, ctypes.c_int, ctypes.c_float, ctypes.c_int]
        L.orc_add_residual_rmsnorm.argtypes = [_f32p, _u16p, _u16p, _u16p, ctypes.c_int, ctypes.c_int, ctypes.c_float]
        L.orc_swiglu.argtypes = [_f32p, _u16p, _u16p, ctypes.c_long]
        L.orc_rope_rows.argtypes = [_f32p, _u16p, _f32p, ctypes.c_int, ctypes.c_int, ctypes.c_int,
                                    ctypes.c_int, ctypes.c_int, ctypes.c_int]
        L.orc_attention.argtypes = [_f32p, _u16p, _u16p, _u16p, ctypes.c_int, ctypes.c_int,
                                    ctypes.c_int, ctypes.c_int, ctypes.c_float]
        L.orc_gemv.argtypes = [_f32p, _u16p, _u16p, ctypes.c_int, ctypes.c_int]
        L.orc_set_threads.argtypes = [ctypes.c_int]
        L.orc_prefill.restype = ctypes.c_int
        L.orc_prefill.argtypes = [_P(_Config), _P(_Weights), ctypes.c_void_p, _P(ctypes.c_int32),
                                  ctypes.c_int, ctypes.c_int, ctypes.c_int, _f32p]
        _lib = L
    return _lib


def _ptr(a: np.ndarray, ct):
    assert a.flags["C_CONTIGUOUS"]
    return a.ctypes.data_as(_P(ct))


def config_of(geom) -> _Config:
    return _Config(geom.hidden_size, geom.intermediate_size, geom.num_layers, geom.num_heads,
                   geom.num_kv_heads, geom.head_dim, geom.vocab_size, geom.rms_norm_eps,
                   geom.rope_theta, int(geom.rope_scaling), geom.rope_factor,
                   geom.rope_low_freq_factor, geom.rope_high_freq_factor,
                   geom.rope_original_max_position_embeddings)


def rope_inv_freq(geom) -> np.ndarray:
    out = np.zeros(geom.head_dim // 2, dtype=np.float32)
    c = config_of(geom)
    lib().orc_rope_inv_freq(ctypes.byref(c), _ptr(out, ctypes.c_float))
    return out


class Model:
    """The fp32 host evaluation of one sequence (contiguous KV, like
    src/kv_cache.cu:104-119)."""

    def __init__(self, block, max_seq: int):
        self.block = block
        self.geom = block.geom
        self.cfg = config_of(self.geom)
        L = lib()
        g = self.geom
        base = block.data.ctypes.data

        def p(name):
            return ctypes.cast(base + block.offsets[name][0] * 2, _u16p)

        n = g.num_layers
        arr = lambda suffix: (_u16p * n)(*[p(f"layers.{l}.{suffix}") for l in range(n)])
        self._keep = [arr(s) for s in ("input_norm", "qkv", "o", "post_norm", "gate_up", "down")]
        self.w = _Weights(p("embed"), p("final_norm"), p(block.lm_head_group), *self._keep)
        self.state = L.orc_state_new(ctypes.byref(self.cfg), max_seq)
        self.max_seq = max_seq

    def __del__(self):
        try:
            lib().orc_state_free(self.state)
        except Exception:
            pass

    def reset(self):
        lib().orc_state_reset(self.state)

    def decode(self, token: int, position: int, mode: int = MODE_FP32, taps: bool = False):
        g = self.geom
        logits = np.empty(g.vocab_size, dtype=np.float32)
        tp = np.empty((g.num_layers + 2, g.hidden_size), dtype=np.float32) if taps else None
        rc = lib().orc_decode(ctypes.byref(self.cfg), ctypes.byref(self.w), self.state, int(token),
                              int(position), int(mode), _ptr(logits, ctypes.c_float),
                              _ptr(tp, ctypes.c_float) if taps else None)
        if rc != 0:
            raise ValueError(f"oracle decode rejected token {token} at position {position}")
        return (logits, tp) if taps else logits

    def prefill(self, tokens, start: int, mode: int = MODE_FP32, logits: bool = True):
        """Tokens at positions start..start+len-1 as one chunk (orc_prefill):
        appends their K/V to the cache and returns the last row's logits."""
        ids = np.ascontiguousarray(np.asarray(tokens, dtype=np.int32))
        out = np.empty(self.geom.vocab_size, dtype=np.float32) if logits else None
        rc = lib().orc_prefill(ctypes.byref(self.cfg), ctypes.byref(self.w), self.state,
                               _ptr(ids, ctypes.c_int32), int(ids.size), int(start), int(mode),
                               _ptr(out, ctypes.c_float) if logits else None)
        if rc != 0:
            raise ValueError(f"oracle prefill rejected {ids.size} tokens at position {start} (rc {rc})")
        return out


def argmax(logits: np.ndarray) -> int:
    l = np.ascontiguousarray(logits, dtype=np.float32)
    return int(lib().orc_argmax(_ptr(l, ctypes.c_float), l.size))


def sample(logits: np.ndarray, temperature: float, top_k: int, top_p: float, uniform: float) -> int:
    l = np.ascontiguousarray(logits, dtype=np.float32)
    inv_t = float(np.float32(1.0) / np.float32(temperature)) if temperature > 0 else 0.0
    return int(lib().orc_sample(_ptr(l, ctypes.c_float), l.size, inv_t, int(top_k),
                                float(top_p), float(uniform)))


def det_expf(x: float) -> float:
    return float(lib().orc_det_expf(float(x)))


def philox(ctr, key):
    c = (ctypes.c_uint32 * 4)(*ctr)
    k = (ctypes.c_uint32 * 2)(*key)
    o = (ctypes.c_uint32 * 4)()
    lib().orc_philox4x32_10(c, k, o)
    return list(o)


def philox_uniform(seed: int, counter: int, stream: int) -> float:
    return float(lib().orc_philox_uniform(seed, counter, stream))


def tree_sum_1024(e: np.ndarray) -> float:
    a = np.ascontiguousarray(e, dtype=np.float32)
    return float(lib().orc_tree_sum_1024(_ptr(a, ctypes.c_float), a.size))


def page_permutation(n: int, seed: int) -> np.ndarray:
    out = np.empty(n, dtype=np.int32)
    lib().orc_page_permutation(_ptr(out, ctypes.c_int32), n, seed)
    return out


def paged_reserve(tables: np.ndarray, page_size: int, old_length: int, new_length: int,
                  pages_mapped: int, pool_pages: int, order: Optional[np.ndarray] = None) -> int:
    layers, max_pages = tables.shape
    return int(lib().orc_paged_reserve(_ptr(tables, ctypes.c_int32), layers, max_pages, page_size,
                                       old_length, new_length, pages_mapped, pool_pages,
                                       _ptr(order, ctypes.c_int32) if order is not None else None))


def gemv(w: np.ndarray, x: np.ndarray) -> np.ndarray:
    rows, cols = w.shape
    y = np.empty(rows, dtype=np.float32)
    lib().orc_gemv(_ptr(y, ctypes.c_float), _ptr(np.ascontiguousarray(w), ctypes.c_uint16),
                   _ptr(np.ascontiguousarray(x), ctypes.c_uint16), rows, cols)
    return y


def rmsnorm(x: np.ndarray, w: np.ndarray, eps: float, round_out: bool = True) -> np.ndarray:
    tokens, dim = x.shape
    out = np.empty((tokens, dim), dtype=np.float32)
    lib().orc_rmsnorm(_ptr(out, ctypes.c_float), _ptr(np.ascontiguousarray(x), ctypes.c_uint16),
                      _ptr(np.ascontiguousarray(w), ctypes.c_uint16), tokens, dim, eps, int(round_out))
    return out


def add_residual_rmsnorm(x: np.ndarray, delta: np.ndarray, w: np.ndarray, eps: float):
    """Returns (normed fp32 [bf16-rounded], updated x bf16 bits)."""
    x = np.ascontiguousarray(x.copy())
    tokens, dim = x.shape
    out = np.empty((tokens, dim), dtype=np.float32)
    lib().orc_add_residual_rmsnorm(_ptr(out, ctypes.c_float), _ptr(x, ctypes.c_uint16),
                                   _ptr(np.ascontiguousarray(delta), ctypes.c_uint16),
                                   _ptr(np.ascontiguousarray(w), ctypes.c_uint16), tokens, dim, eps)
    return out, x


def swiglu(gate: np.ndarray, up: np.ndarray) -> np.ndarray:
    out = np.empty(gate.size, dtype=np.float32)
    lib().orc_swiglu(_ptr(out, ctypes.c_float), _ptr(np.ascontiguousarray(gate), ctypes.c_uint16),
                     _ptr(np.ascontiguousarray(up), ctypes.c_uint16), gate.size)
    return out


def rope_rows(x: np.ndarray, inv_freq: np.ndarray, start: int, heads: int, head_dim: int,
              src_row_stride: int, head_major: bool) -> np.ndarray:
    tokens = x.shape[0]
    out = np.empty(tokens * heads * head_dim, dtype=np.float32)
    lib().orc_rope_rows(_ptr(out, ctypes.c_float), _ptr(np.ascontiguousarray(x), ctypes.c_uint16),
                        _ptr(np.ascontiguousarray(inv_freq, dtype=np.float32), ctypes.c_float),
                        tokens, start, heads, head_dim, src_row_stride, int(head_major))
    return out


def attention(q: np.ndarray, keys: np.ndarray, values: np.ndarray, num_heads: int,
              num_kv_heads: int, head_dim: int, positions: int) -> np.ndarray:
    out = np.empty(num_heads * head_dim, dtype=np.float32)
    scale = float(np.float32(1.0) / np.sqrt(np.float32(head_dim)))
    lib().orc_attention(_ptr(out, ctypes.c_float), _ptr(np.ascontiguousarray(q), ctypes.c_uint16),
                        _ptr(np.ascontiguousarray(keys), ctypes.c_uint16),
                        _ptr(np.ascontiguousarray(values), ctypes.c_uint16), num_heads,
                        num_kv_heads, head_dim, positions, scale)
    return out


def ref_rope_inv_freq(config_json: str) -> Optional[np.ndarray]:
    """The reference's own compute_rope_inv_freq (oracle/_ref), or None when
    the reference sources were not available to build it."""
    if not os.path.exists(REF_LIB_PATH):
        return None
    L = ctypes.CDLL(REF_LIB_PATH)
    L.ref_rope_inv_freq.restype = ctypes.c_int
    L.ref_rope_inv_freq.argtypes = [ctypes.c_char_p, _f32p, ctypes.c_int, ctypes.c_char_p, ctypes.c_int]
    out = np.zeros(512, dtype=np.float32)
    err = ctypes.create_string_buffer(512)
    n = L.ref_rope_inv_freq(config_json.encode(), _ptr(out, ctypes.c_float), 512, err, 512)
    if n < 0:
        raise ValueError(err.value.decode())
    return out[:n].copy()

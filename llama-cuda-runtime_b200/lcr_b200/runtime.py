"""Python front end of liblcr_b200.so (the C ABI in include/lcr_b200.h).

Mirrors the reference's host interface for the decode path: ``Model`` has
``prefill``, ``decode``, ``sample``, ``reset``, ``position`` and
``logits_to_host`` with the meaning of src/model.h:60-127, and the
module-level ``launch_*`` functions mirror src/kernels.cuh. Device memory and
streams come from torch; every call goes through the C ABI. There is no CPU
fallback: without the built library or a CUDA device these raise.
"""
from __future__ import annotations

import ctypes
import os
from typing import Optional, Sequence

import numpy as np

from . import checkpoint as ck

PKG_DIR = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
LIB_PATH = os.path.join(PKG_DIR, "liblcr_b200.so")
HEADER = os.path.join(os.path.dirname(PKG_DIR), "include", "lcr_b200.h")

LCR_OK = 0
STATUS_NAMES = {0: "LCR_OK", 1: "LCR_ERR_INVALID", 2: "LCR_ERR_SHAPE", 3: "LCR_ERR_CUDA",
                4: "LCR_ERR_TIMEOUT", 5: "LCR_ERR_POOL", 6: "LCR_ERR_STATE", 7: "LCR_ERR_NO_DEVICE"}
FLAG_NO_PDL = 1
FLAG_NO_GRAPH = 2
FLAG_NO_PERSISTENT = 4
FLAG_TRACE = 8
# The persistent step with fp32 activations (bf16 hi/lo GEMV inputs, fp32
# q/k/v, attention output, residual stream and SwiGLU) instead of the
# reference's bf16 storage rounding: closer to the fp32 host evaluation, about
# 10 % slower.
FLAG_FP32_ACT = 16
# Tests only: the persistent step's waits give up after 50 ms and CTA 0 skips
# its first arrival (a grid barrier, or its first exchange words), so every
# step stops with LCR_ERR_TIMEOUT.
FLAG_TEST_TIMEOUT = 32
# lcr_prefill one decode step per token (the decode step's maths) instead of
# the tcgen05 chunks of up to 2048 prompt rows.
FLAG_PER_TOKEN_PREFILL = 64
# The persistent step's attention phase on CUDA cores (8 lanes per cached
# position) instead of the tensor pipe (mma.sync over 16-position units).
FLAG_CUDA_CORE_ATTENTION = 128
# The persistent step's phases meet at grid barriers instead of exchanging
# tagged words (the default with bf16 activations and the tensor-pipe
# attention; the results are the same bits).
FLAG_GRID_BARRIERS = 256


class LcrError(RuntimeError):
    """A non-OK lcr_status, with lcr_last_error_string()."""

    def __init__(self, status: int, message: str):
        super().__init__(f"{STATUS_NAMES.get(status, status)}: {message}")
        self.status = status


class ModelDesc(ctypes.Structure):
    _fields_ = [("hidden_size", ctypes.c_int), ("intermediate_size", ctypes.c_int),
                ("num_layers", ctypes.c_int), ("num_heads", ctypes.c_int),
                ("num_kv_heads", ctypes.c_int), ("head_dim", ctypes.c_int),
                ("vocab_size", ctypes.c_int), ("rms_norm_eps", ctypes.c_float),
                ("rope_theta", ctypes.c_float), ("rope_scaling", ctypes.c_int),
                ("rope_factor", ctypes.c_float), ("rope_low_freq_factor", ctypes.c_float),
                ("rope_high_freq_factor", ctypes.c_float),
                ("rope_original_max_position_embeddings", ctypes.c_int)]


class LayerWeights(ctypes.Structure):
    _fields_ = [("input_norm", ctypes.c_void_p), ("qkv_proj", ctypes.c_void_p),
                ("o_proj", ctypes.c_void_p), ("post_attention_norm", ctypes.c_void_p),
                ("gate_up_proj", ctypes.c_void_p), ("down_proj", ctypes.c_void_p)]


class Weights(ctypes.Structure):
    _fields_ = [("embedding", ctypes.c_void_p), ("final_norm", ctypes.c_void_p),
                ("lm_head", ctypes.c_void_p), ("layers", ctypes.POINTER(LayerWeights))]


class Options(ctypes.Structure):
    _fields_ = [("device", ctypes.c_int), ("max_seq", ctypes.c_int), ("paged", ctypes.c_int),
                ("page_size", ctypes.c_int), ("attention_splits", ctypes.c_int),
                ("page_order_seed", ctypes.c_uint64), ("gemv_ctas", ctypes.c_int),
                ("flags", ctypes.c_int)]


class BatchOptions(ctypes.Structure):
    _fields_ = [("device", ctypes.c_int), ("max_batch", ctypes.c_int), ("max_seq", ctypes.c_int),
                ("page_size", ctypes.c_int), ("pool_pages", ctypes.c_int), ("flags", ctypes.c_int)]


class KvView(ctypes.Structure):
    _fields_ = [("keys", ctypes.c_void_p), ("values", ctypes.c_void_p),
                ("page_table", ctypes.c_void_p), ("page_size", ctypes.c_int),
                ("page_stride", ctypes.c_int), ("head_stride", ctypes.c_int),
                ("num_kv_heads", ctypes.c_int), ("head_dim", ctypes.c_int)]


_V = ctypes.c_void_p
_I = ctypes.c_int
_F = ctypes.c_float
_SIGS = {
    "lcr_last_error_string": (ctypes.c_char_p, []),
    "lcr_status_string": (ctypes.c_char_p, [_I]),
    "lcr_version": (_I, []),
    "lcr_embedding_lookup": (_I, [_V, _V, _V, _I, _I, _V]),
    "lcr_rmsnorm": (_I, [_V, _V, _V, _I, _I, _F, _V]),
    "lcr_add_residual": (_I, [_V, _V, ctypes.c_int64, _V]),
    "lcr_add_residual_rmsnorm": (_I, [_V, _V, _V, _V, _I, _I, _F, _V]),
    "lcr_swiglu": (_I, [_V, _V, _V, ctypes.c_int64, _V]),
    "lcr_swiglu_strided": (_I, [_V, _V, _V, _I, _I, _I, _V]),
    "lcr_rope_q": (_I, [_V, _V, _V, _I, _I, _I, _I, _I, _V]),
    "lcr_rope_write_kv": (_I, [ctypes.POINTER(KvView), _V, _V, _V, _I, _I, _I, _I, _V]),
    "lcr_causal_softmax": (_I, [_V, _V, _I, _I, _I, _I, _V]),
    "lcr_merge_heads": (_I, [_V, _V, _I, _I, _I, _V]),
    "lcr_gather_kv": (_I, [_V, _V, ctypes.POINTER(KvView), _I, _V]),
    "lcr_decode_attention": (_I, [_V, _V, ctypes.POINTER(KvView), _I, _I, _I, _F, _I, _I, _V, _V]),
    "lcr_decode_attention_noalloc": (_I, [_V, _V, ctypes.POINTER(KvView), _I, _I, _I, _F, _I, _I, _V]),
    "lcr_decode_attention_scratch_floats": (ctypes.c_size_t, [_I, _I, _I]),
    "lcr_choose_attention_splits": (_I, [_I, _I, _I]),
    "lcr_sample": (_I, [_V, _V, _I, _F, _I, _F, _F, _V, _V]),
    "lcr_sample_scratch_floats": (ctypes.c_size_t, [_I, _I]),
    "lcr_gemm_nt": (_I, [_V, _I, _V, _V, _I, _I, _I, _V]),
    "lcr_ctx_create": (_I, [ctypes.POINTER(ModelDesc), ctypes.POINTER(Weights),
                            ctypes.POINTER(Options), ctypes.POINTER(_V)]),
    "lcr_ctx_destroy": (None, [_V]),
    "lcr_rope_inv_freq": (_I, [ctypes.POINTER(ModelDesc), _V, _I]),
    "lcr_reset": (_I, [_V]),
    "lcr_position": (_I, [_V]),
    "lcr_decode": (_I, [_V, _I, ctypes.POINTER(_V)]),
    "lcr_prefill": (_I, [_V, _V, _I, ctypes.POINTER(_V)]),
    "lcr_logits_to_host": (_I, [_V, _V]),
    "lcr_sample_logits": (_I, [_V, _V, _F, _I, _F, _F, ctypes.POINTER(_I)]),
    "lcr_generate_greedy": (_I, [_V, _I, _I, _V]),
    "lcr_set_token": (_I, [_V, _V, _I]),
    "lcr_step_host": (_I, [_V, ctypes.c_int32, _I, _V]),
    "lcr_enqueue_steps": (_I, [_V, _I]),
    "lcr_read_token": (_I, [_V, _V]),
    "lcr_sync": (_I, [_V]),
    "lcr_ctx_stream": (_V, [_V]),
    "lcr_kv_view_of": (_I, [_V, _I, ctypes.POINTER(KvView)]),
    "lcr_page_tables": (_I, [_V, _V, ctypes.POINTER(_I)]),
    "lcr_reserve_length": (_I, [_V, _I]),
    "lcr_weight_bytes_per_token": (ctypes.c_size_t, [_V]),
    "lcr_kv_bytes_per_position": (ctypes.c_size_t, [_V]),
    "lcr_step_launches": (_I, [_V]),
    "lcr_device_status": (_I, [_V]),
    "lcr_time_steps": (_I, [_V, _I, ctypes.POINTER(_F)]),
    "lcr_time_gemv": (_I, [_V, _I, _I, _I, ctypes.POINTER(_F)]),
    "lcr_copy_trace": (_I, [_V, _V, _I, ctypes.POINTER(_I)]),
    "lcr_batch_create": (_I, [_V, _V, _V, ctypes.POINTER(_V)]),
    "lcr_batch_destroy": (None, [_V]),
    "lcr_batch_set_pages": (_I, [_V, _I, _V, _I]),
    "lcr_batch_set_sampling": (_I, [_V, _I, _F, _I, _F, ctypes.c_uint64]),
    "lcr_batch_step": (_I, [_V, _I, _V, _V]),
    "lcr_batch_read": (_I, [_V, _V, _I]),
    "lcr_batch_fill_kv": (_I, [_V, _I, _I, ctypes.c_uint64]),
    "lcr_batch_prefill": (_I, [_V, _I, _V, _I, _I]),
    "lcr_batch_logits": (_I, [_V, _I, _V]),
    "lcr_batch_sync": (_I, [_V]),
    "lcr_batch_stream": (_V, [_V]),
    "lcr_batch_step_launches": (_I, [_V, _I]),
    "lcr_batch_time_steps": (_I, [_V, _I, ctypes.POINTER(_F)]),
}

_lib: Optional[ctypes.CDLL] = None


def lib() -> ctypes.CDLL:
    """Loads liblcr_b200.so (built by __graft_entry__.build() or
    `make -C llama-cuda-runtime_b200`). Raises when it is missing: there is no
    fallback path."""
    global _lib
    if _lib is None:
        if not os.path.exists(LIB_PATH):
            raise RuntimeError(f"{LIB_PATH} is not built; run `make -C {PKG_DIR}`")
        L = ctypes.CDLL(LIB_PATH)
        for name, (res, args) in _SIGS.items():
            fn = getattr(L, name)
            fn.restype = res
            fn.argtypes = args
        _lib = L
    return _lib


def check(status: int) -> None:
    if status != LCR_OK:
        raise LcrError(status, lib().lcr_last_error_string().decode(errors="replace"))


def header_functions() -> list:
    """Every function include/lcr_b200.h declares."""
    import re

    text = open(HEADER).read()
    return re.findall(r"^LCR_API [^(]*?\b(lcr_\w+)\(", text, flags=re.M)


# ---------------------------------------------------------------------------
# torch helpers (device memory and streams are torch's; compute is ours)
# ---------------------------------------------------------------------------

def _torch():
    import torch

    return torch


def stream_ptr(stream=None) -> int:
    torch = _torch()
    s = stream if stream is not None else torch.cuda.current_stream()
    return s.cuda_stream


def upload_block(block: ck.WeightBlock, device: int = 0):
    """The weight block as one device allocation (src/model.cu:186-207)."""
    torch = _torch()
    host = torch.from_numpy(block.data.view(np.int16))
    return host.to(f"cuda:{device}")


def _check_weights_device(weights_dev, device: int) -> None:
    """The context's kernels read the weights directly: they must be in that
    device's memory (the C ABI rejects them otherwise; this says so first)."""
    where = getattr(weights_dev, "device", None)
    if where is not None and where.type == "cuda" and where.index != device:
        raise ValueError(f"weights are on cuda:{where.index}, the context is on cuda:{device}")


def desc_of(geom: ck.Geometry) -> ModelDesc:
    return ModelDesc(geom.hidden_size, geom.intermediate_size, geom.num_layers, geom.num_heads,
                     geom.num_kv_heads, geom.head_dim, geom.vocab_size, geom.rms_norm_eps,
                     geom.rope_theta, int(geom.rope_scaling), geom.rope_factor,
                     geom.rope_low_freq_factor, geom.rope_high_freq_factor,
                     geom.rope_original_max_position_embeddings)


def rope_inv_freq(geom: ck.Geometry) -> np.ndarray:
    """The context's RoPE inverse frequencies for `geom` (lcr_rope_inv_freq)."""
    out = np.zeros(geom.head_dim // 2, dtype=np.float32)
    d = desc_of(geom)
    check(lib().lcr_rope_inv_freq(ctypes.byref(d), out.ctypes.data, out.size))
    return out


class Model:
    """The decode context (Model, src/model.h:60-127) over a device copy of a
    WeightBlock. ``max_seq``, ``paged``, ``page_size`` and
    ``attention_splits`` are Model::Options (src/model.h:62-77)."""

    def __init__(self, block: ck.WeightBlock, weights_dev=None, *, device: int = 0,
                 max_seq: int = 4096, paged: bool = False, page_size: int = 16,
                 attention_splits: int = 0, page_order_seed: int = 0, gemv_ctas: int = 0,
                 flags: int = 0):
        self.geom = block.geom
        self.block = block
        self.device = device
        self.weights_dev = weights_dev if weights_dev is not None else upload_block(block, device)
        _check_weights_device(self.weights_dev, device)
        base = self.weights_dev.data_ptr()
        g = self.geom
        addr = lambda name: base + block.offsets[name][0] * 2
        self._layers = (LayerWeights * g.num_layers)(*[
            LayerWeights(*[addr(n) for n in block.layer_groups(l)]) for l in range(g.num_layers)])
        self._weights = Weights(addr("embed"), addr("final_norm"), addr(block.lm_head_group), self._layers)
        self._desc = desc_of(g)
        self.options = Options(device, max_seq, int(paged), page_size, attention_splits,
                               page_order_seed, gemv_ctas, flags)
        ctx = ctypes.c_void_p()
        check(lib().lcr_ctx_create(ctypes.byref(self._desc), ctypes.byref(self._weights),
                                   ctypes.byref(self.options), ctypes.byref(ctx)))
        self.ctx = ctx
        self.max_seq = max_seq

    def close(self):
        if getattr(self, "ctx", None):
            lib().lcr_ctx_destroy(self.ctx)
            self.ctx = None

    def __del__(self):
        try:
            self.close()
        except Exception:
            pass

    # --- Model interface -------------------------------------------------
    @property
    def position(self) -> int:
        return lib().lcr_position(self.ctx)

    def reset(self) -> None:
        check(lib().lcr_reset(self.ctx))

    def decode(self, token: int) -> int:
        """One token at the current position; returns the device logits
        pointer (valid until the next call)."""
        out = ctypes.c_void_p()
        check(lib().lcr_decode(self.ctx, int(token), ctypes.byref(out)))
        return out.value

    def prefill(self, tokens: Sequence[int]) -> int:
        arr = np.ascontiguousarray(np.asarray(tokens, dtype=np.int32))
        out = ctypes.c_void_p()
        check(lib().lcr_prefill(self.ctx, arr.ctypes.data, arr.size, ctypes.byref(out)))
        return out.value

    def logits_to_host(self) -> np.ndarray:
        out = np.empty(self.geom.vocab_size, dtype=np.float32)
        check(lib().lcr_logits_to_host(self.ctx, out.ctypes.data))
        return out

    def sample(self, logits_ptr: int, temperature: float, top_k: int, top_p: float,
               uniform: float) -> int:
        tok = ctypes.c_int()
        check(lib().lcr_sample_logits(self.ctx, logits_ptr, float(temperature), int(top_k),
                                      float(top_p), float(uniform), ctypes.byref(tok)))
        return tok.value

    def generate_greedy(self, first_token: int, steps: int) -> np.ndarray:
        out = np.empty(steps, dtype=np.int32)
        check(lib().lcr_generate_greedy(self.ctx, int(first_token), int(steps), out.ctypes.data))
        return out

    def reserve_length(self, length: int) -> None:
        check(lib().lcr_reserve_length(self.ctx, int(length)))

    def page_tables(self) -> tuple:
        g = self.geom
        max_pages = (self.max_seq + self.options.page_size - 1) // self.options.page_size
        t = np.full((g.num_layers, max_pages), -1, dtype=np.int32)
        mapped = ctypes.c_int()
        check(lib().lcr_page_tables(self.ctx, t.ctypes.data, ctypes.byref(mapped)))
        return t, mapped.value

    def kv_view(self, layer: int) -> KvView:
        v = KvView()
        check(lib().lcr_kv_view_of(self.ctx, int(layer), ctypes.byref(v)))
        return v

    @property
    def stream(self) -> int:
        return lib().lcr_ctx_stream(self.ctx)

    def weight_bytes_per_token(self) -> int:
        return int(lib().lcr_weight_bytes_per_token(self.ctx))

    def kv_bytes_per_position(self) -> int:
        return int(lib().lcr_kv_bytes_per_position(self.ctx))

    def step_launches(self) -> int:
        return int(lib().lcr_step_launches(self.ctx))

    # --- async loop pieces ------------------------------------------------
    def set_token(self, host_token_ptr: int, position: int) -> None:
        check(lib().lcr_set_token(self.ctx, host_token_ptr, int(position)))

    def step_host(self, token: int, position: int) -> int:
        """One decode step of `token` at `position` and its greedy next token,
        synchronously, in one call (lcr_step_host)."""
        out = ctypes.c_int32()
        check(lib().lcr_step_host(self.ctx, int(token), int(position), ctypes.byref(out)))
        return int(out.value)

    def enqueue_steps(self, steps: int) -> None:
        check(lib().lcr_enqueue_steps(self.ctx, int(steps)))

    def read_token(self, host_token_ptr: int) -> None:
        check(lib().lcr_read_token(self.ctx, host_token_ptr))

    def sync(self) -> None:
        check(lib().lcr_sync(self.ctx))

    def time_steps(self, steps: int) -> float:
        ms = ctypes.c_float()
        check(lib().lcr_time_steps(self.ctx, int(steps), ctypes.byref(ms)))
        return ms.value

    def trace(self) -> np.ndarray:
        """Per-CTA phase timestamps of the last step ([ctas][1024] ns)."""
        n = 1024 * 1024
        buf = np.zeros(n, dtype=np.uint64)
        got = ctypes.c_int()
        check(lib().lcr_copy_trace(self.ctx, buf.ctypes.data, n, ctypes.byref(got)))
        return buf[:got.value].reshape(-1, 1024)

    def time_gemv(self, matrix: int, layer: int = 0, reps: int = 20) -> float:
        ms = ctypes.c_float()
        check(lib().lcr_time_gemv(self.ctx, int(matrix), int(layer), int(reps), ctypes.byref(ms)))
        return ms.value


class Batch:
    """Batched decode over a device copy of a WeightBlock: up to ``max_batch``
    sequences in slots, one token each per step (lcr_batch_*). KV pages come
    from a pool of ``pool_pages`` pages of ``page_size`` positions; the caller
    assigns them per slot (``set_pages``), as a continuous-batching scheduler
    does."""

    def __init__(self, block: ck.WeightBlock, weights_dev=None, *, device: int = 0,
                 max_batch: int = 64, max_seq: int = 4096, page_size: int = 16,
                 pool_pages: int = 1024, flags: int = 0):
        self.geom = block.geom
        self.block = block
        self.device = device
        self.weights_dev = weights_dev if weights_dev is not None else upload_block(block, device)
        _check_weights_device(self.weights_dev, device)
        base = self.weights_dev.data_ptr()
        g = self.geom
        addr = lambda name: base + block.offsets[name][0] * 2
        self._layers = (LayerWeights * g.num_layers)(*[
            LayerWeights(*[addr(n) for n in block.layer_groups(l)]) for l in range(g.num_layers)])
        self._weights = Weights(addr("embed"), addr("final_norm"), addr(block.lm_head_group), self._layers)
        self._desc = desc_of(g)
        self.options = BatchOptions(device, max_batch, max_seq, page_size, pool_pages, flags)
        h = ctypes.c_void_p()
        check(lib().lcr_batch_create(ctypes.byref(self._desc), ctypes.byref(self._weights),
                                     ctypes.byref(self.options), ctypes.byref(h)))
        self.h = h
        self.max_batch = max_batch
        self.page_size = page_size

    def close(self):
        if getattr(self, "h", None):
            lib().lcr_batch_destroy(self.h)
            self.h = None

    def __del__(self):
        try:
            self.close()
        except Exception:
            pass

    def set_pages(self, slot: int, pages) -> None:
        arr = np.ascontiguousarray(np.asarray(pages, dtype=np.int32))
        check(lib().lcr_batch_set_pages(self.h, int(slot), arr.ctypes.data, int(arr.size)))

    def set_sampling(self, slot: int, temperature: float = 0.0, top_k: int = 0,
                     top_p: float = 1.0, seed: int = 0) -> None:
        check(lib().lcr_batch_set_sampling(self.h, int(slot), float(temperature), int(top_k),
                                           float(top_p), int(seed)))

    def step(self, tokens, positions) -> None:
        """tokens=None continues each slot with its previous sample."""
        p = np.ascontiguousarray(np.asarray(positions, dtype=np.int32))
        if tokens is None:
            check(lib().lcr_batch_step(self.h, int(p.size), None, p.ctypes.data))
            return
        t = np.ascontiguousarray(np.asarray(tokens, dtype=np.int32))
        assert t.size == p.size
        check(lib().lcr_batch_step(self.h, int(t.size), t.ctypes.data, p.ctypes.data))

    def fill_kv(self, slot: int, length: int, seed: int) -> None:
        check(lib().lcr_batch_fill_kv(self.h, int(slot), int(length), int(seed)))

    def prefill(self, slot: int, tokens, start: int = 0) -> None:
        """Prefill `tokens` for `slot` at positions start .. (tcgen05 GEMMs
        and causal flash attention); the slot's logits / next id then hold
        the last row's."""
        ids = np.ascontiguousarray(np.asarray(tokens, dtype=np.int32))
        check(lib().lcr_batch_prefill(self.h, int(slot), ids.ctypes.data, int(ids.size), int(start)))

    def read(self, n: int) -> np.ndarray:
        out = np.zeros(n, dtype=np.int32)
        check(lib().lcr_batch_read(self.h, out.ctypes.data, int(n)))
        return out

    def logits(self, slot: int) -> np.ndarray:
        out = np.zeros(self.geom.vocab_size, dtype=np.float32)
        check(lib().lcr_batch_logits(self.h, int(slot), out.ctypes.data))
        return out

    def sync(self) -> None:
        check(lib().lcr_batch_sync(self.h))

    @property
    def stream(self) -> int:
        return lib().lcr_batch_stream(self.h)

    def step_launches(self, n: int) -> int:
        return lib().lcr_batch_step_launches(self.h, int(n))

    def time_steps(self, steps: int) -> float:
        ms = ctypes.c_float()
        check(lib().lcr_batch_time_steps(self.h, int(steps), ctypes.byref(ms)))
        return ms.value

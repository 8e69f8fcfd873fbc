"""Model geometry and the seeded random-init checkpoint.

The reference loads a real checkpoint (src/model.cu:112-213); this build runs on
random-init weights of the same architecture, generated from a seed:

* tensors are numbered in ``required_weights`` order (src/config.cpp:197-221):
  the embedding 0, then per layer q, k, v, o, gate, up, down; tensor t is cut
  into chunks of 2**24 elements and chunk c is
  ``default_rng([seed, t, c]).standard_normal(n, dtype=float32) * float32(0.02)``
  (numpy), rounded to bf16 (nearest, ties to even) -- independent streams, so
  the chunks are generated in parallel threads;
* every RMSNorm gain is exactly 1.0 (not drawn);
* there is no lm_head tensor: the output head is the embedding (tied,
  src/model.cu:212).

The weights live in ONE uint16 block in the order a forward pass reads them,
each tensor group 256-byte aligned, with Q/K/V stacked into one ``[q;k;v]``
matrix and gate/up into one ``[gate;up]`` matrix: the device layout of
src/model.cu:160-207. ``WeightBlock.offsets`` gives each group's element
offset, so the same host array feeds the GPU upload and the CPU oracle.
"""
from __future__ import annotations

import dataclasses
import json
import os
from typing import Dict, List, Optional, Tuple

import numpy as np


@dataclasses.dataclass(frozen=True)
class Geometry:
    """Model geometry (the fields of ModelConfig, src/config.h:22-60)."""

    hidden_size: int
    intermediate_size: int
    num_layers: int
    num_heads: int
    num_kv_heads: int
    head_dim: int
    vocab_size: int
    rms_norm_eps: float = 1e-5
    rope_theta: float = 500000.0
    rope_scaling: bool = True
    rope_factor: float = 32.0
    rope_low_freq_factor: float = 1.0
    rope_high_freq_factor: float = 4.0
    rope_original_max_position_embeddings: int = 8192
    max_position_embeddings: int = 131072
    name: str = "custom"

    @property
    def q_dim(self) -> int:
        return self.num_heads * self.head_dim

    @property
    def kv_dim(self) -> int:
        return self.num_kv_heads * self.head_dim

    @property
    def qkv_rows(self) -> int:
        return self.q_dim + 2 * self.kv_dim

    @property
    def heads_per_kv(self) -> int:
        return self.num_heads // self.num_kv_heads

    def kv_bytes_per_position(self) -> int:
        """K and V, every layer, bf16 (src/config.h:47-49)."""
        return self.num_layers * 2 * self.kv_dim * 2

    def weight_bytes_per_token(self) -> int:
        """Bytes one decode step must stream (src/model.cu:91-102)."""
        h, q, kv, f = self.hidden_size, self.q_dim, self.kv_dim, self.intermediate_size
        per = self.num_layers * (h * 2 + q * h + kv * h * 2 + h * q + f * h * 3)
        per += h + self.vocab_size * h
        return per * 2

    def config_json(self) -> dict:
        """A Llama config.json for this geometry (the fields
        src/config.cpp:46-133 reads)."""
        doc = {
            "architectures": ["LlamaForCausalLM"],
            "model_type": "llama",
            "attention_bias": False,
            "mlp_bias": False,
            "hidden_act": "silu",
            "hidden_size": self.hidden_size,
            "intermediate_size": self.intermediate_size,
            "num_hidden_layers": self.num_layers,
            "num_attention_heads": self.num_heads,
            "num_key_value_heads": self.num_kv_heads,
            "head_dim": self.head_dim,
            "vocab_size": self.vocab_size,
            "max_position_embeddings": self.max_position_embeddings,
            "rms_norm_eps": self.rms_norm_eps,
            "rope_theta": self.rope_theta,
            "tie_word_embeddings": True,
            "torch_dtype": "bfloat16",
            "bos_token_id": 128000,
            "eos_token_id": [128001, 128008, 128009],
        }
        if self.rope_scaling:
            doc["rope_scaling"] = {
                "rope_type": "llama3",
                "factor": self.rope_factor,
                "low_freq_factor": self.rope_low_freq_factor,
                "high_freq_factor": self.rope_high_freq_factor,
                "original_max_position_embeddings": self.rope_original_max_position_embeddings,
            }
        return doc


LLAMA_3_2_1B = Geometry(
    hidden_size=2048, intermediate_size=8192, num_layers=16, num_heads=32,
    num_kv_heads=8, head_dim=64, vocab_size=128256, name="llama-3.2-1b")

TINY = Geometry(
    hidden_size=256, intermediate_size=1024, num_layers=2, num_heads=4,
    num_kv_heads=2, head_dim=64, vocab_size=128256, name="tiny")


def small_geometry(layers=2, hidden=256, heads=4, kv_heads=2, head_dim=64,
                   ffn=1024, vocab=4096, name="small") -> Geometry:
    return Geometry(hidden_size=hidden, intermediate_size=ffn, num_layers=layers,
                    num_heads=heads, num_kv_heads=kv_heads, head_dim=head_dim,
                    vocab_size=vocab, name=name)


def float_to_bf16_bits(x: np.ndarray) -> np.ndarray:
    """Round float32 to bf16, nearest with ties to even; returns uint16."""
    u = np.ascontiguousarray(x, dtype=np.float32).view(np.uint32)
    r = (u + np.uint32(0x7FFF) + ((u >> np.uint32(16)) & np.uint32(1))) >> np.uint32(16)
    return r.astype(np.uint16)


def bf16_bits_to_float(b: np.ndarray) -> np.ndarray:
    return (np.asarray(b, dtype=np.uint16).astype(np.uint32) << np.uint32(16)).view(np.float32)


ALIGN_ELEMS = 128  # 256 bytes of bf16 (src/model.cu:186-207)


def _align(n: int) -> int:
    return (n + ALIGN_ELEMS - 1) // ALIGN_ELEMS * ALIGN_ELEMS


@dataclasses.dataclass
class WeightBlock:
    """One host array with every weight in forward-read order."""

    geom: Geometry
    data: np.ndarray  # uint16, bf16 bits
    offsets: Dict[str, Tuple[int, int]]  # group name -> (element offset, element count)

    def view(self, name: str) -> np.ndarray:
        off, n = self.offsets[name]
        return self.data[off:off + n]

    def layer_groups(self, layer: int) -> List[str]:
        p = f"layers.{layer}."
        return [p + s for s in ("input_norm", "qkv", "o", "post_norm", "gate_up", "down")]

    @property
    def nbytes(self) -> int:
        return int(self.data.nbytes)


def block_layout(geom: Geometry) -> Tuple[Dict[str, Tuple[int, int]], int]:
    """Element offsets of every weight group in the read-order block."""
    g = geom
    groups: List[Tuple[str, int]] = [("embed", g.vocab_size * g.hidden_size)]
    for l in range(g.num_layers):
        p = f"layers.{l}."
        groups += [
            (p + "input_norm", g.hidden_size),
            (p + "qkv", g.qkv_rows * g.hidden_size),
            (p + "o", g.hidden_size * g.q_dim),
            (p + "post_norm", g.hidden_size),
            (p + "gate_up", 2 * g.intermediate_size * g.hidden_size),
            (p + "down", g.hidden_size * g.intermediate_size),
        ]
    groups.append(("final_norm", g.hidden_size))
    offsets: Dict[str, Tuple[int, int]] = {}
    off = 0
    for name, n in groups:
        off = _align(off)
        offsets[name] = (off, n)
        off += n
    return offsets, _align(off)


CHUNK = 1 << 24


def _normal_bf16(seed: int, tensor: int, chunk: int, n: int) -> np.ndarray:
    v = np.random.default_rng([seed, tensor, chunk]).standard_normal(n, dtype=np.float32)
    v *= np.float32(0.02)
    return float_to_bf16_bits(v)


def generate(geom: Geometry, seed: int, threads: Optional[int] = None) -> WeightBlock:
    """The seeded random-init checkpoint (procedure in the module docstring)."""
    from concurrent.futures import ThreadPoolExecutor

    offsets, total = block_layout(geom)
    data = np.zeros(total, dtype=np.uint16)
    g = geom
    h = g.hidden_size
    # (element offset, element count) of every drawn tensor, in draw order.
    tensors: List[Tuple[int, int]] = [(offsets["embed"][0], g.vocab_size * h)]
    for l in range(g.num_layers):
        p = f"layers.{l}."
        qkv, o = offsets[p + "qkv"][0], offsets[p + "o"][0]
        gu, dn = offsets[p + "gate_up"][0], offsets[p + "down"][0]
        f_ = g.intermediate_size
        tensors += [(qkv, g.q_dim * h), (qkv + g.q_dim * h, g.kv_dim * h),
                    (qkv + (g.q_dim + g.kv_dim) * h, g.kv_dim * h), (o, h * g.q_dim),
                    (gu, f_ * h), (gu + f_ * h, f_ * h), (dn, h * f_)]
    jobs = []
    for t, (off, n) in enumerate(tensors):
        for c, start in enumerate(range(0, n, CHUNK)):
            jobs.append((t, c, off + start, min(CHUNK, n - start)))

    def run(job):
        t, c, at, m = job
        data[at:at + m] = _normal_bf16(seed, t, c, m)

    with ThreadPoolExecutor(threads or min(32, os.cpu_count() or 1)) as ex:
        list(ex.map(run, jobs))
    one = np.uint16(0x3F80)  # bf16 1.0
    for l in range(g.num_layers):
        for nm in ("input_norm", "post_norm"):
            off, n = offsets[f"layers.{l}.{nm}"]
            data[off:off + n] = one
    off, n = offsets["final_norm"]
    data[off:off + n] = one
    return WeightBlock(geom, data, offsets)


def prompt_ids(seed: int, n: int, high: int = 128000) -> np.ndarray:
    """Prompt token ids, uniform in [0, high), from a stream separate from the
    weights (``default_rng([seed, 1])``)."""
    return np.random.default_rng([seed, 1]).integers(0, high, n).astype(np.int32)


def write_safetensors(model_dir: str, block: WeightBlock) -> None:
    """Writes config.json + model.safetensors with the checkpoint's tensor names
    (the un-fused tensors of required_weights, src/config.cpp:197-221)."""
    g = block.geom
    os.makedirs(model_dir, exist_ok=True)
    with open(os.path.join(model_dir, "config.json"), "w") as f:
        json.dump(g.config_json(), f, indent=2)
    tensors: List[Tuple[str, np.ndarray, List[int]]] = []
    h = g.hidden_size
    tensors.append(("model.embed_tokens.weight", block.view("embed"), [g.vocab_size, h]))
    for l in range(g.num_layers):
        p = f"layers.{l}."
        q = f"model.layers.{l}."
        qkv = block.view(p + "qkv")
        tensors += [
            (q + "input_layernorm.weight", block.view(p + "input_norm"), [h]),
            (q + "self_attn.q_proj.weight", qkv[: g.q_dim * h], [g.q_dim, h]),
            (q + "self_attn.k_proj.weight", qkv[g.q_dim * h:(g.q_dim + g.kv_dim) * h], [g.kv_dim, h]),
            (q + "self_attn.v_proj.weight", qkv[(g.q_dim + g.kv_dim) * h:], [g.kv_dim, h]),
            (q + "self_attn.o_proj.weight", block.view(p + "o"), [h, g.q_dim]),
            (q + "post_attention_layernorm.weight", block.view(p + "post_norm"), [h]),
        ]
        gu = block.view(p + "gate_up")
        f_ = g.intermediate_size
        tensors += [
            (q + "mlp.gate_proj.weight", gu[: f_ * h], [f_, h]),
            (q + "mlp.up_proj.weight", gu[f_ * h:], [f_, h]),
            (q + "mlp.down_proj.weight", block.view(p + "down"), [h, f_]),
        ]
    tensors.append(("model.norm.weight", block.view("final_norm"), [h]))
    header: Dict[str, object] = {}
    off = 0
    for name, arr, shape in tensors:
        nb = int(arr.size) * 2
        header[name] = {"dtype": "BF16", "shape": shape, "data_offsets": [off, off + nb]}
        off += nb
    hb = json.dumps(header, separators=(",", ":")).encode()
    hb += b" " * ((8 - len(hb) % 8) % 8)
    with open(os.path.join(model_dir, "model.safetensors"), "wb") as f:
        f.write(np.uint64(len(hb)).tobytes())
        f.write(hb)
        for _, arr, _ in tensors:
            f.write(np.ascontiguousarray(arr).tobytes())


_CACHE: Dict[Tuple[Geometry, int], WeightBlock] = {}


def cached(geom: Geometry, seed: int) -> WeightBlock:
    """generate(), memoised per process (the 1B block is 2.47 GB)."""
    key = (geom, seed)
    if key not in _CACHE:
        _CACHE[key] = generate(geom, seed)
    return _CACHE[key]

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
    tie_word_embeddings: bool = True

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
            "tie_word_embeddings": self.tie_word_embeddings,
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

    @property
    def lm_head_group(self) -> str:
        """The output head: its own group when the checkpoint has
        lm_head.weight, else the (tied) embedding."""
        return "lm_head" if "lm_head" in self.offsets else "embed"

    def layer_groups(self, layer: int) -> List[str]:
        p = f"layers.{layer}."
        return [p + s for s in ("input_norm", "qkv", "o", "post_norm", "gate_up", "down")]

    @property
    def nbytes(self) -> int:
        return int(self.data.nbytes)


def block_layout(geom: Geometry, lm_head: bool = False) -> Tuple[Dict[str, Tuple[int, int]], int]:
    """Element offsets of every weight group in the read-order block (with
    `lm_head`, an untied output head after the final norm, where the
    reference's loader appends it, src/model.cu:182-186)."""
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
    if lm_head:
        groups.append(("lm_head", g.vocab_size * g.hidden_size))
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
    if "lm_head" in block.offsets:
        tensors.append(("lm_head.weight", block.view("lm_head"), [g.vocab_size, h]))
    write_safetensors_file(os.path.join(model_dir, "model.safetensors"),
                           [(name, "BF16", shape, arr) for name, arr, shape in tensors])


def write_safetensors_file(path: str, tensors) -> None:
    """One safetensors file: the little-endian u64 header length, the JSON
    header (name -> dtype, shape, data_offsets) padded with spaces to 8 bytes,
    then the tensors' bytes in order. `tensors`: (name, dtype, shape, array)."""
    header: Dict[str, object] = {}
    off = 0
    for name, dtype, shape, arr in tensors:
        nb = int(np.asarray(arr).nbytes)
        header[name] = {"dtype": dtype, "shape": list(shape), "data_offsets": [off, off + nb]}
        off += nb
    hb = json.dumps(header, separators=(",", ":")).encode()
    hb += b" " * ((8 - len(hb) % 8) % 8)
    with open(path, "wb") as f:
        f.write(np.uint64(len(hb)).tobytes())
        f.write(hb)
        for _, _, _, arr in tensors:
            f.write(np.ascontiguousarray(arr).tobytes())


class CheckpointError(ValueError):
    """A checkpoint directory this runtime cannot load (the reference's
    lcr::Error from ModelConfig / SafetensorsArchive / Model::load_weights)."""


def geometry_from_config(doc: dict, name: str = "checkpoint") -> Geometry:
    """The model geometry of a config.json document: the fields, defaults and
    checks of ModelConfig::from_json_string and validate
    (src/config.cpp:40-133, 161-184)."""
    def need(cond, msg):
        if not cond:
            raise CheckpointError(msg)

    if "model_type" in doc:
        need(doc["model_type"] == "llama",
             f'this runtime only implements the Llama architecture, config.json says '
             f'model_type="{doc["model_type"]}"')

    def req(key):
        v = doc.get(key)
        need(isinstance(v, (int, float)) and not isinstance(v, bool),
             f'config.json is missing the integer field "{key}"')
        return int(v)

    hidden, ffn, layers = req("hidden_size"), req("intermediate_size"), req("num_hidden_layers")
    heads, vocab, max_pos = req("num_attention_heads"), req("vocab_size"), req("max_position_embeddings")
    kv_heads = int(doc["num_key_value_heads"]) if "num_key_value_heads" in doc else heads
    hd = doc.get("head_dim")
    head_dim = int(hd) if isinstance(hd, (int, float)) and not isinstance(hd, bool) else \
        (hidden // heads if heads > 0 else 0)
    eps = float(np.float32(doc.get("rms_norm_eps", 1e-5)))
    theta = float(np.float32(doc.get("rope_theta", 500000.0)))
    tie = bool(doc.get("tie_word_embeddings", True))
    if isinstance(doc.get("attention_bias"), bool):
        need(not doc["attention_bias"], "attention projections with bias are not implemented")
    if isinstance(doc.get("mlp_bias"), bool):
        need(not doc["mlp_bias"], "MLP projections with bias are not implemented")
    if isinstance(doc.get("hidden_act"), str):
        need(doc["hidden_act"] == "silu",
             f'only the SiLU/SwiGLU MLP is implemented, config.json says "{doc["hidden_act"]}"')
    scaling, factor, low, high, orig = False, 32.0, 1.0, 4.0, 8192
    rs = doc.get("rope_scaling")
    if isinstance(rs, dict):
        kind = rs.get("rope_type") if isinstance(rs.get("rope_type"), str) else rs.get("type", "default")
        if not isinstance(kind, str):
            kind = "default"
        if kind not in ("default", "none"):
            need(kind == "llama3", f'only llama3 RoPE scaling is implemented, config.json says "{kind}"')
            scaling = True
            factor = float(np.float32(rs.get("factor", factor)))
            low = float(np.float32(rs.get("low_freq_factor", low)))
            high = float(np.float32(rs.get("high_freq_factor", high)))
            orig = int(rs.get("original_max_position_embeddings", orig))
    need(hidden > 0 and ffn > 0 and layers > 0,
         "config.json has a non-positive hidden_size, intermediate_size, or num_hidden_layers")
    need(heads > 0 and kv_heads > 0, "config.json has a non-positive head count")
    need(heads % kv_heads == 0,
         f"num_attention_heads ({heads}) must be a multiple of num_key_value_heads ({kv_heads})")
    need(head_dim > 0 and head_dim % 2 == 0, f"head_dim must be positive and even for RoPE, got {head_dim}")
    need(vocab > 0, "vocab_size must be positive")
    need(eps > 0.0, "rms_norm_eps must be positive")
    need(theta > 1.0, "rope_theta must be greater than one")
    if scaling:
        need(factor > 0.0, "RoPE scaling factor must be positive")
        need(high > low, "RoPE high_freq_factor must exceed low_freq_factor")
        need(orig > 0, "RoPE original_max_position_embeddings must be positive")
    return Geometry(hidden_size=hidden, intermediate_size=ffn, num_layers=layers, num_heads=heads,
                    num_kv_heads=kv_heads, head_dim=head_dim, vocab_size=vocab, rms_norm_eps=eps,
                    rope_theta=theta, rope_scaling=scaling, rope_factor=factor, rope_low_freq_factor=low,
                    rope_high_freq_factor=high, rope_original_max_position_embeddings=orig,
                    max_position_embeddings=max_pos, name=name, tie_word_embeddings=tie)


_DTYPE_BYTES = {"F64": 8, "F32": 4, "F16": 2, "BF16": 2, "I64": 8, "I32": 4, "I8": 1, "U8": 1, "BOOL": 1}


def _read_header(path: str):
    """(tensors by name: (dtype, shape, begin, end) in absolute file
    offsets, file size) of one safetensors file, with the checks of
    SafetensorsFile (src/safetensors.cpp:99-128)."""
    size = os.path.getsize(path)
    if size <= 8:
        raise CheckpointError(f"{path} is too small to be a safetensors file ({size} bytes)")
    with open(path, "rb") as f:
        n = int(np.frombuffer(f.read(8), dtype="<u8")[0])
        if n > size - 8:
            raise CheckpointError(f"{path}: header of {n} bytes does not fit in the file")
        try:
            header = json.loads(f.read(n).decode("utf-8"))
        except ValueError as e:
            raise CheckpointError(f"{path}: the header is not valid JSON ({e})") from None
    start = 8 + n
    out = {}
    for name, meta in header.items():
        if name == "__metadata__":
            continue
        dtype = meta.get("dtype")
        if dtype not in _DTYPE_BYTES:
            raise CheckpointError(f'unknown safetensors dtype "{dtype}"')
        if dtype == "F64":
            raise CheckpointError("F64 tensors are not supported")
        shape = [int(d) for d in meta.get("shape", [])]
        b, e = (int(x) for x in meta.get("data_offsets", [0, 0]))
        count = int(np.prod(shape)) if shape else 1
        if e - b != count * _DTYPE_BYTES[dtype] or start + e > size or b < 0:
            raise CheckpointError(f'{path}: tensor "{name}" has inconsistent data offsets')
        out[name] = (dtype, shape, start + b, start + e)
    return out, size


def _archive(model_dir: str):
    """name -> (file, dtype, shape, begin, end): model.safetensors, or the
    shards named by model.safetensors.index.json (src/safetensors.cpp:130-170)."""
    single = os.path.join(model_dir, "model.safetensors")
    index = os.path.join(model_dir, "model.safetensors.index.json")
    files = []
    if os.path.exists(single):
        files = [single]
    elif os.path.exists(index):
        with open(index) as f:
            wm = json.load(f).get("weight_map")
        if not isinstance(wm, dict):
            raise CheckpointError(f"{index} has no weight_map")
        files = [os.path.join(model_dir, s) for s in sorted(set(wm.values()))]
    else:
        raise CheckpointError(f"no model.safetensors or model.safetensors.index.json in {model_dir}")
    tensors = {}
    for path in files:
        hdr, _ = _read_header(path)
        for name, (dtype, shape, b, e) in hdr.items():
            if name in tensors:
                raise CheckpointError(f'tensor "{name}" appears in more than one shard')
            tensors[name] = (path, dtype, shape, b, e)
    return tensors


def load_checkpoint(model_dir: str, name: Optional[str] = None) -> WeightBlock:
    """A safetensors checkpoint directory (config.json + model.safetensors or
    an index of shards) as a read-order WeightBlock -- Model::load_weights
    (src/model.cu:112-213): every tensor BF16 with the shape its config
    implies; q/k/v and gate/up concatenated along the output rows; the output
    head is lm_head.weight when present, else the embedding, which then
    requires tie_word_embeddings. Tensors are read through memory maps."""
    with open(os.path.join(model_dir, "config.json")) as f:
        g = geometry_from_config(json.load(f), name or os.path.basename(os.path.normpath(model_dir)))
    tensors = _archive(model_dir)
    has_head = "lm_head.weight" in tensors
    if not has_head and not g.tie_word_embeddings:
        raise CheckpointError("the checkpoint has no lm_head.weight and config.json does not say the "
                              "embeddings are tied")
    offsets, total = block_layout(g, lm_head=has_head)
    data = np.zeros(total, dtype=np.uint16)
    maps: Dict[str, np.memmap] = {}

    def read(tname, shape):
        if tname not in tensors:
            raise CheckpointError(f'checkpoint has no tensor "{tname}"')
        path, dtype, got, b, e = tensors[tname]
        if dtype != "BF16":
            raise CheckpointError(f'tensor "{tname}" is {dtype} but this build computes in BF16')
        if list(got) != list(shape):
            raise CheckpointError(f'tensor "{tname}" has shape {got}, expected {list(shape)}')
        if path not in maps:
            maps[path] = np.memmap(path, dtype=np.uint8, mode="r")
        return maps[path][b:e].view(np.uint16)

    def place(group, parts):
        off, n = offsets[group]
        at = off
        for tname, shape in parts:
            arr = read(tname, shape)
            data[at:at + arr.size] = arr
            at += arr.size
        assert at - off == n, group

    h, q, kv, f_ = g.hidden_size, g.q_dim, g.kv_dim, g.intermediate_size
    place("embed", [("model.embed_tokens.weight", [g.vocab_size, h])])
    for l in range(g.num_layers):
        p, t = f"layers.{l}.", f"model.layers.{l}."
        place(p + "input_norm", [(t + "input_layernorm.weight", [h])])
        place(p + "qkv", [(t + "self_attn.q_proj.weight", [q, h]), (t + "self_attn.k_proj.weight", [kv, h]),
                          (t + "self_attn.v_proj.weight", [kv, h])])
        place(p + "o", [(t + "self_attn.o_proj.weight", [h, q])])
        place(p + "post_norm", [(t + "post_attention_layernorm.weight", [h])])
        place(p + "gate_up", [(t + "mlp.gate_proj.weight", [f_, h]), (t + "mlp.up_proj.weight", [f_, h])])
        place(p + "down", [(t + "mlp.down_proj.weight", [h, f_])])
    place("final_norm", [("model.norm.weight", [h])])
    if has_head:
        place("lm_head", [("lm_head.weight", [g.vocab_size, h])])
    return WeightBlock(geom=g, data=data, offsets=offsets)


_CACHE: Dict[Tuple[Geometry, int], WeightBlock] = {}


def cached(geom: Geometry, seed: int) -> WeightBlock:
    """generate(), memoised per process (the 1B block is 2.47 GB)."""
    key = (geom, seed)
    if key not in _CACHE:
        _CACHE[key] = generate(geom, seed)
    return _CACHE[key]

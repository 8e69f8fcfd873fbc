"""The safetensors checkpoint loader (lcr_b200.checkpoint.load_checkpoint)
against the writer and the reference loader's rules (src/config.cpp:40-184,
src/safetensors.cpp:99-170, src/model.cu:112-213): a round trip to the same
read-order block, sharded archives, an untied output head, and every refusal.
CPU only."""
import json
import os

import numpy as np
import pytest

from lcr_b200 import checkpoint as ck

SMALL = ck.small_geometry(layers=2, hidden=64, heads=4, kv_heads=2, head_dim=16, ffn=128, vocab=96,
                          name="small")


@pytest.fixture(scope="module")
def block():
    return ck.generate(SMALL, 3)


def test_round_trip_is_the_same_block(block, tmp_path):
    ck.write_safetensors(str(tmp_path), block)
    got = ck.load_checkpoint(str(tmp_path))
    assert got.offsets == block.offsets
    assert np.array_equal(got.data, block.data)
    assert got.lm_head_group == "embed"
    g = got.geom
    for f in ("hidden_size", "intermediate_size", "num_layers", "num_heads", "num_kv_heads", "head_dim",
              "vocab_size", "rms_norm_eps", "rope_theta", "rope_scaling", "rope_factor",
              "rope_original_max_position_embeddings", "tie_word_embeddings"):
        want = getattr(SMALL, f)
        # config.json floats are read as float32 (json get<float>)
        assert getattr(g, f) == (float(np.float32(want)) if isinstance(want, float) else want), f


def _tensors(model_dir):
    with open(os.path.join(model_dir, "model.safetensors"), "rb") as f:
        n = int(np.frombuffer(f.read(8), "<u8")[0])
        header = json.loads(f.read(n))
        body = f.read()
    return [(name, meta["dtype"], meta["shape"],
             np.frombuffer(body[meta["data_offsets"][0]:meta["data_offsets"][1]], np.uint8))
            for name, meta in sorted(header.items(), key=lambda kv: kv[1]["data_offsets"][0])]


def test_sharded_archive(block, tmp_path):
    src = tmp_path / "single"
    ck.write_safetensors(str(src), block)
    tensors = _tensors(str(src))
    out = tmp_path / "sharded"
    out.mkdir()
    (out / "config.json").write_text((src / "config.json").read_text())
    half = len(tensors) // 2
    weight_map = {}
    for i, part in enumerate((tensors[:half], tensors[half:])):
        name = f"model-{i + 1:05d}-of-00002.safetensors"
        ck.write_safetensors_file(str(out / name), part[::-1])  # any order inside a shard
        weight_map.update({t[0]: name for t in part})
    (out / "model.safetensors.index.json").write_text(json.dumps({"weight_map": weight_map}))
    got = ck.load_checkpoint(str(out))
    assert np.array_equal(got.data, block.data)


def test_untied_output_head(block, tmp_path):
    ck.write_safetensors(str(tmp_path), block)
    tensors = _tensors(str(tmp_path))
    head = ck.float_to_bf16_bits(np.random.default_rng(9).standard_normal(SMALL.vocab_size * SMALL.hidden_size)
                                 .astype(np.float32))
    ck.write_safetensors_file(str(tmp_path / "model.safetensors"),
                              tensors + [("lm_head.weight", "BF16", [SMALL.vocab_size, SMALL.hidden_size], head)])
    got = ck.load_checkpoint(str(tmp_path))
    assert got.lm_head_group == "lm_head"
    assert np.array_equal(got.view("lm_head"), head)
    assert np.array_equal(got.view("embed"), block.view("embed"))
    # the head follows the final norm in the read-order block
    assert got.offsets["lm_head"][0] > got.offsets["final_norm"][0]


def _edit(tmp_path, block, config=None, drop=None, retype=None, reshape=None):
    ck.write_safetensors(str(tmp_path), block)
    if config:
        doc = json.loads((tmp_path / "config.json").read_text())
        doc.update(config)
        doc = {k: v for k, v in doc.items() if v is not None}
        (tmp_path / "config.json").write_text(json.dumps(doc))
    tensors = _tensors(str(tmp_path))
    out = []
    for name, dtype, shape, raw in tensors:
        if name == drop:
            continue
        if name == retype:
            raw = ck.bf16_bits_to_float(raw.view(np.uint16)).view(np.uint8)
            dtype = "F32"
        if name == reshape:
            shape = [shape[0] * shape[1] // 2, 2] if len(shape) == 2 else shape
        out.append((name, dtype, shape, raw))
    ck.write_safetensors_file(str(tmp_path / "model.safetensors"), out)
    return str(tmp_path)


@pytest.mark.parametrize("edit, message", [
    (dict(config={"model_type": "mistral"}), "only implements the Llama architecture"),
    (dict(config={"hidden_size": None}), 'missing the integer field "hidden_size"'),
    (dict(config={"num_key_value_heads": 3}), "must be a multiple of num_key_value_heads"),
    (dict(config={"hidden_act": "gelu"}), "only the SiLU/SwiGLU MLP"),
    (dict(config={"attention_bias": True}), "with bias are not implemented"),
    (dict(config={"rope_scaling": {"rope_type": "linear", "factor": 2.0}}), "only llama3 RoPE scaling"),
    (dict(config={"rope_theta": 1.0}), "rope_theta must be greater than one"),
    (dict(config={"tie_word_embeddings": False}), "no lm_head.weight"),
    (dict(drop="model.layers.1.mlp.up_proj.weight"), 'no tensor "model.layers.1.mlp.up_proj.weight"'),
    (dict(retype="model.layers.0.self_attn.k_proj.weight"), "is F32 but this build computes in BF16"),
    (dict(reshape="model.layers.0.self_attn.o_proj.weight"), "has shape"),
])
def test_refusals(block, tmp_path, edit, message):
    d = _edit(tmp_path, block, **edit)
    with pytest.raises(ck.CheckpointError, match=message):
        ck.load_checkpoint(d)


def test_config_defaults_and_rope_type_field():
    doc = dict(hidden_size=64, intermediate_size=128, num_hidden_layers=1, num_attention_heads=4,
               vocab_size=32, max_position_embeddings=512)
    g = ck.geometry_from_config(doc)
    assert g.num_kv_heads == 4 and g.head_dim == 16  # MHA; head_dim implied
    assert g.rms_norm_eps == pytest.approx(1e-5) and g.rope_theta == 500000.0
    assert not g.rope_scaling and g.tie_word_embeddings
    g = ck.geometry_from_config(dict(doc, rope_scaling={"type": "llama3", "factor": 8.0}))
    assert g.rope_scaling and g.rope_factor == 8.0 and g.rope_original_max_position_embeddings == 8192
    g = ck.geometry_from_config(dict(doc, rope_scaling={"rope_type": "default"}))
    assert not g.rope_scaling


def test_missing_archive_and_truncated_file(tmp_path, block):
    ck.write_safetensors(str(tmp_path), block)
    os.rename(tmp_path / "model.safetensors", tmp_path / "other.safetensors")
    with pytest.raises(ck.CheckpointError, match="no model.safetensors"):
        ck.load_checkpoint(str(tmp_path))
    (tmp_path / "model.safetensors").write_bytes(b"\x05\x00")
    with pytest.raises(ck.CheckpointError, match="too small"):
        ck.load_checkpoint(str(tmp_path))

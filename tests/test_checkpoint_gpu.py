"""A safetensors checkpoint through the loader and the C ABI: the tiny model
written and loaded back decodes bit for bit as the generated block does, and
an untied output head (lm_head.weight) is the head the decode step reads
(against the oracle, which reads the same head)."""
import numpy as np
import pytest

import oracle
from lcr_b200 import checkpoint as ck
from lcr_b200 import runtime as rt

pytestmark = pytest.mark.gpu

torch = pytest.importorskip("torch")
if not torch.cuda.is_available():
    pytest.skip("needs a CUDA device", allow_module_level=True)


def test_loaded_checkpoint_decodes_like_the_block(tmp_path):
    block = ck.cached(ck.TINY, 0)
    ck.write_safetensors(str(tmp_path), block)
    loaded = ck.load_checkpoint(str(tmp_path))
    prompt = ck.prompt_ids(0, 24)
    a = rt.Model(block, max_seq=64)
    b = rt.Model(loaded, max_seq=64)
    a.prefill(prompt)
    b.prefill(prompt)
    assert np.array_equal(a.logits_to_host(), b.logits_to_host())
    first = int(np.argmax(a.logits_to_host()))
    assert a.generate_greedy(first, 8).tolist() == b.generate_greedy(first, 8).tolist()


def test_untied_head_is_read(tmp_path):
    block = ck.cached(ck.TINY, 0)
    g = block.geom
    offsets, total = ck.block_layout(g, lm_head=True)
    data = np.zeros(total, np.uint16)
    for name, (off, n) in block.offsets.items():
        data[offsets[name][0]:offsets[name][0] + n] = block.view(name)
    head = ck.float_to_bf16_bits(np.random.default_rng(4).standard_normal(g.vocab_size * g.hidden_size)
                                 .astype(np.float32) * np.float32(0.02))
    data[offsets["lm_head"][0]:offsets["lm_head"][0] + head.size] = head
    untied = ck.WeightBlock(geom=g, data=data, offsets=offsets)
    ck.write_safetensors(str(tmp_path), untied)
    loaded = ck.load_checkpoint(str(tmp_path))
    assert loaded.lm_head_group == "lm_head"
    prompt = ck.prompt_ids(1, 20)
    m = rt.Model(loaded, max_seq=64)
    m.prefill(prompt)
    got = m.logits_to_host()
    want = oracle.Model(loaded, 64).prefill(prompt, 0, oracle.MODE_BF16)
    tied = oracle.Model(block, 64).prefill(prompt, 0, oracle.MODE_BF16)
    assert np.abs(got - want).max() <= 2e-2
    assert np.abs(got - tied).max() > 0.1  # a different head, visibly

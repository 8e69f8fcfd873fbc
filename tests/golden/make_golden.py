"""Regenerates the golden fixtures in tests/golden/ (run in the build container:
it imports transformers and, when present, the reference sources' compiled
RoPE function in oracle/_ref).

* tiny_seed0_hf.npz -- transformers' LlamaForCausalLM (fp32, eager attention)
  on the seed-0 tiny random-init checkpoint: the 32-id prompt, 16 greedy
  tokens, full logits of the first two generation steps, the top-64 logits of
  every step and the residual-stream taps of the first step (the taps
  tools/dump_reference.py:68-79 of the reference records). It pins the fp32
  oracle end to end; the reference ships no golden logits of its own.
* ref_rope.json -- the reference's own compute_rope_inv_freq
  (src/config.cpp:223-259, compiled from the reference tree into oracle/_ref)
  for the Llama-3.2-1B config (llama3 scaling) and an unscaled config, as
  float32 bit patterns.

Usage: python tests/golden/make_golden.py
"""
import json
import os
import sys

import numpy as np

HERE = os.path.dirname(os.path.abspath(__file__))
REPO = os.path.dirname(os.path.dirname(HERE))
sys.path.insert(0, os.path.join(REPO, "llama-cuda-runtime_b200"))
sys.path.insert(0, REPO)

from lcr_b200 import checkpoint as ck  # noqa: E402

PROMPT_LEN = 32
GEN = 16
TOPK = 64


def hf_model(block):
    import torch
    from transformers import LlamaConfig, LlamaForCausalLM

    g = block.geom
    cfg = LlamaConfig(**{k: v for k, v in g.config_json().items()
                         if k not in ("architectures", "model_type", "torch_dtype")})
    cfg._attn_implementation = "eager"
    torch.manual_seed(0)
    model = LlamaForCausalLM(cfg).float().eval()
    f = lambda name, shape: torch.from_numpy(
        ck.bf16_bits_to_float(block.view(name)).reshape(shape).copy())
    h, qd, kvd, F = g.hidden_size, g.q_dim, g.kv_dim, g.intermediate_size
    with torch.no_grad():
        model.model.embed_tokens.weight.copy_(f("embed", (g.vocab_size, h)))
        for l, layer in enumerate(model.model.layers):
            p = f"layers.{l}."
            qkv = f(p + "qkv", (g.qkv_rows, h))
            layer.self_attn.q_proj.weight.copy_(qkv[:qd])
            layer.self_attn.k_proj.weight.copy_(qkv[qd:qd + kvd])
            layer.self_attn.v_proj.weight.copy_(qkv[qd + kvd:])
            layer.self_attn.o_proj.weight.copy_(f(p + "o", (h, qd)))
            gu = f(p + "gate_up", (2 * F, h))
            layer.mlp.gate_proj.weight.copy_(gu[:F])
            layer.mlp.up_proj.weight.copy_(gu[F:])
            layer.mlp.down_proj.weight.copy_(f(p + "down", (h, F)))
            layer.input_layernorm.weight.copy_(f(p + "input_norm", (h,)))
            layer.post_attention_layernorm.weight.copy_(f(p + "post_norm", (h,)))
        model.model.norm.weight.copy_(f("final_norm", (h,)))
        model.tie_weights()
    assert model.lm_head.weight.data_ptr() == model.model.embed_tokens.weight.data_ptr()
    return model


def make_tiny():
    import torch

    block = ck.generate(ck.TINY, 0)
    model = hf_model(block)
    prompt = ck.prompt_ids(0, PROMPT_LEN)
    ids = torch.from_numpy(prompt.astype(np.int64))[None]
    full_logits, top_ids, top_vals, tokens = [], [], [], []
    taps = None
    with torch.no_grad():
        out = model(ids, use_cache=True, output_hidden_states=True)
        past = out.past_key_values
        logits = out.logits[0, -1].float().numpy()
        # hidden_states: embed, layer_0 .. layer_{n-2}, final norm applied to last
        hs = [t[0, -1].float().numpy() for t in out.hidden_states]
        taps = np.stack(hs)
        for step in range(GEN + 1):
            order = np.argsort(-logits, kind="stable")[:TOPK]
            top_ids.append(order.astype(np.int32))
            top_vals.append(logits[order].astype(np.float32))
            if step < 2:
                full_logits.append(logits.astype(np.float32))
            if step == GEN:
                break
            nxt = int(np.argmax(logits))
            tokens.append(nxt)
            out = model(torch.tensor([[nxt]]), past_key_values=past, use_cache=True)
            past = out.past_key_values
            logits = out.logits[0, -1].float().numpy()
    np.savez_compressed(
        os.path.join(HERE, "tiny_seed0_hf.npz"), prompt=prompt, greedy=np.array(tokens, np.int32),
        logits_first2=np.stack(full_logits), top_ids=np.stack(top_ids), top_vals=np.stack(top_vals),
        taps_prompt_last=taps.astype(np.float32))
    print("wrote tiny_seed0_hf.npz; greedy", tokens)


def make_rope():
    import oracle

    unscaled = ck.Geometry(hidden_size=2048, intermediate_size=5632, num_layers=22,
                           num_heads=32, num_kv_heads=32, head_dim=64, vocab_size=32000,
                           rope_theta=10000.0, rope_scaling=False)
    out = {}
    for name, g in (("llama-3.2-1b", ck.LLAMA_3_2_1B), ("unscaled", unscaled)):
        doc = g.config_json()
        ref = oracle.ref_rope_inv_freq(json.dumps(doc))
        if ref is None:
            print("reference sources not built (oracle/_ref); ref_rope.json left as is")
            return
        out[name] = {"config": doc, "inv_freq_bits": [int(v) for v in ref.view(np.uint32)]}
    with open(os.path.join(HERE, "ref_rope.json"), "w") as f:
        json.dump(out, f, indent=1)
    print("wrote ref_rope.json")


if __name__ == "__main__":
    make_rope()
    make_tiny()

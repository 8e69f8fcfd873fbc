"""A 2-layer model of the Llama-3.2-1B geometry (hidden 2048, 32 query / 8 KV
heads of 64, ffn 8192, vocab 128256; seed 7) against committed oracle
fixtures (tests/golden/make_golden_1b.py): the 2048-row tcgen05 prefill chunk
with its attention at 4 query heads per KV head, a 1300 + 199 split of the
prompt, and one batched decode step of 8 sequences (contexts of 1 .. 1024
ids) through the 1B-shape projections of the batch step.

Gates. At this geometry the bf16-storage algorithm itself (the reference's)
is 0.033-0.042 max-abs from the fp32 evaluation, above the north-star 3e-2,
so the gates are relative, as for the full 1B model: max-abs against fp32 at
most 1.5x the bf16 algorithm's own distance from fp32, and cosine >= 0.999.
Against the bf16-storage oracle the same 1.5x bound: two bf16 evaluations
whose roundings fall in other places drift apart about as far as each is
from fp32 -- the oracle's own per-token and chunked evaluations of the 64-
and 300-id contexts of b8_1b2l.npz differ by 0.024 and 0.021."""
import os

import numpy as np
import pytest

from lcr_b200 import checkpoint as ck
from lcr_b200 import runtime as rt

pytestmark = pytest.mark.gpu

torch = pytest.importorskip("torch")
if not torch.cuda.is_available():
    pytest.skip("needs a CUDA device", allow_module_level=True)

import dataclasses  # noqa: E402

GOLDEN = os.path.join(os.path.dirname(os.path.abspath(__file__)), "golden")
GEOM = dataclasses.replace(ck.LLAMA_3_2_1B, num_layers=2, name="llama-3.2-1b-2layer")
SEED = 7
SLACK = 1.5
MIN_COS = 0.999


def cos(a, b):
    a, b = np.asarray(a, np.float64), np.asarray(b, np.float64)
    return float(a @ b / np.linalg.norm(a) / np.linalg.norm(b))


@pytest.fixture(scope="module")
def model():
    block = ck.cached(GEOM, SEED)
    return block, rt.upload_block(block)


def gate(got, f32_at, b16_at, idx, label):
    """got: the GPU's full logits; f32_at / b16_at: the oracle's over idx
    (f32_at may be the full vector, then idx selects)."""
    f32_sub = f32_at[idx] if f32_at.size == got.size else f32_at
    ref_dist = float(np.abs(b16_at - f32_sub).max())
    d32 = float(np.abs(got[idx] - f32_sub).max())
    d16 = float(np.abs(got[idx] - b16_at).max())
    c = cos(got, f32_at) if f32_at.size == got.size else cos(got[idx], f32_sub)
    print(f"{label}: max-abs vs fp32 {d32:.4f} (bf16 algorithm {ref_dist:.4f}), vs bf16 {d16:.4f}, "
          f"cos {c:.6f}")
    assert c >= MIN_COS, label
    assert d32 <= SLACK * ref_dist, label
    assert d16 <= SLACK * ref_dist, label
    if f32_at.size == got.size:
        full = float(np.abs(got - f32_at).max())
        assert full <= SLACK * ref_dist, label


@pytest.mark.parametrize("paged", [False, True])
def test_prefill_chunk_2048_and_split(model, paged):
    block, wdev = model
    fx = np.load(os.path.join(GOLDEN, "p2_1b2l.npz"))
    prompt = fx["prompt"]
    kw = dict(max_seq=2048 + 16, paged=paged, page_size=16, page_order_seed=5 if paged else 0)
    m = rt.Model(block, wdev, **kw)
    m.prefill(prompt)
    gate(m.logits_to_host(), fx["full_fp32"], fx["full_bf16"], fx["full_idx"], f"2048-row chunk paged={paged}")
    s = rt.Model(block, wdev, **kw)
    s.prefill(prompt[:1300])
    s.prefill(prompt[1300:1499])
    gate(s.logits_to_host(), fx["split_fp32"], fx["split_bf16"], fx["split_idx"], f"1300 + 199 paged={paged}")
    m.close()
    s.close()


def test_batch_prefill_chunk_2048(model):
    """The same chunk through lcr_batch_prefill on a slot of a batch pool."""
    block, wdev = model
    fx = np.load(os.path.join(GOLDEN, "p2_1b2l.npz"))
    bt = rt.Batch(block, wdev, max_batch=2, max_seq=2048 + 16, page_size=16, pool_pages=300)
    order = np.random.default_rng(3).permutation(300)
    bt.set_pages(1, order[:129])
    bt.prefill(1, fx["prompt"], 0)
    gate(bt.logits(1), fx["full_fp32"], fx["full_bf16"], fx["full_idx"], "batch slot 1, 2048-row chunk")
    bt.close()


def test_batch_step_8_slots(model):
    """8 sequences: each context's first n-1 ids prefilled on its slot's
    pages, then one batched step of the last ids at positions n-1."""
    block, wdev = model
    fx = np.load(os.path.join(GOLDEN, "b8_1b2l.npz"))
    lengths = [int(n) for n in fx["lengths"]]
    page = 16
    per = [(n + page - 1) // page for n in lengths]
    bt = rt.Batch(block, wdev, max_batch=8, max_seq=1024 + 16, page_size=page, pool_pages=sum(per) + 8)
    order = np.random.default_rng(11).permutation(sum(per) + 8)
    at = 0
    for slot, n in enumerate(lengths):
        bt.set_pages(slot, order[at:at + per[slot]])
        at += per[slot]
        ids = fx[f"ids{slot}"]
        if n > 1:
            bt.prefill(slot, ids[:-1], 0)
    bt.step([int(fx[f"ids{s}"][-1]) for s in range(8)], [n - 1 for n in lengths])
    for slot, n in enumerate(lengths):
        gate(bt.logits(slot), fx[f"fp32_{slot}"], fx[f"bf16_{slot}"], fx[f"idx{slot}"],
             f"batched slot {slot} (context {n})")
    bt.close()

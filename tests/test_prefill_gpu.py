"""Chunked prefill (lcr_batch_prefill: tcgen05 projections over the chunk's
rows, causal flash attention over the slot's pages) through the C ABI
against the oracle, which evaluates the same prompt one position at a time
(the decode step's maths): the last row's logits after each chunk, then
decode steps that read the K/V the prefill wrote. Tolerances are the
north-star ones used for the batched path: max-abs 3e-2 and cosine 0.999
against fp32, 2e-2 against the bf16-rounding oracle."""
import numpy as np
import pytest

import oracle
from lcr_b200 import checkpoint as ck
from lcr_b200 import runtime as rt

pytestmark = pytest.mark.gpu

torch = pytest.importorskip("torch")
if not torch.cuda.is_available():
    pytest.skip("needs a CUDA device", allow_module_level=True)

MAX_ABS = 3e-2
MIN_COS = 0.999
PAGE = 16

# tiny (head_dim 64, 2 query heads per KV head) and a wide-head geometry
# (head_dim 128, 8 query heads per KV head) that the 1B model does not cover
WIDE = ck.small_geometry(layers=2, hidden=256, heads=8, kv_heads=1, head_dim=128, ffn=1024, vocab=4096,
                         name="wide")


def cos(a, b):
    a, b = np.asarray(a, np.float64), np.asarray(b, np.float64)
    return float(a @ b / np.linalg.norm(a) / np.linalg.norm(b))


@pytest.fixture(scope="module", params=["tiny", "wide"])
def model(request):
    geom = ck.TINY if request.param == "tiny" else WIDE
    block = ck.cached(geom, 0) if request.param == "tiny" else ck.generate(geom, 5)
    return request.param, block, rt.upload_block(block)


def _check(got, l32, l16, what):
    abs32 = float(np.abs(got - l32).max())
    abs16 = float(np.abs(got - l16).max())
    c = cos(got, l32)
    assert abs32 <= MAX_ABS and c >= MIN_COS and abs16 <= 2e-2, (what, abs32, c, abs16)


@pytest.mark.parametrize("chunks", [(24, 16), (150,), (7, 33, 1)])
def test_prefill_chunks_then_decode_match_oracle(model, chunks):
    name, block, wdev = model
    total = sum(chunks)
    max_seq = 224
    per = max_seq // PAGE
    pool = 3 * per
    bt = rt.Batch(block, wdev, max_batch=4, max_seq=max_seq, page_size=PAGE, pool_pages=pool)
    slot = 2
    bt.set_pages(slot, oracle.page_permutation(pool, 17)[:per])
    bt.set_sampling(slot, 0.0)
    vocab = block.geom.vocab_size
    prompt = np.asarray(ck.prompt_ids(300 + total, total + 8), dtype=np.int64) % vocab
    r16 = oracle.Model(block, max_seq)
    r32 = oracle.Model(block, max_seq)
    start = 0
    for n in chunks:
        bt.prefill(slot, prompt[start:start + n], start)
        for p in range(start, start + n):
            l16 = r16.decode(int(prompt[p]), p, oracle.MODE_BF16)
            l32 = r32.decode(int(prompt[p]), p, oracle.MODE_FP32)
        got = bt.logits(slot)
        _check(got, l32, l16, f"{name} chunk ending at {start + n}")
        ids = bt.read(4)
        assert int(ids[slot]) == int(np.argmax(got))
        start += n
    # Decode on from the prefilled cache: a one-slot step is row 0 and reads
    # slot 0's page table, so slot 0 gets the prefilled pages.
    bt.set_pages(0, oracle.page_permutation(pool, 17)[:per])
    bt.set_sampling(0, 0.0)
    for p in range(total, total + 4):
        bt.step([int(prompt[p])], [p])
        l16 = r16.decode(int(prompt[p]), p, oracle.MODE_BF16)
        l32 = r32.decode(int(prompt[p]), p, oracle.MODE_FP32)
        _check(bt.logits(0), l32, l16, f"{name} decode at {p}")
    bt.close()


def test_batched_decode_wide_heads_match_oracle(model):
    """The batched decode step (tensor-pipe attention, persistent work items)
    on both geometries: staggered slots, shuffled pages, per-sequence parity."""
    name, block, wdev = model
    slots, max_seq, steps = 6, 96, 40
    per = max_seq // PAGE
    pool = slots * per + 3
    bt = rt.Batch(block, wdev, max_batch=slots, max_seq=max_seq, page_size=PAGE, pool_pages=pool)
    order = oracle.page_permutation(pool, 23)
    vocab = block.geom.vocab_size
    seqs = []
    for s in range(slots):
        bt.set_pages(s, order[s * per:(s + 1) * per])
        bt.set_sampling(s, 0.0)
        seqs.append(np.asarray(ck.prompt_ids(500 + s, max_seq), dtype=np.int64) % vocab)
    for t in range(steps):
        n = min(slots, t + 1)
        bt.step([int(seqs[s][t - s]) for s in range(n)], [t - s for s in range(n)])
    for s in range(slots):
        r16 = oracle.Model(block, max_seq)
        r32 = oracle.Model(block, max_seq)
        for p in range(steps - s):
            l16 = r16.decode(int(seqs[s][p]), p, oracle.MODE_BF16)
            l32 = r32.decode(int(seqs[s][p]), p, oracle.MODE_FP32)
        _check(bt.logits(s), l32, l16, f"{name} slot {s}")
    bt.close()


def test_prefill_rejects_bad_inputs(model):
    name, block, wdev = model
    bt = rt.Batch(block, wdev, max_batch=2, max_seq=32, page_size=PAGE, pool_pages=4)
    with pytest.raises(rt.LcrError):
        bt.prefill(0, [1, 2, 3], 30)  # positions 30..32 outside max_seq 32
    with pytest.raises(rt.LcrError):
        bt.prefill(2, [1], 0)  # slot 2 of 2
    with pytest.raises(rt.LcrError):
        bt.prefill(0, [block.geom.vocab_size], 0)  # token outside the vocabulary
    with pytest.raises(rt.LcrError):
        bt.prefill(0, [1, 2, 3], 0)  # slot 0 has no pages yet
    bt.set_pages(1, [2])
    with pytest.raises(rt.LcrError):
        bt.prefill(1, list(range(1, 18)), 0)  # 17 positions, one 16-position page
    bt.prefill(1, list(range(1, 17)), 0)
    with pytest.raises(rt.LcrError):
        bt.step([1, 1], [16, 16])  # row 0 (slot 0) has no pages, row 1's page ends at 15
    bt.close()


def test_batcher_with_prefill_generates_oracle_greedy_ids(model):
    """Continuous batching end to end: sequences admitted into 2 slots with
    their prompts prefilled in 32-token chunks, greedy decoding with device
    token feedback, retirement and slot compaction; every sequence's ids
    (the prefill's sample, then one per step) are the oracle's greedy
    continuation of its prompt -- up to a near tie, after which the two
    continuations may legitimately part."""
    from lcr_b200 import scheduler as sch
    name, block, wdev = model
    vocab = block.geom.vocab_size
    lengths, target, max_seq = [40, 70, 25, 33], 5, 96
    per = max_seq // PAGE
    bt = rt.Batch(block, wdev, max_batch=2, max_seq=max_seq, page_size=PAGE, pool_pages=2 * per + 2)
    cb = sch.ContinuousBatcher(bt, page_size=PAGE, pool_pages=2 * per + 2, page_seed=9, temperature=0.0,
                               prefill_chunk=32, record=True)
    seqs = []
    for i, n in enumerate(lengths):
        prompt = (np.asarray(ck.prompt_ids(700 + i, n), dtype=np.int64) % vocab).astype(np.int32)
        seqs.append(sch.Sequence(sid=i, context=n, target=target, seed=i, prompt=prompt))
        cb.submit(seqs[-1])
    for _ in range(40):
        cb.fill()
        if cb.step() == 0 and not cb.waiting:
            break
    assert cb.finished == len(lengths)
    for q in seqs:
        assert len(q.tokens) == target + 1
        r = oracle.Model(block, max_seq)
        for p in range(q.context):
            logits = r.decode(int(q.prompt[p]), p, oracle.MODE_BF16)
        for k, got in enumerate(q.tokens):
            want = int(np.argmax(logits))
            if got != want:
                top2 = np.sort(logits)[-2:]
                assert top2[1] - top2[0] < 2e-2, (name, q.sid, k, got, want)
                break
            logits = r.decode(got, q.context + k, oracle.MODE_BF16)
    bt.close()


def test_persistent_projections_match_per_tile_kernel():
    """Prefill chunks of a 2-layer model with the 1B geometry: 1300 rows
    (every projection on 256-row tiles of the persistent kernel, the last one
    partial), then 199 rows (gate/up on one 256-row tile, the rest split-K).
    The persistent projection kernel (two TMEM accumulators, one CTA per SM
    walking tiles) and the one-CTA-per-tile kernel with 128-row tiles (option
    bit 4) must give bit-identical logits, through the second chunk and a
    decode step that read the first chunk's K/V."""
    import dataclasses
    geom = dataclasses.replace(ck.LLAMA_3_2_1B, num_layers=2)
    block = ck.generate(geom, 3)
    wdev = rt.upload_block(block)
    max_seq = 1536
    per = max_seq // PAGE
    prompt = np.asarray(ck.prompt_ids(41, 1500), dtype=np.int64) % geom.vocab_size
    got = []
    for flags in (0, 4):
        bt = rt.Batch(block, wdev, max_batch=1, max_seq=max_seq, page_size=PAGE, pool_pages=per, flags=flags)
        bt.set_pages(0, oracle.page_permutation(per, 5))
        bt.set_sampling(0, 0.0)
        bt.prefill(0, prompt[:1300], 0)
        first = bt.logits(0).copy()
        bt.prefill(0, prompt[1300:1499], 1300)
        second = bt.logits(0).copy()
        bt.step([int(prompt[1499])], [1499])
        got.append((first, second, bt.logits(0).copy()))
        bt.close()
    for a, b, what in zip(got[0], got[1], ("first chunk", "second chunk", "decode")):
        assert np.isfinite(a).all() and np.array_equal(a, b), what

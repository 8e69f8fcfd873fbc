"""Batched decode (lcr_batch_*) through the C ABI against the oracle: every
slot is a separate sequence with its own length and shuffled KV pages, decoded
one token per step with the tensor-core projections; each slot's logits must
match the oracle's evaluation of that sequence alone (the north-star
tolerances: max-abs 3e-2 and cosine 0.999 against fp32), greedy picks must be
the oracle's argmax, and top-k/top-p sampling with Philox must pick exactly
what the oracle's sampler picks from the same logits."""
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


def cos(a, b):
    a, b = np.asarray(a, np.float64), np.asarray(b, np.float64)
    return float(a @ b / np.linalg.norm(a) / np.linalg.norm(b))


@pytest.fixture(scope="module")
def tiny():
    block = ck.cached(ck.TINY, 0)
    return block, rt.upload_block(block)


def _run_staggered(bt, slots, steps, seqs):
    """Slot s joins at step s: at step t the first min(slots, t + 1) slots
    decode, slot s at position t - s, teacher-forced with seqs[s]."""
    for t in range(steps):
        n = min(slots, t + 1)
        toks = [int(seqs[s][t - s]) for s in range(n)]
        pos = [t - s for s in range(n)]
        bt.step(toks, pos)
    bt.sync()


@pytest.mark.parametrize("slots", [20, 64])
def test_batch_matches_oracle_per_sequence(tiny, slots):
    block, wdev = tiny
    steps = 48 if slots == 20 else 70
    max_seq = 96
    pool = slots * (max_seq // PAGE) + 7
    bt = rt.Batch(block, wdev, max_batch=slots, max_seq=max_seq, page_size=PAGE, pool_pages=pool)
    order = oracle.page_permutation(pool, 31)
    per = max_seq // PAGE
    seqs = []
    for s in range(slots):
        bt.set_pages(s, order[s * per:(s + 1) * per])
        bt.set_sampling(s, 0.0)
        seqs.append(ck.prompt_ids(1000 + s, max_seq))
    _run_staggered(bt, slots, steps, seqs)
    got_ids = bt.read(slots)
    worst = dict(abs32=0.0, cos=1.0, abs16=0.0)
    for s in range(slots):
        length = steps - s
        if length <= 0:
            continue
        r16 = oracle.Model(block, max_seq)
        r32 = oracle.Model(block, max_seq)
        for p in range(length):
            l16 = r16.decode(int(seqs[s][p]), p, oracle.MODE_BF16)
            l32 = r32.decode(int(seqs[s][p]), p, oracle.MODE_FP32)
        got = bt.logits(s)
        worst["abs32"] = max(worst["abs32"], float(np.abs(got - l32).max()))
        worst["abs16"] = max(worst["abs16"], float(np.abs(got - l16).max()))
        worst["cos"] = min(worst["cos"], cos(got, l32))
        assert int(got_ids[s]) == int(np.argmax(got)), f"slot {s}: greedy id is not the argmax"
        if int(got_ids[s]) != oracle.argmax(l16):
            top2 = np.sort(l16)[-2:]
            assert top2[1] - top2[0] < 2 * np.abs(got - l16).max(), f"slot {s}: greedy id differs"
    print(f"{slots} slots: {worst}")
    assert worst["abs32"] <= MAX_ABS and worst["cos"] >= MIN_COS
    assert worst["abs16"] <= 2e-2
    bt.close()


def test_batch_sampling_is_the_oracle_sampler(tiny):
    """Per-slot temperature / top-k / top-p with Philox uniforms of (seed,
    position): the picks equal the oracle sampler's on the same logits."""
    block, wdev = tiny
    slots, max_seq = 24, 64
    pool = slots * (max_seq // PAGE)
    bt = rt.Batch(block, wdev, max_batch=slots, max_seq=max_seq, page_size=PAGE, pool_pages=pool)
    params = []
    for s in range(slots):
        bt.set_pages(s, list(range(s * (max_seq // PAGE), (s + 1) * (max_seq // PAGE))))
        t, k, p = [(0.8, 50, 0.9), (1.0, 0, 0.95), (0.5, 5, 1.0), (1.3, 200, 0.7)][s % 4]
        seed = 0x9E3779B97F4A7C15 ^ (s * 7919)
        bt.set_sampling(s, t, k, p, seed)
        params.append((t, k, p, seed))
    seqs = [ck.prompt_ids(2000 + s, max_seq) for s in range(slots)]
    for t in range(12):
        bt.step([int(seqs[s][t]) for s in range(slots)], [t] * slots)
    ids = bt.read(slots)
    for s in range(slots):
        t, k, p, seed = params[s]
        logits = bt.logits(s)
        u = oracle.philox_uniform(seed & 0xFFFFFFFFFFFFFFFF, 11, 0)
        assert int(ids[s]) == oracle.sample(logits, t, k, p, u), f"slot {s}"
    bt.close()


def test_batch_rejects_bad_inputs(tiny):
    block, wdev = tiny
    bt = rt.Batch(block, wdev, max_batch=4, max_seq=32, page_size=PAGE, pool_pages=8)
    with pytest.raises(rt.LcrError) as e:
        bt.set_pages(0, [0, 8])  # page 8 is outside a pool of 8
    assert e.value.status == 5
    with pytest.raises(rt.LcrError):
        bt.step([1, 2], [0, 32])  # position 32 is outside max_seq 32
    with pytest.raises(rt.LcrError):
        bt.step([1] * 5, [0] * 5)  # 5 slots in a batch of 4
    bt.close()


def test_device_feedback_equals_host_round_trip(tiny):
    """tokens=None (each slot continues with its last sample, on the device)
    gives the same steps as reading the samples back and passing them in."""
    block, wdev = tiny
    slots, max_seq = 12, 48
    runs = []
    for feedback in (True, False):
        bt = rt.Batch(block, wdev, max_batch=slots, max_seq=max_seq, page_size=PAGE,
                      pool_pages=slots * (max_seq // PAGE))
        for s in range(slots):
            bt.set_pages(s, list(range(s * (max_seq // PAGE), (s + 1) * (max_seq // PAGE))))
            bt.set_sampling(s, 0.9, 40, 0.95, 1234 + s)
        bt.step([int(t) for t in ck.prompt_ids(77, slots)], [0] * slots)
        ids = []
        for t in range(1, 20):
            if feedback:
                bt.step(None, [t] * slots)
            else:
                bt.step(bt.read(slots), [t] * slots)
            ids.append(bt.read(slots).copy())
        runs.append((np.array(ids), bt.logits(slots - 1)))
        bt.close()
    assert np.array_equal(runs[0][0], runs[1][0])
    assert np.array_equal(runs[0][1], runs[1][1])


def test_scheduler_runs_config4_shape_on_tiny(tiny):
    """The continuous batcher on the device: staggered sequences with
    synthetic contexts, arrivals filling freed slots, sampled steps."""
    from lcr_b200 import scheduler as sch
    block, wdev = tiny
    slots, max_seq = 16, 256
    pool = (slots + 2) * (max_seq // PAGE)
    bt = rt.Batch(block, wdev, max_batch=slots, max_seq=max_seq, page_size=PAGE, pool_pages=pool)
    cb = sch.ContinuousBatcher(bt, page_size=PAGE, pool_pages=pool, page_seed=3)
    rng = np.random.default_rng(3)
    for q in sch.config4_workload(rng, slots, 24, 16, 200):
        cb.submit(q)
    sid = slots
    decoded = 0
    for _ in range(60):
        new, sid = sch.config4_arrivals(rng, sid, 2.0, 24, 16, 200)
        for q in new:
            cb.submit(q)
        cb.fill()
        decoded += cb.step()
    ids = bt.read(cb.active())
    assert cb.finished >= 30 and decoded == 60 * slots
    assert np.all((ids >= 0) & (ids < block.geom.vocab_size))
    bt.close()


def test_weights_outside_the_device_are_rejected():
    """A context reads its weights directly, so lcr_batch_create refuses
    weights that are not in its device's memory (here: pageable host memory)
    instead of letting the first kernel fault; with two GPUs, weights on the
    other GPU are refused too."""
    block = ck.cached(ck.TINY, 0)
    host = torch.from_numpy(block.data.view(np.int16))
    with pytest.raises(rt.LcrError):
        rt.Batch(block, host, max_batch=2, max_seq=64, page_size=16, pool_pages=8)
    if torch.cuda.device_count() >= 2:
        w0 = rt.upload_block(block, 0)
        with pytest.raises(ValueError):
            rt.Batch(block, w0, device=1, max_batch=2, max_seq=64, page_size=16, pool_pages=8)

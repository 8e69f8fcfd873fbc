"""Continuous-batching host logic (lcr_b200.scheduler) on CPU, over a fake
batch that records the calls a runtime.Batch would receive."""
import os
import sys

import numpy as np
import pytest

sys.path.insert(0, os.path.join(os.path.dirname(os.path.dirname(os.path.abspath(__file__))),
                                "llama-cuda-runtime_b200"))
from lcr_b200 import scheduler as S  # noqa: E402


class FakeBatch:
    def __init__(self, slots=8):
        self.max_batch = slots
        self.calls = []
        self.pages = {}
        self.next = np.arange(slots, dtype=np.int32) + 100

    def set_pages(self, slot, pages):
        self.pages[slot] = list(pages)
        self.calls.append(("pages", slot, len(pages)))

    def set_sampling(self, slot, *args):
        self.calls.append(("sampling", slot) + tuple(args))

    def fill_kv(self, slot, length, seed):
        self.calls.append(("fill", slot, length, seed))

    def step(self, tokens, positions):
        self.calls.append(("step", None if tokens is None else list(tokens), list(positions)))

    def read(self, n):
        return self.next[:n]


def test_page_pool_round_trip_and_exhaustion():
    pool = S.PagePool(10, seed=5)
    a = pool.take(4)
    b = pool.take(6)
    assert sorted(a + b) == list(range(10)) and pool.used == 10
    with pytest.raises(MemoryError):
        pool.take(1)
    pool.give(a)
    assert pool.used == 6 and sorted(pool.take(4)) == sorted(a)


def test_admission_reserves_whole_length_and_retires():
    b = FakeBatch(4)
    cb = S.ContinuousBatcher(b, page_size=16, pool_pages=64, page_seed=3)
    seqs = [S.Sequence(sid=i, context=30 + i, target=2 + i, seed=7 + i) for i in range(4)]
    for q in seqs:
        cb.submit(q)
    cb.fill()
    assert cb.active() == 4
    # pages for context + target positions, rounded up to whole pages
    assert cb.pool.used == sum((q.context + q.target + 15) // 16 for q in seqs)
    fills = [c for c in b.calls if c[0] == "fill"]
    assert [(c[1], c[2]) for c in fills] == [(i, 30 + i) for i in range(4)]
    cb.step()
    cb.step()  # sequence 0 (target 2) is done
    assert cb.finished == 1 and cb.slots[0] is None
    steps = [c for c in b.calls if c[0] == "step"]
    assert steps[0] == ("step", None, [30, 31, 32, 33])
    assert steps[1] == ("step", None, [31, 32, 33, 34])
    cb.step()  # slot 0 is a gap: the others move down, their tokens read back
    last = [c for c in b.calls if c[0] == "step"][-1]
    assert last == ("step", [101, 102, 103], [33, 34, 35])
    assert b.pages[0] == seqs[1].pages and b.pages[2] == seqs[3].pages


def test_config4_workload_is_steady_and_seeded():
    rng = np.random.default_rng(3)
    init = S.config4_workload(rng)
    assert len(init) == 64
    assert all(128 <= q.context <= 4096 for q in init)
    assert sorted(q.generated for q in init) == [i * 2 for i in range(64)]
    arrivals, nxt = S.config4_arrivals(np.random.default_rng(9), 64)
    assert nxt == 64 + len(arrivals)
    again, _ = S.config4_arrivals(np.random.default_rng(9), 64)
    assert [(q.context, q.seed) for q in arrivals] == [(q.context, q.seed) for q in again]
    # the full batch retires about one sequence every two steps
    b = FakeBatch(64)
    cb = S.ContinuousBatcher(b, page_size=16, pool_pages=64 * 300)
    for q in init:
        cb.submit(q)
    cb.fill()
    for _ in range(40):
        cb.step()
    assert 18 <= cb.finished <= 22


def test_config5_requests_and_sharding():
    """Config 5's request set: lognormal contexts (median 2048) clipped to
    [512, 32768], seeded; the longest-processing-time split puts every
    request on exactly one shard with near-equal expected bytes."""
    from lcr_b200 import serve
    c = serve.config5_requests(512, 1.0)
    assert np.array_equal(c, serve.config5_requests(512, 1.0))
    assert c.min() >= 512 and c.max() <= 32768 and 1800 <= np.median(c) <= 2300
    for shards in (1, 2, 4, 8):
        parts = [serve.shard_requests(c, k, shards, 256) for k in range(shards)]
        assert sorted(i for p in parts for i in p) == list(range(512))
        loads = [sum(int(c[i]) + 256 for i in p) for p in parts]
        assert max(loads) - min(loads) <= int(c.max()) + 256

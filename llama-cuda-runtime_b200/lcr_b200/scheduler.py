"""Continuous batching on lcr_batch: slots, a KV page pool and the config-4
workload.

The reference decodes one sequence per Model and allocates pages for it from
a counter (src/kv_cache.cu:73-102). Here many sequences share one pool: a
free list hands pages out (in a seeded shuffled order, so physical order is
scattered as in config 3) and takes them back when a sequence finishes; a
sequence reserves its whole length (context + tokens to decode) when it is
admitted, so a step never waits for pages.
"""
from __future__ import annotations

from collections import deque
from dataclasses import dataclass, field
from typing import Optional

import numpy as np


class PagePool:
    """Free list over pages [0, n)."""

    def __init__(self, n: int, seed: int = 0):
        order = np.arange(n, dtype=np.int32)
        if seed:
            np.random.default_rng(seed).shuffle(order)
        self.free = deque(int(p) for p in order)
        self.size = n

    def take(self, k: int) -> list:
        if k > len(self.free):
            raise MemoryError(f"KV pool exhausted: {k} pages wanted, {len(self.free)} free")
        return [self.free.popleft() for _ in range(k)]

    def give(self, pages) -> None:
        self.free.extend(pages)

    @property
    def used(self) -> int:
        return self.size - len(self.free)


@dataclass
class Sequence:
    sid: int
    context: int          # cached positions when admitted (the prompt)
    target: int           # tokens to decode
    seed: int             # Philox key of its sampling
    generated: int = 0
    pages: list = field(default_factory=list)
    prompt: Optional[np.ndarray] = None  # context token ids, for a real prefill
    tokens: list = field(default_factory=list)  # sampled ids, when recorded

    @property
    def position(self) -> int:  # position decoded by the next step
        return self.context + self.generated

    @property
    def done(self) -> bool:
        return self.generated >= self.target


class ContinuousBatcher:
    """Keeps the slots of a runtime.Batch full: admits waiting sequences into
    free slots (pages reserved, sampling set, the context prefilled in chunks
    of `prefill_chunk` tokens through lcr_batch_prefill when the sequence has
    a prompt, else written by lcr_batch_fill_kv as a synthetic stand-in),
    steps every slot with device token feedback, and retires sequences that
    reached their target. With `record`, every sampled id is read back and
    kept on its sequence (one host round trip per step)."""

    def __init__(self, batch, *, page_size: int, pool_pages: int, page_seed: int = 0,
                 temperature: float = 0.8, top_k: int = 50, top_p: float = 0.9,
                 prefill_chunk: int = 2048, record: bool = False):
        self.batch = batch
        self.page_size = page_size
        self.pool = PagePool(pool_pages, page_seed)
        self.slots: list = [None] * batch.max_batch
        self.waiting: deque = deque()
        self.sampling = (temperature, top_k, top_p)
        self.finished = 0
        self.admitted = 0
        self.prefill_chunk = prefill_chunk
        self.record = record

    def submit(self, seq: Sequence) -> None:
        self.waiting.append(seq)

    def _admit(self, slot: int, seq: Sequence) -> None:
        need = (seq.context + seq.target + self.page_size - 1) // self.page_size
        seq.pages = self.pool.take(need)
        self.batch.set_pages(slot, seq.pages)
        t, k, p = self.sampling
        self.batch.set_sampling(slot, t, k, p, seq.seed)
        if seq.prompt is not None:
            # The prompt through the prefill path; its last row's sample is the
            # slot's next token, which the first step feeds back.
            assert len(seq.prompt) == seq.context and seq.generated == 0
            for at in range(0, seq.context, self.prefill_chunk):
                self.batch.prefill(slot, seq.prompt[at:at + self.prefill_chunk], at)
            if self.record:
                seq.tokens.append(int(self.batch.read(slot + 1)[slot]))
        else:
            # Positions below seq.position hold its context (and any tokens it
            # is assumed to have decoded already).
            self.batch.fill_kv(slot, seq.position, seq.seed)
        self.slots[slot] = seq
        self.admitted += 1

    def fill(self) -> None:
        for slot, seq in enumerate(self.slots):
            if seq is None and self.waiting:
                self._admit(slot, self.waiting.popleft())

    def active(self) -> int:
        """Leading slots in use (lcr_batch_step decodes slots [0, n))."""
        n = 0
        while n < len(self.slots) and self.slots[n] is not None:
            n += 1
        return n

    def _compact(self):
        """Moves the last occupied slots into gaps so the occupied slots form a
        prefix. A moved sequence's next token is its previous sample, read
        back from its old slot; returns explicit tokens for this step (or None
        when nothing moved)."""
        occupied = [b for b, q in enumerate(self.slots) if q is not None]
        if not occupied or occupied[-1] == len(occupied) - 1:
            return None
        prev = self.batch.read(occupied[-1] + 1)
        tokens = [int(prev[b]) for b in range(len(self.slots)) if b < len(prev)]
        out = []
        for dst in range(len(occupied)):
            src = occupied[dst]
            if src != dst:
                seq = self.slots[src]
                self.slots[dst], self.slots[src] = seq, None
                self.batch.set_pages(dst, seq.pages)
                t, k, p = self.sampling
                self.batch.set_sampling(dst, t, k, p, seq.seed)
            out.append(tokens[src])
        return out

    def step(self) -> int:
        """One decode step of the occupied slots; returns tokens decoded."""
        tokens = self._compact()
        n = self.active()
        if n == 0:
            return 0
        self.batch.step(tokens, [self.slots[b].position for b in range(n)])
        ids = self.batch.read(n) if self.record else None
        for b in range(n):
            seq = self.slots[b]
            seq.generated += 1
            if ids is not None:
                seq.tokens.append(int(ids[b]))
            if seq.done:
                self.pool.give(seq.pages)
                self.slots[b] = None
                self.finished += 1
        return n


def config4_workload(rng: np.random.Generator, batch: int = 64, target: int = 128,
                     lo: int = 128, hi: int = 4096):
    """The initial sequences of config 4: contexts uniform in [lo, hi],
    `target` tokens each; sequence i starts as if it had decoded
    i * target // batch tokens already, so completions are spread over the
    steps from the start (steady state), not bunched at step `target`."""
    seqs = []
    for i in range(batch):
        s = Sequence(sid=i, context=int(rng.integers(lo, hi + 1)), target=target,
                     seed=int(rng.integers(1, 2**63)))
        s.generated = i * target // batch
        seqs.append(s)
    return seqs


def config4_arrivals(rng: np.random.Generator, next_sid: int, mean: float = 4.0,
                     target: int = 128, lo: int = 128, hi: int = 4096):
    """One step's Poisson(mean) arrivals, contexts uniform in [lo, hi]."""
    out = []
    for _ in range(int(rng.poisson(mean))):
        out.append(Sequence(sid=next_sid, context=int(rng.integers(lo, hi + 1)), target=target,
                            seed=int(rng.integers(1, 2**63))))
        next_sid += 1
    return out, next_sid

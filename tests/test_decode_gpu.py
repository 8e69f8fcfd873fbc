"""The whole decode step through the C ABI against the fp32 host oracle on the
same random-init checkpoints (greedy ids identical,
per-step logits max-abs <= 3e-2 and cosine >= 0.999), plus the step's
variants that must agree with each other bit for bit."""
import ctypes
import os

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


def cos(a, b):
    a, b = np.asarray(a, np.float64), np.asarray(b, np.float64)
    return float(a @ b / np.linalg.norm(a) / np.linalg.norm(b))


@pytest.fixture(scope="module")
def tiny():
    block = ck.cached(ck.TINY, 0)
    return block, rt.upload_block(block)


# With fp32 activations (FLAG_FP32_ACT) the only rounding left is the bf16 KV
# cache, so the step tracks the oracle's fp32-with-bf16-cache mode closely.
TINY_F32_ABS = 3e-3


@pytest.mark.parametrize("flags", [rt.FLAG_PER_TOKEN_PREFILL, 0, rt.FLAG_FP32_ACT])
def test_tiny_prefill_and_greedy_vs_oracle(tiny, flags):
    """Prompt + 16 greedy steps on the tiny model, every step within the
    north-star gates of the fp32 oracle; the reference rounding also within
    1e-2 of the bf16-storage oracle (the prompt as decode steps, or as one
    chunk like the default tcgen05 prefill), fp32 activations within 3e-3 of
    the oracle's fp32 evaluation over a bf16 KV cache."""
    block, wdev = tiny
    prompt = ck.prompt_ids(0, 32)
    m = rt.Model(block, wdev, max_seq=64, flags=flags)
    # The chunk's bf16 probabilities are rounded per 16-key tile before
    # normalisation, the reference's after (tests/test_prefill_chunked_gpu.py).
    own_mode, own_tol = {rt.FLAG_FP32_ACT: (oracle.MODE_FP32_KV_BF16, TINY_F32_ABS),
                         rt.FLAG_PER_TOKEN_PREFILL: (oracle.MODE_BF16, 1e-2),
                         0: (oracle.MODE_BF16, 2e-2)}[flags]
    ref32 = oracle.Model(block, 64)
    own = oracle.Model(block, 64)
    m.prefill(prompt)
    for pos, tok in enumerate(prompt):
        l32 = ref32.decode(int(tok), pos, oracle.MODE_FP32)
    if flags == 0:
        lown = own.prefill(prompt, 0, own_mode)
    else:
        for pos, tok in enumerate(prompt):
            lown = own.decode(int(tok), pos, own_mode)
    got = m.logits_to_host()
    pos = len(prompt)
    for step in range(17):
        assert np.abs(got - l32).max() <= MAX_ABS and cos(got, l32) >= MIN_COS, step
        assert np.abs(got - lown).max() <= own_tol, step
        if step == 16:
            break
        tok = int(np.argmax(got))
        assert tok == oracle.argmax(lown), f"step {step}: greedy id differs from the oracle"
        m.decode(tok)
        got = m.logits_to_host()
        l32 = ref32.decode(tok, pos, oracle.MODE_FP32)
        lown = own.decode(tok, pos, own_mode)
        pos += 1


def test_device_greedy_loop_matches_host_loop(tiny):
    block, wdev = tiny
    prompt = ck.prompt_ids(0, 20)
    a = rt.Model(block, wdev, max_seq=128)
    a.prefill(prompt[:-1])
    dev_tokens = a.generate_greedy(int(prompt[-1]), 40)
    b = rt.Model(block, wdev, max_seq=128)
    b.prefill(prompt)
    host_tokens = []
    for _ in range(40):
        t = int(np.argmax(b.logits_to_host()))
        host_tokens.append(t)
        b.decode(t)
    assert dev_tokens.tolist() == host_tokens
    assert a.position == 19 + 40 and b.position == 20 + 40


@pytest.mark.parametrize("variant", [dict(paged=True, page_order_seed=7),
                                     dict(paged=True, page_size=32),
                                     dict(flags=rt.FLAG_NO_GRAPH),
                                     dict(flags=rt.FLAG_NO_PERSISTENT),
                                     dict(flags=rt.FLAG_NO_PERSISTENT | rt.FLAG_NO_PDL),
                                     dict(flags=rt.FLAG_NO_PERSISTENT | rt.FLAG_NO_GRAPH,
                                          paged=True, page_order_seed=3),
                                     dict(attention_splits=3), dict(gemv_ctas=37,
                                                                    flags=rt.FLAG_NO_PERSISTENT),
                                     dict(flags=rt.FLAG_FP32_ACT, paged=True, page_order_seed=5),
                                     dict(tensor_pipe=True), dict(tensor_pipe=True, paged=True, page_order_seed=9),
                                     dict(tensor_pipe=True, flags=rt.FLAG_FP32_ACT, paged=True, page_order_seed=5)])
def test_step_variants_are_bit_identical(tiny, variant):
    """Layout and scheduling options of the step change no result bit; a
    different split or CTA count, or the multi-kernel step, changes only the
    fp32 summation order; fp32 activations stay within the north-star gate of
    the reference rounding. These compare the persistent step with its
    CUDA-core attention phase, which shares its device functions with the
    multi-kernel step. The tensor-pipe attention phase (the default) sums in
    another order and carries the softmax weights as a bf16 pair, so its
    attention outputs may round to the neighbouring bf16 value; on this model
    one such flip moves the logits by about 6e-3, so it is held to 1e-2, the
    tolerance against the bf16-storage oracle, and to the same greedy ids."""
    block, wdev = tiny
    prompt = ck.prompt_ids(3, 40)
    variant = dict(variant)
    tensor_pipe = variant.pop("tensor_pipe", False)
    multi = variant.get("flags", 0) & rt.FLAG_NO_PERSISTENT
    # The prompt as decode steps, so that it runs through the variant too.
    cc = rt.FLAG_CUDA_CORE_ATTENTION
    variant["flags"] = variant.get("flags", 0) | rt.FLAG_PER_TOKEN_PREFILL | (0 if tensor_pipe else cc)
    base = rt.Model(block, wdev, max_seq=96, flags=rt.FLAG_PER_TOKEN_PREFILL | cc)
    other = rt.Model(block, wdev, max_seq=96, **variant)
    base.prefill(prompt)
    other.prefill(prompt)
    a, b = base.logits_to_host(), other.logits_to_host()
    order_changes = ("attention_splits" in variant or "gemv_ctas" in variant or multi)
    if variant["flags"] & rt.FLAG_FP32_ACT:
        # fp32 activations against the reference rounding: the bf16 storage
        # of the intermediate tensors, not only the order
        assert np.abs(a - b).max() < 3e-2
    elif tensor_pipe:
        assert np.abs(a - b).max() < 1e-2
    elif order_changes:
        # a different split / CTA count, or the multi-kernel step's attention
        # partition, changes the fp32 summation order only
        assert np.abs(a - b).max() < 1e-3
    else:
        assert np.array_equal(a, b)
    ta = base.generate_greedy(int(np.argmax(a)), 8)
    tb = other.generate_greedy(int(np.argmax(b)), 8)
    assert ta.tolist() == tb.tolist()


@pytest.mark.parametrize("paged", [False, True])
@pytest.mark.parametrize("length,splits", [(40, 0), (700, 0), (700, 6), (700, 11)])
def test_exchange_matches_grid_barriers(tiny, paged, length, splits):
    """The persistent step's tagged-word exchange between phases (default)
    and its grid barriers compute the same bits: the prompt as decode steps,
    then greedy steps -- one split per KV head at 40 positions, the default
    two at 700 (merged by split 0 with the O prologue's arithmetic), and six
    and eleven at 700 (merged by four split CTAs per KV head)."""
    block, wdev = tiny
    prompt = ck.prompt_ids(5, length)
    kw = dict(max_seq=length + 24, paged=paged, page_size=16, page_order_seed=13, attention_splits=splits)
    a = rt.Model(block, wdev, flags=rt.FLAG_PER_TOKEN_PREFILL, **kw)
    b = rt.Model(block, wdev, flags=rt.FLAG_PER_TOKEN_PREFILL | rt.FLAG_GRID_BARRIERS, **kw)
    a.prefill(prompt)
    b.prefill(prompt)
    la, lb = a.logits_to_host(), b.logits_to_host()
    assert np.array_equal(la, lb)
    first = int(np.argmax(la))
    assert a.generate_greedy(first, 12).tolist() == b.generate_greedy(first, 12).tolist()
    assert np.array_equal(a.logits_to_host(), b.logits_to_host())


@pytest.mark.parametrize("paged", [False, True])
@pytest.mark.parametrize("splits", [0, 11])
def test_tiny_long_context_vs_oracle(tiny, paged, splits):
    """700 cached positions: several 128-position KV stages per attention
    split and many splits per KV head, shuffled physical pages when paged --
    the persistent step's long-context path (config 3's shape on the tiny
    model) against the oracle, after the prompt's chunked prefill (against
    the oracle's chunk of the same rounding points)."""
    block, wdev = tiny
    prompt = ck.prompt_ids(3, 700)
    m = rt.Model(block, wdev, max_seq=760, paged=paged, page_size=16, page_order_seed=99,
                 attention_splits=splits)
    ref32 = oracle.Model(block, 760)
    ref16 = oracle.Model(block, 760)
    m.prefill(prompt)
    l32 = ref32.prefill(prompt, 0, oracle.MODE_FP32)
    l16 = ref16.prefill(prompt, 0, oracle.MODE_BF16)
    got = m.logits_to_host()
    pos = len(prompt)
    for step in range(6):
        assert np.abs(got - l32).max() <= MAX_ABS and cos(got, l32) >= MIN_COS, step
        # 2e-2: the chunk's per-tile bf16 probabilities against the
        # reference's normalised ones (tests/test_prefill_chunked_gpu.py)
        assert np.abs(got - l16).max() <= 2e-2, step
        tok = int(np.argmax(got))
        assert tok == oracle.argmax(l16), f"step {step}: greedy id differs from the bf16 oracle"
        m.decode(tok)
        got = m.logits_to_host()
        l32 = ref32.decode(tok, pos, oracle.MODE_FP32)
        l16 = ref16.decode(tok, pos, oracle.MODE_BF16)
        pos += 1


def test_paged_block_tables_match_oracle_allocator(tiny):
    block, wdev = tiny
    g = block.geom
    seed = 12345
    m = rt.Model(block, wdev, max_seq=200, paged=True, page_size=16, page_order_seed=seed)
    m.prefill(ck.prompt_ids(5, 10))
    m.generate_greedy(1, 23)  # length 34 -> 3 pages per layer
    tables, mapped = m.page_tables()
    max_pages = (200 + 15) // 16
    pool = max_pages * g.num_layers
    want = np.full((g.num_layers, max_pages), -1, np.int32)
    order = oracle.page_permutation(pool, seed)
    n = oracle.paged_reserve(want, 16, 0, 10, 0, pool, order)
    n = oracle.paged_reserve(want, 16, 10, 33, n, pool, order)
    n = oracle.paged_reserve(want, 16, 33, 34, n, pool, order)
    assert mapped == n
    assert np.array_equal(tables, want)


@pytest.mark.parametrize("sync", [0, rt.FLAG_GRID_BARRIERS], ids=["exchange", "grid-barriers"])
def test_timeout_path_reports_and_recovers(tiny, sync):
    """A wait that never ends, made on purpose without faulting anything: the
    test switch bounds every wait at 50 ms and has CTA 0 skip its first
    arrival at a grid barrier, or, with the tagged-word exchange, keep its
    first q/k/v rows out of the exchange. The waiting CTAs give up, raise the
    abort bit, the producers stop at it and drain the copies they issued, and
    every step of the prompt ends quickly; the host reads LCR_ERR_TIMEOUT.
    The context is then destroyed, and fresh contexts on the same device and
    weights compute the normal result."""
    import time

    block, wdev = tiny
    prompt = ck.prompt_ids(0, 8)
    # The prompt as decode steps: each one a persistent step that times out.
    per_token = rt.FLAG_PER_TOKEN_PREFILL | sync
    m = rt.Model(block, wdev, max_seq=32, flags=rt.FLAG_TEST_TIMEOUT | per_token)
    t0 = time.perf_counter()
    with pytest.raises(rt.LcrError) as e:
        m.prefill(prompt)
    assert e.value.status == 4, e.value  # LCR_ERR_TIMEOUT
    assert time.perf_counter() - t0 < 10.0
    m.close()
    a = rt.Model(block, wdev, max_seq=32, flags=per_token)
    a.prefill(prompt)
    got = a.logits_to_host()
    ref = oracle.Model(block, 32)
    for pos, tok in enumerate(prompt):
        want = ref.decode(int(tok), pos, oracle.MODE_BF16)
    assert np.abs(got - want).max() <= 1e-2
    b = rt.Model(block, wdev, max_seq=32, flags=per_token)
    b.prefill(prompt)
    assert np.array_equal(b.logits_to_host(), got)


def test_bad_inputs_are_rejected(tiny):
    block, wdev = tiny
    m = rt.Model(block, wdev, max_seq=8)
    with pytest.raises(rt.LcrError) as e:
        m.decode(-1)
    assert e.value.status == 1
    m.prefill([1, 2, 3, 4, 5, 6, 7, 8])
    with pytest.raises(rt.LcrError) as e:
        m.decode(3)
    assert e.value.status == 6  # the cache is full
    with pytest.raises(rt.LcrError):
        rt.Model(block, wdev, max_seq=8, paged=True, page_size=8)


def rel_rms(got, want):
    """tools/validate_main.cu:103-105 of the reference: error RMS over signal RMS."""
    got, want = np.asarray(got, np.float64), np.asarray(want, np.float64)
    return float(np.sqrt(np.mean((got - want) ** 2)) / np.sqrt(np.mean(want ** 2)))


# Cosine gate of the reference's validator (tools/validate_main.cu:149-153).
# Its rel-RMS <= 0.02 is not usable on these logits: the bf16-storage
# algorithm itself already sits near 0.02 from fp32 on the random-init 1B
# model, so the distance gates below are relative to that algorithm's own.
SLACK = 1.5
# Top-2 gap under which two correct bf16 evaluations may pick different ids:
# two summation orders of the oracle already differ by 0.07-0.10 in max-abs on
# this model (tests/test_oracle.py::test_bf16_reproducibility_floor_1b).
NEAR_TIE = 0.06


def test_1b_config2_teacher_forced_vs_oracle():
    """Config 2: Llama-3.2-1B geometry, seed 1, 128-id prompt, 256 greedy
    tokens generated on the device, every step re-evaluated on the GPU's
    tokens by the fp32 oracle (cosine >= 0.999; rel-RMS and max-abs within
    1.5x of the bf16-storage algorithm's own distance from fp32) and by the
    bf16-storage oracle (greedy ids identical wherever the top-2 gap is above
    the algorithm's reproducibility floor)."""
    g = ck.LLAMA_3_2_1B
    block = ck.cached(g, 1)
    prompt = ck.prompt_ids(1, 128)
    steps = int(os.environ.get("LCR_TEST_1B_STEPS", "256"))
    m = rt.Model(block, max_seq=512)
    m.prefill(prompt[:-1])
    gen = m.generate_greedy(int(prompt[-1]), steps)
    r16 = oracle.Model(block, 512)
    r32 = oracle.Model(block, 512)
    for pos, tok in enumerate(prompt[:-1]):
        r16.decode(int(tok), pos, oracle.MODE_BF16)
        r32.decode(int(tok), pos, oracle.MODE_FP32)
    m2 = rt.Model(block, m.weights_dev, max_seq=512)
    m2.prefill(prompt[:-1])
    tok, pos = int(prompt[-1]), len(prompt) - 1
    worst = dict(abs16=0.0, abs32=0.0, rms32=0.0, cos32=1.0, ref_abs32=0.0, ref_rms32=0.0)
    near_ties, mismatches = 0, []
    for s in range(steps):
        m2.decode(tok)
        got = m2.logits_to_host()
        w16 = r16.decode(tok, pos, oracle.MODE_BF16)
        w32 = r32.decode(tok, pos, oracle.MODE_FP32)
        worst["abs16"] = max(worst["abs16"], float(np.abs(got - w16).max()))
        worst["abs32"] = max(worst["abs32"], float(np.abs(got - w32).max()))
        worst["rms32"] = max(worst["rms32"], rel_rms(got, w32))
        worst["cos32"] = min(worst["cos32"], cos(got, w32))
        worst["ref_abs32"] = max(worst["ref_abs32"], float(np.abs(w16 - w32).max()))
        worst["ref_rms32"] = max(worst["ref_rms32"], rel_rms(w16, w32))
        if int(np.argmax(got)) != int(gen[s]):
            mismatches.append(("graph-vs-step", s))
        if int(gen[s]) != oracle.argmax(w16):
            top2 = np.sort(w16)[-2:]
            gap = float(top2[1] - top2[0])
            # A flip is a near tie when the oracle's top-2 gap is within twice
            # the GPU's measured distance from it at this very step.
            if gap < max(NEAR_TIE, 2.0 * float(np.abs(got - w16).max())):
                near_ties += 1
            else:
                mismatches.append(("oracle", s, gap))
        tok, pos = int(gen[s]), pos + 1
    print(f"1B over {steps} steps: {worst}, near ties {near_ties}")
    assert not mismatches, mismatches
    assert worst["cos32"] >= MIN_COS
    assert worst["rms32"] <= SLACK * worst["ref_rms32"]
    assert worst["abs32"] <= SLACK * worst["ref_abs32"]
    assert near_ties <= steps // 10


def test_1b_config3_paged_shuffled_matches_contiguous():
    """Config 3's shape at full size: Llama-3.2-1B (seed 1), an 8192-id prompt
    (seed 2), then greedy steps. A paged cache of 16-position pages in a
    shuffled physical order (page_order_seed 2) and a contiguous cache of the
    same length must give bit-identical logits and token ids: the page table
    only moves where a position's K/V rows live, and both contexts use the
    same split count (same max_seq), so the summation order is the same."""
    g = ck.LLAMA_3_2_1B
    block = ck.cached(g, 1)
    wdev = rt.upload_block(block, 0)
    prompt = ck.prompt_ids(2, 8192)
    max_seq = 8192 + 32
    paged = rt.Model(block, wdev, max_seq=max_seq, paged=True, page_size=16, page_order_seed=2)
    flat = rt.Model(block, wdev, max_seq=max_seq)
    paged.prefill(prompt)
    flat.prefill(prompt)
    a, b = paged.logits_to_host(), flat.logits_to_host()
    assert np.all(np.isfinite(a))
    assert np.array_equal(a, b)
    tables, mapped = paged.page_tables()
    assert mapped == g.num_layers * (8192 // 16)
    first = tables[0][tables[0] >= 0]
    assert len(first) == 8192 // 16 and len(set(first.tolist())) == len(first)
    assert not np.array_equal(first, np.sort(first)), "the physical page order is not shuffled"
    ta = paged.generate_greedy(int(np.argmax(a)), 16)
    tb = flat.generate_greedy(int(np.argmax(b)), 16)
    assert ta.tolist() == tb.tolist()
    assert np.array_equal(paged.logits_to_host(), flat.logits_to_host())
    paged.close()
    flat.close()


GOLDEN = os.path.join(os.path.dirname(os.path.abspath(__file__)), "golden")

# Gates against the fp32 host evaluation at 1B (tests/golden/make_golden_1b.py).
# The fp32-activation step sits on the floor of the bf16 KV cache format: the
# oracle itself, fp32 everywhere but the cache, is 0.033 from fp32 on the
# first logits of configuration 2. The reference rounding sits on the floor of
# its own algorithm (two summation orders differ by 0.07-0.10).
FIXTURE_GATES = {0: dict(full=0.15, top=0.12), rt.FLAG_FP32_ACT: dict(full=0.04, top=0.03)}


def _fixture_run(m, fx, steps, gates, label):
    """Teacher-forces the fp32 oracle's greedy ids: the first logits against
    the fixture's full vector, every step's top-32 logits against the
    fixture's, and the greedy id equal to the fixture's wherever its top-2 gap
    is more than twice the step's measured distance (a near tie otherwise)."""
    got = m.logits_to_host()
    full = float(np.abs(got - fx["logits0"]).max())
    c = cos(got, fx["logits0"])
    worst, ties, flips = 0.0, [], []
    for s in range(steps):
        ti, tv = fx["top_idx"][s], fx["top_val"][s]
        dist = float(np.abs(got[ti] - tv).max())
        worst = max(worst, dist)
        if int(np.argmax(got)) != int(fx["ids"][s]):
            (ties if float(fx["gap"][s]) < 2.0 * dist else flips).append((s, float(fx["gap"][s])))
        if s + 1 < steps:
            m.decode(int(fx["ids"][s]))
            got = m.logits_to_host()
    print(f"{label}: first logits max-abs {full:.4f} cos {c:.6f}; top-32 worst {worst:.4f} "
          f"over {steps} steps; near-tie flips {ties}")
    assert not flips, flips
    assert c >= MIN_COS
    assert full <= gates["full"] and worst <= gates["top"]
    return full, worst, ties


@pytest.mark.parametrize("flags", [0, rt.FLAG_FP32_ACT])
def test_1b_config2_vs_fp32_fixture(flags):
    """Configuration 2 against the committed fp32 oracle run
    (c2_fp32_1b.npz): 256 teacher-forced steps, then a free-running greedy
    generation whose first divergence from the oracle's ids (if any) must be
    at a near tie."""
    fx = np.load(os.path.join(GOLDEN, "c2_fp32_1b.npz"))
    block = ck.cached(ck.LLAMA_3_2_1B, 1)
    wdev = rt.upload_block(block, 0)
    m = rt.Model(block, wdev, max_seq=512, flags=flags)
    m.prefill(fx["prompt"])
    full, worst, _ = _fixture_run(m, fx, 256, FIXTURE_GATES[flags], f"config 2 flags {flags}")
    free = rt.Model(block, wdev, max_seq=512, flags=flags)
    free.prefill(fx["prompt"])
    first = int(np.argmax(free.logits_to_host()))
    ids = np.concatenate([[first], free.generate_greedy(first, 255)])
    diverge = np.flatnonzero(ids != fx["ids"])
    at = int(diverge[0]) if diverge.size else None
    print(f"config 2 flags {flags}: free-running greedy ids equal to the fp32 oracle's for "
          f"{256 if at is None else at} of 256 steps" +
          ("" if at is None else f" (first divergence at a top-2 gap of {float(fx['gap'][at]):.4f})"))
    if at is not None:
        assert float(fx["gap"][at]) < 2.0 * worst, "free-running ids left the oracle's at a clear margin"


def test_1b_config3_vs_fp32_fixture():
    """Configuration 3 (8192-id prompt, paged cache in shuffled physical
    order) against the committed fp32 oracle run (c3_fp32_1b.npz): the logits
    after the prompt and 16 teacher-forced greedy steps."""
    fx = np.load(os.path.join(GOLDEN, "c3_fp32_1b.npz"))
    block = ck.cached(ck.LLAMA_3_2_1B, 1)
    m = rt.Model(block, max_seq=8192 + 32, paged=True, page_size=16, page_order_seed=2)
    m.prefill(fx["prompt"])
    _fixture_run(m, fx, 16, FIXTURE_GATES[0], "config 3")

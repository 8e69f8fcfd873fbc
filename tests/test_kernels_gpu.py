"""Every per-kernel C entry point against the CPU oracle on the same seeded
inputs -- the structure of the reference's tests/test_kernels.cu (nested-loop
references, bf16-rounded inputs, tolerance 3e-2 of max |expected|) plus B200
split counts, shuffled pages and bit-exact sampling."""
import ctypes

import numpy as np
import pytest

import oracle
from lcr_b200 import checkpoint as ck
from lcr_b200 import runtime as rt

pytestmark = pytest.mark.gpu

TOL = 3e-2  # relative to max |expected| (tests/test_kernels.cu:35)

torch = pytest.importorskip("torch")
if not torch.cuda.is_available():
    pytest.skip("needs a CUDA device", allow_module_level=True)

L = rt.lib()
RNG = np.random.default_rng(20260904)


def bf(x):
    return ck.float_to_bf16_bits(np.asarray(x, np.float32))


def fl(b):
    return ck.bf16_bits_to_float(b)


def dev(a):
    a = np.ascontiguousarray(a)
    if a.dtype == np.uint16:
        a = a.view(np.int16)
    return torch.from_numpy(a).cuda()


_KEEP = []


def dptr(a):
    """Device copy of `a` kept alive for the test session (kernels run
    asynchronously, so an inline temporary could be freed and its memory
    handed to the next upload before the kernel reads it)."""
    t = dev(a)
    _KEEP.append(t)
    return t.data_ptr()


def host_bf(t):
    return t.cpu().numpy().view(np.uint16)


def S():
    return rt.stream_ptr()


def expect_close(got, want, tol=TOL, what=""):
    got, want = np.asarray(got, np.float64), np.asarray(want, np.float64)
    scale = max(np.abs(want).max(), 1e-6)
    err = np.abs(got - want).max() / scale
    i = int(np.argmax(np.abs(got - want)))
    assert err <= tol, (f"{what}: worst relative error {err:.3g} > {tol} at {i} "
                        f"(got {got.flat[i]:.6g}, want {want.flat[i]:.6g}, scale {scale:.4g})")


def run(status):
    rt.check(status)
    torch.cuda.synchronize()


def test_rmsnorm():
    x = bf(RNG.normal(size=(5, 2048)))
    w = bf(RNG.normal(0, 0.5, 2048))
    out = torch.empty(5 * 2048, dtype=torch.int16, device="cuda")
    run(L.lcr_rmsnorm(out.data_ptr(), dptr(x), dptr(w), 5, 2048, 1e-5, S()))
    want = oracle.rmsnorm(x, w, 1e-5, round_out=True)
    expect_close(fl(host_bf(out)).reshape(5, 2048), want, 1e-2, "rmsnorm")


def test_add_residual_rmsnorm_and_residual():
    x = bf(RNG.normal(size=(3, 2048)))
    d = bf(RNG.normal(size=(3, 2048)))
    w = bf(RNG.normal(0, 0.5, 2048))
    xd, out = dev(x), torch.empty(3 * 2048, dtype=torch.int16, device="cuda")
    run(L.lcr_add_residual_rmsnorm(out.data_ptr(), xd.data_ptr(), dptr(d),
                                   dptr(w), 3, 2048, 1e-5, S()))
    want_out, want_x = oracle.add_residual_rmsnorm(x, d, w, 1e-5)
    assert np.array_equal(host_bf(xd).reshape(3, 2048), want_x)  # stored sum is exact
    expect_close(fl(host_bf(out)).reshape(3, 2048), want_out, 1e-2, "add_residual_rmsnorm")
    count = 8192 * 3 + 5  # not a multiple of eight (tests/test_kernels.cu:156)
    a, b = bf(RNG.normal(size=count)), bf(RNG.normal(size=count))
    ad = dev(a)
    run(L.lcr_add_residual(ad.data_ptr(), dptr(b), count, S()))
    assert np.array_equal(host_bf(ad), bf(fl(a) + fl(b)))


def test_swiglu_plain_and_strided():
    count = 8192 * 3 + 5
    g, u = bf(RNG.normal(size=count)), bf(RNG.normal(size=count))
    out = torch.empty(count, dtype=torch.int16, device="cuda")
    run(L.lcr_swiglu(out.data_ptr(), dptr(g), dptr(u), count, S()))
    expect_close(fl(host_bf(out)), oracle.swiglu(g, u), TOL, "swiglu")
    tokens, width = 3, 1000
    gu = bf(RNG.normal(size=(tokens, 2 * width)))
    gud = dev(gu)
    out2 = torch.empty(tokens * width, dtype=torch.int16, device="cuda")
    run(L.lcr_swiglu_strided(out2.data_ptr(), gud.data_ptr(), gud.data_ptr() + width * 2, tokens,
                             width, 2 * width, S()))
    want = np.stack([oracle.swiglu(gu[t, :width], gu[t, width:]) for t in range(tokens)])
    expect_close(fl(host_bf(out2)).reshape(tokens, width), want, TOL, "swiglu_strided")


def test_embedding_lookup_exact():
    table = bf(RNG.normal(size=(128, 2048)))
    ids = np.array([7, 0, 127, 63], np.int32)
    out = torch.empty(4 * 2048, dtype=torch.int16, device="cuda")
    run(L.lcr_embedding_lookup(out.data_ptr(), dptr(table), dptr(ids), 4, 2048,
                               S()))
    assert np.array_equal(host_bf(out).reshape(4, 2048), table[ids])


def test_rope_q():
    tokens, heads, d, start = 3, 4, 64, 11
    q = bf(RNG.normal(size=(tokens, heads * d)))
    inv = (500000.0 ** (-2.0 * np.arange(32) / 64)).astype(np.float32)
    out = torch.empty(tokens * heads * d, dtype=torch.int16, device="cuda")
    run(L.lcr_rope_q(out.data_ptr(), dptr(q), dptr(inv), tokens, start, heads, d,
                     heads * d, S()))
    want = oracle.rope_rows(q, inv, start, heads, d, heads * d, head_major=True)
    expect_close(fl(host_bf(out)), want, TOL, "rope_q")


@pytest.mark.parametrize("rows,k,n,fp32", [(1, 2048, 3072, 0), (1, 8192, 2048, 0),
                                           (3, 2048, 1000, 1), (2, 256, 700, 0),
                                           (1, 1024, 256, 1), (2, 768, 333, 0),
                                           # batched: the tcgen05 path (>= 16 rows)
                                           (16, 2048, 3072, 1), (64, 2048, 2048, 0),
                                           (100, 1024, 700, 1), (200, 512, 384, 0),
                                           (32, 8192, 256, 1), (17, 64, 130, 1),
                                           # persistent 128-row tiles: CTAs walk
                                           # several tiles (one K slab each in
                                           # the second case)
                                           (300, 256, 8192, 0), (257, 64, 20000, 1)])
def test_gemm_nt(rows, k, n, fp32):
    x = bf(RNG.normal(size=(rows, k)))
    w = bf(RNG.normal(0, 0.02, size=(n, k)))
    y = torch.empty(rows * n, dtype=torch.float32 if fp32 else torch.int16, device="cuda")
    run(L.lcr_gemm_nt(y.data_ptr(), fp32, dptr(x), dptr(w), rows, k, n, S()))
    got = y.cpu().numpy() if fp32 else fl(host_bf(y))
    want = np.concatenate([oracle.gemv(w, x[r]) for r in range(rows)])
    # fp32 outputs: both sides accumulate in fp32, in different orders (the
    # oracle left to right, the kernels in lane / tensor-core trees), so the
    # rounding difference grows like sqrt(k).
    expect_close(got, want, 1e-5 * max(1.0, np.sqrt(k / 2048)) if fp32 else 1e-2, "gemm_nt")


# --- decode attention: the reference's 11 cases (tests/test_kernels.cu:417-440)
# plus B200 split counts, long contexts and shuffled physical pages ---------

def _attention_case(heads, kv_heads, d, positions, splits, paged, shuffled=False, seed=0):
    rng = np.random.default_rng(seed + positions * 7 + splits)
    kvd = kv_heads * d
    keys = bf(rng.normal(size=(positions, kvd)))
    values = bf(rng.normal(size=(positions, kvd)))
    q = bf(rng.normal(size=heads * d))
    max_seq = positions + 8
    page = 16
    if paged:
        max_pages = (max_seq + page - 1) // page
        pool = max_pages + 3
        order = oracle.page_permutation(pool, 99) if shuffled else np.arange(pool, dtype=np.int32)
        table = order[:max_pages].astype(np.int32)
        kp = torch.zeros(pool * kv_heads * page * d, dtype=torch.int16, device="cuda")
        vp = torch.zeros_like(kp)
        td = dev(table)
        view = rt.KvView(kp.data_ptr(), vp.data_ptr(), td.data_ptr(), page, kv_heads * page * d,
                         page * d, kv_heads, d)
    else:
        kp = torch.zeros(kv_heads * max_seq * d, dtype=torch.int16, device="cuda")
        vp = torch.zeros_like(kp)
        view = rt.KvView(kp.data_ptr(), vp.data_ptr(), None, max_seq, 0, max_seq * d, kv_heads, d)
    zeros = dev(np.zeros(d // 2, np.float32))
    kd, vd = dev(keys), dev(values)
    # Fill the cache through the real write path with a zero rotation
    # (tests/test_kernels.cu:325-339).
    run(L.lcr_rope_write_kv(ctypes.byref(view), kd.data_ptr(), vd.data_ptr(), zeros.data_ptr(),
                            positions, 0, int(paged), kvd, S()))
    out = torch.empty(heads * d, dtype=torch.int16, device="cuda")
    nscr = max(2, L.lcr_decode_attention_scratch_floats(heads, d, splits))
    scr = torch.empty(nscr, dtype=torch.float32, device="cuda")
    scale = float(np.float32(1.0) / np.sqrt(np.float32(d)))
    run(L.lcr_decode_attention(out.data_ptr(), dptr(q), ctypes.byref(view), heads,
                               heads // kv_heads, positions, scale, int(paged), splits,
                               scr.data_ptr(), S()))
    want = oracle.attention(q, keys, values, heads, kv_heads, d, positions)
    expect_close(fl(host_bf(out)), want, TOL, f"attention {heads}/{kv_heads} d{d} p{positions} s{splits}")


@pytest.mark.parametrize("heads,kv,d,pos,splits,paged", [
    (32, 8, 64, 200, 1, False), (32, 8, 64, 200, 8, False), (32, 8, 64, 197, 7, False),
    (32, 8, 64, 5, 64, False), (8, 8, 64, 130, 4, False), (8, 1, 64, 130, 4, False),
    (8, 2, 128, 100, 2, False), (32, 8, 64, 1, 1, False),
    (32, 8, 64, 200, 1, True), (32, 8, 64, 200, 8, True), (32, 8, 64, 201, 4, True)])
def test_decode_attention_reference_cases(heads, kv, d, pos, splits, paged):
    _attention_case(heads, kv, d, pos, splits, paged)


@pytest.mark.parametrize("pos,splits,paged,shuffled", [
    (4096, 18, False, False), (8448, 18, True, True), (3000, 37, True, True), (1000, 1, True, True),
    (17, 18, False, False)])
def test_decode_attention_b200_cases(pos, splits, paged, shuffled):
    _attention_case(32, 8, 64, pos, splits, paged, shuffled)


# --- sampling ---------------------------------------------------------------

def _sample(logits_dev, vocab, temperature, top_k, top_p, u):
    out = torch.empty(1, dtype=torch.int32, device="cuda")
    scr = torch.empty(int(L.lcr_sample_scratch_floats(vocab, top_k)), dtype=torch.float32,
                      device="cuda")
    run(L.lcr_sample(out.data_ptr(), logits_dev.data_ptr(), vocab, temperature, top_k, top_p, u,
                     scr.data_ptr(), S()))
    return int(out.item())


def test_sampling_known_answers():
    """tests/test_kernels.cu:468-508."""
    vocab = 4096
    lg = np.full(vocab, -20.0, np.float32)
    lg[1234], lg[99], lg[7] = 5.0, 4.0, 3.0
    d = dev(lg)
    assert _sample(d, vocab, 0.0, 0, 1.0, 0.0) == 1234
    assert _sample(d, vocab, 0.0, 0, 1.0, 0.999) == 1234
    assert _sample(d, vocab, 1.0, 1, 1.0, 0.5) == 1234
    for u in (0.01, 0.5, 0.99):
        assert _sample(d, vocab, 1.0, 0, 0.9, u) in (1234, 99)
    pair = np.full(vocab, -60.0, np.float32)
    pair[3] = pair[9] = 1.0
    d2 = dev(pair)
    assert _sample(d2, vocab, 1.0, 0, 1.0, 0.25) == 3
    assert _sample(d2, vocab, 1.0, 0, 1.0, 0.75) == 9
    assert _sample(d2, vocab, 0.0, 0, 1.0, 0.5) == 3


def test_sampling_bit_exact_vs_oracle():
    rng = np.random.default_rng(11)
    vocab = 128256
    cases = 0
    for trial in range(48):
        lg = rng.normal(0, 3.0, vocab).astype(np.float32)
        if trial % 4 == 1:
            lg = np.round(lg * 2) / 2  # many exact ties at the cutoff
        if trial % 8 == 3:
            lg[:] = 1.5  # a flat row: the lowest 1024 ids are the candidates
        t = [0.0, 0.5, 0.8, 1.0, 1.3][trial % 5]
        k = [0, 1, 50, 2000, 1024, 7][trial % 6]
        p = [1.0, 0.9, 0.5, 0.999][trial % 4]
        u = float(np.float32(rng.uniform()))
        d = dev(lg)
        got = _sample(d, vocab, t, k, p, u)
        want = oracle.sample(lg, t, k, p, u)
        assert got == want, (trial, t, k, p, u, got, want)
        cases += 1
    assert cases == 48


def test_argmax_tie_goes_to_lowest_id():
    lg = np.zeros(128256, np.float32)
    lg[[77777, 5000, 128255]] = 2.0
    assert _sample(dev(lg), lg.size, 0.0, 0, 1.0, 0.5) == 5000


# --- the prefill launchers of the boundary (src/kernels.cuh:74-94) ----------

@pytest.mark.parametrize("heads,rows,keys,start", [(4, 37, 100, 63), (2, 5, 64, 0), (3, 16, 300, 100)])
def test_causal_softmax(heads, rows, keys, start):
    """Nested-loop causal softmax (the structure of tests/test_kernels.cu's
    prefill softmax case): row r sees keys up to start + r; masked entries,
    including columns past the chunk when `keys` is wider, are exactly 0."""
    scores = RNG.normal(0, 3, size=(heads, rows, keys)).astype(np.float32)
    probs = torch.empty(heads * rows * keys, dtype=torch.int16, device="cuda")
    run(L.lcr_causal_softmax(probs.data_ptr(), dptr(scores), heads, rows, keys, start, S()))
    got = fl(host_bf(probs)).reshape(heads, rows, keys)
    want = np.zeros_like(scores, dtype=np.float64)
    for h in range(heads):
        for r in range(rows):
            lim = min(keys, start + r + 1)
            e = np.exp(scores[h, r, :lim].astype(np.float64) - scores[h, r, :lim].max())
            want[h, r, :lim] = e / e.sum()
            assert not got[h, r, lim:].any()
    expect_close(got, want, TOL, "causal_softmax")
    assert np.abs(got - want).max() <= 4e-3  # bf16 rounding of values <= 1


@pytest.mark.parametrize("d", [64, 128, 20])
def test_merge_heads_exact(d):
    heads, tokens = 6, 9
    x = bf(RNG.normal(size=(heads, tokens, d)))
    out = torch.empty(tokens * heads * d, dtype=torch.int16, device="cuda")
    run(L.lcr_merge_heads(out.data_ptr(), dptr(x), tokens, heads, d, S()))
    assert np.array_equal(host_bf(out).reshape(tokens, heads * d), x.transpose(1, 0, 2).reshape(tokens, heads * d))


@pytest.mark.parametrize("paged", [False, True])
def test_gather_kv_exact(paged):
    """The cached positions as contiguous [kv_head][position][d] rows, through
    a shuffled page table (a negative entry reads as zero rows)."""
    kv_heads, d, page, positions = 2, 64, 16, 70
    max_seq = 96
    if paged:
        max_pages = max_seq // page
        pool = max_pages + 2
        table = oracle.page_permutation(pool, 5)[:max_pages].astype(np.int32)
        kp = bf(RNG.normal(size=pool * kv_heads * page * d))
        vp = bf(RNG.normal(size=pool * kv_heads * page * d))
        view = rt.KvView(dptr(kp), dptr(vp), dptr(table), page, kv_heads * page * d, page * d, kv_heads, d)

        def row(store, h, p):
            base = (int(table[p // page]) * kv_heads * page + h * page + p % page) * d
            return store[base:base + d]
    else:
        kp = bf(RNG.normal(size=kv_heads * max_seq * d))
        vp = bf(RNG.normal(size=kv_heads * max_seq * d))
        view = rt.KvView(dptr(kp), dptr(vp), None, max_seq, 0, max_seq * d, kv_heads, d)

        def row(store, h, p):
            base = (h * max_seq + p) * d
            return store[base:base + d]
    ok = torch.empty(kv_heads * positions * d, dtype=torch.int16, device="cuda")
    ov = torch.empty_like(ok)
    run(L.lcr_gather_kv(ok.data_ptr(), ov.data_ptr(), ctypes.byref(view), positions, S()))
    gk, gv = host_bf(ok).reshape(kv_heads, positions, d), host_bf(ov).reshape(kv_heads, positions, d)
    for h in range(kv_heads):
        for p in range(positions):
            assert np.array_equal(gk[h, p], row(kp, h, p)) and np.array_equal(gv[h, p], row(vp, h, p)), (h, p)

"""lcr_decode_attention_noalloc (split partials in a static device array)
against lcr_decode_attention (caller scratch) on the same cache and query.
Named to be collected last, so it runs both alone and after every other test
has used the device."""
import ctypes

import numpy as np
import pytest

import oracle
from lcr_b200 import checkpoint as ck
from lcr_b200 import runtime as rt

L = rt.lib()
LIMIT = 1 << 19  # LCR_NOALLOC_ATTENTION_SCRATCH_FLOATS
TOL = 1e-6  # relative to max |reference output|: the same kernels run


def _cuda():
    torch = pytest.importorskip("torch")
    if not torch.cuda.is_available():
        pytest.skip("needs a CUDA device")
    return torch


def _case(torch, heads, kv_heads, d, positions, splits, paged, seed):
    """Fills a cache through lcr_rope_write_kv (zero rotation) and returns
    (view, q, keepalive) for `positions` cached positions."""
    rng = np.random.default_rng(seed)
    kvd = kv_heads * d
    keys = ck.float_to_bf16_bits(rng.normal(size=(positions, kvd)).astype(np.float32))
    values = ck.float_to_bf16_bits(rng.normal(size=(positions, kvd)).astype(np.float32))
    q = ck.float_to_bf16_bits(rng.normal(size=heads * d).astype(np.float32))

    def dev(a):
        a = np.ascontiguousarray(a)
        return torch.from_numpy(a.view(np.int16) if a.dtype == np.uint16 else a).cuda()

    page = 16
    max_seq = positions + 8
    keep = []
    if paged:
        max_pages = (max_seq + page - 1) // page
        pool = max_pages + 3
        table = dev(oracle.page_permutation(pool, seed)[:max_pages].astype(np.int32))
        kp = torch.zeros(pool * kv_heads * page * d, dtype=torch.int16, device="cuda")
        vp = torch.zeros_like(kp)
        view = rt.KvView(kp.data_ptr(), vp.data_ptr(), table.data_ptr(), page,
                         kv_heads * page * d, page * d, kv_heads, d)
        keep.append(table)
    else:
        kp = torch.zeros(kv_heads * max_seq * d, dtype=torch.int16, device="cuda")
        vp = torch.zeros_like(kp)
        view = rt.KvView(kp.data_ptr(), vp.data_ptr(), None, max_seq, 0, max_seq * d, kv_heads, d)
    kd, vd, qd = dev(keys), dev(values), dev(q)
    zeros = dev(np.zeros(d // 2, np.float32))
    keep += [kp, vp, kd, vd, qd, zeros]
    rt.check(L.lcr_rope_write_kv(ctypes.byref(view), kd.data_ptr(), vd.data_ptr(),
                                 zeros.data_ptr(), positions, 0, int(paged), kvd,
                                 rt.stream_ptr()))
    return view, qd, keep


CASES = [  # heads, kv_heads, head_dim, positions, splits, paged
    (32, 8, 64, 4096, 18, False),
    (32, 8, 64, 3000, 37, True),
    (32, 8, 64, 1000, 64, True),   # 32 x 63 x 66 = 133,056 floats
    (8, 2, 128, 100, 2, False),
    (32, 8, 64, 200, 1, False),    # one split: no partials at all
]


@pytest.mark.gpu
@pytest.mark.parametrize("heads,kv,d,pos,splits,paged", CASES)
def test_noalloc_matches_scratch_entry(heads, kv, d, pos, splits, paged):
    torch = _cuda()
    view, q, keep = _case(torch, heads, kv, d, pos, splits, paged, seed=pos + splits)
    scale = float(np.float32(1.0) / np.sqrt(np.float32(d)))
    s = rt.stream_ptr()
    nscr = max(2, L.lcr_decode_attention_scratch_floats(heads, d, splits))
    scratch = torch.empty(nscr, dtype=torch.float32, device="cuda")
    want = torch.empty(heads * d, dtype=torch.int16, device="cuda")
    rt.check(L.lcr_decode_attention(want.data_ptr(), q.data_ptr(), ctypes.byref(view), heads,
                                    heads // kv, pos, scale, int(paged), splits,
                                    scratch.data_ptr(), s))
    got = [torch.full((heads * d,), -1, dtype=torch.int16, device="cuda") for _ in range(2)]
    for out in got:  # two calls in a row share the static partials
        rt.check(L.lcr_decode_attention_noalloc(out.data_ptr(), q.data_ptr(), ctypes.byref(view),
                                                heads, heads // kv, pos, scale, int(paged),
                                                splits, s))
    torch.cuda.synchronize()
    ref = ck.bf16_bits_to_float(want.cpu().numpy().view(np.uint16)).astype(np.float64)
    scale_ref = max(np.abs(ref).max(), 1e-6)
    for k, out in enumerate(got):
        val = ck.bf16_bits_to_float(out.cpu().numpy().view(np.uint16)).astype(np.float64)
        err = np.abs(val - ref).max() / scale_ref
        assert err <= TOL, f"call {k + 1}: relative error {err:.3g} against lcr_decode_attention"
    del keep


@pytest.mark.gpu
def test_noalloc_interleaved_shapes():
    """Calls of different shapes, one after another on one stream with no
    host synchronisation between them, reuse the array in turn: every result
    equals lcr_decode_attention's on caller scratch (same kernels, so bit for
    bit), whatever the previous call left in the array."""
    torch = _cuda()
    s = rt.stream_ptr()
    cases = [CASES[0], CASES[3], CASES[2], CASES[0]]
    keep, pairs = [], []
    for heads, kv, d, pos, splits, paged in cases:
        view, q, k = _case(torch, heads, kv, d, pos, splits, paged, seed=7)
        keep += [k, view, q]
        scale = float(np.float32(1.0) / np.sqrt(np.float32(d)))
        out = torch.empty(heads * d, dtype=torch.int16, device="cuda")
        want = torch.empty(heads * d, dtype=torch.int16, device="cuda")
        nscr = max(2, L.lcr_decode_attention_scratch_floats(heads, d, splits))
        scratch = torch.empty(nscr, dtype=torch.float32, device="cuda")
        keep.append(scratch)
        rt.check(L.lcr_decode_attention_noalloc(out.data_ptr(), q.data_ptr(), ctypes.byref(view),
                                                heads, heads // kv, pos, scale, int(paged),
                                                splits, s))
        rt.check(L.lcr_decode_attention(want.data_ptr(), q.data_ptr(), ctypes.byref(view), heads,
                                        heads // kv, pos, scale, int(paged), splits,
                                        scratch.data_ptr(), s))
        pairs.append((out, want))
    torch.cuda.synchronize()
    for k, (out, want) in enumerate(pairs):
        assert np.array_equal(out.cpu().numpy(), want.cpu().numpy()), f"call {k + 1}"
    del keep


def test_noalloc_rejects_oversized_partials():
    """64 heads x 64 splits x (128 + 2) floats exceed the static array; the
    check runs on the host before any CUDA call."""
    view = rt.KvView(None, None, None, 16, 0, 0, 8, 128)
    need = 64 * 64 * (128 + 2)
    assert need > LIMIT
    status = L.lcr_decode_attention_noalloc(None, None, ctypes.byref(view), 64, 8, 4096, 0.1, 0,
                                            64, None)
    assert status == 2  # LCR_ERR_SHAPE
    msg = L.lcr_last_error_string().decode()
    assert str(need) in msg and str(LIMIT) in msg

"""lcr_step_host, the one-call form of the reference's host decode loop
(Model::decode, src/model.cu:347-368, then the greedy read-back of
src/main.cu:455-463): the same tokens and logits as the asynchronous pieces
(lcr_set_token, lcr_enqueue_steps, lcr_read_token, lcr_sync), and the
status of a bad call reported."""
import ctypes

import numpy as np
import pytest

from lcr_b200 import checkpoint as ck
from lcr_b200 import runtime as rt

pytestmark = pytest.mark.gpu


@pytest.fixture(scope="module")
def tiny():
    block = ck.cached(ck.TINY, 0)
    return block, rt.upload_block(block)


@pytest.mark.parametrize("paged", [False, True])
def test_step_host_matches_pieces(tiny, paged):
    block, wdev = tiny
    prompt = ck.prompt_ids(2, 12)
    kw = dict(max_seq=64, paged=paged, page_size=16, page_order_seed=7)
    a = rt.Model(block, wdev, **kw)
    b = rt.Model(block, wdev, **kw)
    a.prefill(prompt)
    b.prefill(prompt)
    tok = int(np.argmax(a.logits_to_host()))
    assert tok == int(np.argmax(b.logits_to_host()))
    buf = (ctypes.c_int32 * 1)(tok)
    pos = len(prompt)
    for _ in range(10):
        got = a.step_host(tok, pos)
        b.set_token(ctypes.addressof(buf), pos)
        b.enqueue_steps(1)
        b.read_token(ctypes.addressof(buf))
        b.sync()
        assert got == buf[0]
        assert np.array_equal(a.logits_to_host(), b.logits_to_host())
        tok = got
        pos += 1


def test_step_host_rejects_bad_arguments(tiny):
    block, wdev = tiny
    m = rt.Model(block, wdev, max_seq=32)
    with pytest.raises(rt.LcrError):
        m.step_host(-1, 0)
    with pytest.raises(rt.LcrError):
        m.step_host(1, 32)
    m.prefill(ck.prompt_ids(2, 4))
    assert 0 <= m.step_host(1, 4) < ck.TINY.vocab_size

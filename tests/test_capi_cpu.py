"""The C-ABI library without a GPU: it loads, exports every function
include/lcr_b200.h declares, and reports errors through status codes."""
import ctypes
import os
import subprocess

import pytest

from lcr_b200 import checkpoint as ck
from lcr_b200 import runtime as rt


@pytest.fixture(scope="module")
def L():
    if not os.path.exists(rt.LIB_PATH):
        subprocess.run(["make", "-s", "-j4", "-C", rt.PKG_DIR], check=True)
    return rt.lib()


def test_every_header_symbol_is_exported(L):
    declared = rt.header_functions()
    assert len(declared) >= 40
    out = subprocess.run(["nm", "-D", "--defined-only", rt.LIB_PATH], capture_output=True,
                         text=True, check=True).stdout
    exported = {line.split()[-1] for line in out.splitlines() if " T " in line}
    missing = [f for f in declared if f not in exported]
    assert not missing, missing
    # and the Python binding declares a signature for each
    assert not [f for f in declared if f not in rt._SIGS]


def test_no_private_symbols_leak(L):
    out = subprocess.run(["nm", "-D", "--defined-only", rt.LIB_PATH], capture_output=True,
                         text=True, check=True).stdout
    exported = [line.split()[-1] for line in out.splitlines() if " T " in line]
    assert all(name.startswith("lcr_") for name in exported), exported


def test_status_strings(L):
    assert L.lcr_status_string(0) == b"ok"
    assert L.lcr_status_string(4) == b"device wait timed out"
    assert L.lcr_version() >= 100


def test_argument_errors_need_no_device(L):
    # Null pointers and bad sizes are rejected on the host, like LCR_CHECK.
    assert L.lcr_decode_attention(None, None, None, 32, 4, 0, 0.125, 0, 1, None, None) == 1
    assert b"at least one cached position" in L.lcr_last_error_string()
    assert L.lcr_sample(None, None, 0, 0.0, 0, 1.0, 0.0, None, None) == 1
    assert b"empty vocabulary" in L.lcr_last_error_string()
    assert L.lcr_rmsnorm(None, None, None, 0, 2048, 1e-5, None) == 0  # zero tokens: no-op
    assert L.lcr_decode_attention_scratch_floats(32, 64, 1) == 0
    assert L.lcr_decode_attention_scratch_floats(32, 64, 8) == 32 * 8 * 66


def test_choose_attention_splits_matches_reference_rule(L):
    # src/kernels/attention.cu:419-431: ~2 blocks per SM, >= 256 positions per
    # split, at most 64.
    assert L.lcr_choose_attention_splits(8, 200, 148) == 1
    assert L.lcr_choose_attention_splits(8, 4096, 148) == 16
    assert L.lcr_choose_attention_splits(8, 100000, 148) == 37
    assert L.lcr_choose_attention_splits(1, 100000, 148) == 64


def test_context_without_device_fails_cleanly(L):
    import torch

    if torch.cuda.is_available():
        pytest.skip("a GPU is present")
    desc = rt.desc_of(ck.TINY)
    layers = (rt.LayerWeights * 2)(*[rt.LayerWeights(16, 16, 16, 16, 16, 16) for _ in range(2)])
    w = rt.Weights(16, 16, 16, layers)
    o = rt.Options(0, 64, 0, 16, 0, 0, 0, 0)
    ctx = ctypes.c_void_p()
    st = L.lcr_ctx_create(ctypes.byref(desc), ctypes.byref(w), ctypes.byref(o), ctypes.byref(ctx))
    assert st == 7 and not ctx.value


def test_library_rope_table_bit_exact_vs_reference_code(L):
    """The inverse frequencies the library rotates with are bit-identical to
    the reference's own compute_rope_inv_freq (src/config.cpp:223-259, its
    output committed in tests/golden/ref_rope.json), scaled and unscaled."""
    import json

    import numpy as np

    golden = json.load(open(os.path.join(os.path.dirname(__file__), "golden", "ref_rope.json")))
    for name, geom in (("llama-3.2-1b", ck.LLAMA_3_2_1B),
                       ("unscaled", ck.Geometry(hidden_size=2048, intermediate_size=5632, num_layers=22,
                                                 num_heads=32, num_kv_heads=32, head_dim=64, vocab_size=32000,
                                                 rope_theta=10000.0, rope_scaling=False))):
        cfg = golden[name]["config"]
        assert cfg["rope_theta"] == geom.rope_theta and cfg["head_dim"] == geom.head_dim
        got = rt.rope_inv_freq(geom).view(np.uint32).tolist()
        assert got == golden[name]["inv_freq_bits"], name

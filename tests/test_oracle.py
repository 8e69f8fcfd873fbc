"""The CPU oracle against every golden vector and known answer the reference's
own tests hold for this path, plus transformers' fp32 Llama (CPU only)."""
import json
import math
import os

import numpy as np
import pytest

from lcr_b200 import checkpoint as ck

GOLDEN = os.path.join(os.path.dirname(__file__), "golden")


# --- RoPE table: tests/test_config.cpp:120-182 of the reference -------------

def test_rope_unscaled_known_answer(oracle_lib):
    g = ck.Geometry(hidden_size=2048, intermediate_size=5632, num_layers=22, num_heads=32,
                    num_kv_heads=32, head_dim=64, vocab_size=32000, rope_theta=10000.0,
                    rope_scaling=False)
    f = oracle_lib.rope_inv_freq(g)
    assert f.size == 32
    for i in range(32):
        want = 10000.0 ** (-(2 * i) / 64.0)
        assert abs(f[i] - want) <= want * 1e-6


def test_rope_llama3_bands_known_answer(oracle_lib):
    f = oracle_lib.rope_inv_freq(ck.LLAMA_3_2_1B)
    old, low_w, high_w = 8192.0, 8192.0, 2048.0
    bands = [0, 0, 0]
    for i in range(32):
        base = 500000.0 ** (-(2 * i) / 64.0)
        wl = 2 * math.pi / base
        if wl < high_w:
            want, b = base, 0
        elif wl > low_w:
            want, b = base / 32.0, 1
        else:
            s = (old / wl - 1.0) / 3.0
            want, b = (1 - s) * base / 32.0 + s * base, 2
        bands[b] += 1
        assert abs(f[i] - want) <= abs(want) * 1e-5
    assert all(n > 0 for n in bands)
    assert abs(f[0] - 1.0) < 1e-9
    slowest = 500000.0 ** (-62.0 / 64.0)
    assert abs(f[31] - slowest / 32.0) <= slowest * 1e-6
    assert np.all(np.diff(f) < 0)


def test_rope_bit_exact_vs_reference_code(oracle_lib):
    """The reference's own compute_rope_inv_freq, compiled from its sources
    (fixture made by tests/golden/make_golden.py)."""
    with open(os.path.join(GOLDEN, "ref_rope.json")) as fh:
        ref = json.load(fh)
    geoms = {
        "llama-3.2-1b": ck.LLAMA_3_2_1B,
        "unscaled": ck.Geometry(hidden_size=2048, intermediate_size=5632, num_layers=22,
                                num_heads=32, num_kv_heads=32, head_dim=64, vocab_size=32000,
                                rope_theta=10000.0, rope_scaling=False),
    }
    for name, g in geoms.items():
        ours = oracle_lib.rope_inv_freq(g).view(np.uint32)
        assert ours.tolist() == ref[name]["inv_freq_bits"], name


# --- Sampling: tests/test_kernels.cu:468-508 of the reference ----------------

def test_sampling_known_answers(oracle_lib):
    vocab = 4096
    lg = np.full(vocab, -20.0, np.float32)
    lg[1234], lg[99], lg[7] = 5.0, 4.0, 3.0
    assert oracle_lib.sample(lg, 0.0, 0, 1.0, 0.0) == 1234
    assert oracle_lib.sample(lg, 0.0, 0, 1.0, 0.999) == 1234
    assert oracle_lib.sample(lg, 1.0, 1, 1.0, 0.5) == 1234
    for u in (0.01, 0.5, 0.99):
        assert oracle_lib.sample(lg, 1.0, 0, 0.9, u) in (1234, 99)
    pair = np.full(vocab, -60.0, np.float32)
    pair[3] = pair[9] = 1.0
    assert oracle_lib.sample(pair, 1.0, 0, 1.0, 0.25) == 3
    assert oracle_lib.sample(pair, 1.0, 0, 1.0, 0.75) == 9
    assert oracle_lib.sample(pair, 0.0, 0, 1.0, 0.5) == 3


def test_sampling_matches_direct_definition(oracle_lib):
    """Top-k/top-p on random logits against a numpy statement of the same
    definition (double precision; decisions far from the boundaries agree)."""
    rng = np.random.default_rng(5)
    agree = 0
    for trial in range(40):
        lg = rng.normal(0, 2.0, 3000).astype(np.float32)
        t, k, p, u = 0.8, int(rng.integers(0, 60)), float(rng.uniform(0.5, 1.0)), float(rng.uniform())
        s = (lg.astype(np.float64) - lg.max()) / t
        e = np.exp(s)
        order = np.lexsort((np.arange(lg.size), -s))
        m = min(k if k > 0 else lg.size, 1024)
        probs = e[order[:m]] / e.sum()
        cum = np.cumsum(probs)
        keep = m if p >= 1.0 else min(m, int(np.searchsorted(cum, p)) + 1)
        target = u * cum[keep - 1]
        want = order[min(int(np.searchsorted(cum[:keep], target)), keep - 1)]
        got = oracle_lib.sample(lg, t, k, p, u)
        agree += got == want
    assert agree >= 38


def test_argmax_tie_lowest_index(oracle_lib):
    lg = np.zeros(1000, np.float32)
    lg[[17, 400, 999]] = 3.0
    assert oracle_lib.argmax(lg) == 17


def test_det_expf_error_bound(oracle_lib):
    xs = np.concatenate([np.linspace(-87.9, 88.0, 4001), np.linspace(-1, 1, 2001)]).astype(np.float32)
    worst = 0.0
    for x in xs:
        got = oracle_lib.det_expf(float(x))
        want = math.exp(float(x))
        worst = max(worst, abs(got - want) / float(np.spacing(np.float32(want))))
    assert worst <= 2.0
    assert oracle_lib.det_expf(-100.0) == 0.0


def test_philox_known_answers(oracle_lib):
    """Philox4x32-10 known-answer vectors published with the Random123 library
    (Salmon et al., SC'11)."""
    assert oracle_lib.philox([0, 0, 0, 0], [0, 0]) == [0x6627E8D5, 0xE169C58D, 0xBC57AC4C, 0x9B00DBD8]
    assert oracle_lib.philox([0xFFFFFFFF] * 4, [0xFFFFFFFF] * 2) == [0x408F276D, 0x41C83B0E, 0xA20BC7C6, 0x6D5451FD]
    assert oracle_lib.philox([0x243F6A88, 0x85A308D3, 0x13198A2E, 0x03707344],
                             [0xA4093822, 0x299F31D0]) == [0xD16CFE09, 0x94FDCCEB, 0x5001E420, 0x24126EA1]
    u = oracle_lib.philox_uniform(123, 7, 3)
    assert 0.0 <= u < 1.0


def test_tree_sum_close_to_fsum(oracle_lib):
    e = np.random.default_rng(1).random(128256).astype(np.float32)
    assert abs(oracle_lib.tree_sum_1024(e) - math.fsum(e.tolist())) < 1e-2


# --- KV page accounting: tests/test_kernels.cu:442-464 of the reference -------

def test_paged_reserve_accounting(oracle_lib):
    layers, max_pages, page = 1, 64, 16
    t = np.full((layers, max_pages), -1, np.int32)
    mapped = oracle_lib.paged_reserve(t, page, 0, 10, 0, 64)
    assert mapped * page == 16  # one page: 16 positions live
    mapped = oracle_lib.paged_reserve(t, page, 10, 33, mapped, 64)
    assert mapped * page == 48
    again = oracle_lib.paged_reserve(t, page, 33, 40, mapped, 64)
    assert again == mapped
    assert t[0, :3].tolist() == [0, 1, 2]


def test_paged_reserve_layer_order_and_exhaustion(oracle_lib):
    t = np.full((3, 8), -1, np.int32)
    m = oracle_lib.paged_reserve(t, 16, 0, 20, 0, 100)
    assert m == 6 and t[:, :2].tolist() == [[0, 1], [2, 3], [4, 5]]
    assert oracle_lib.paged_reserve(np.full((3, 8), -1, np.int32), 16, 0, 20, 0, 5) == -1


def test_page_permutation_is_a_permutation(oracle_lib):
    p = oracle_lib.page_permutation(1000, 42)
    assert sorted(p.tolist()) == list(range(1000))
    assert p.tolist() != list(range(1000))
    assert p.tolist() == oracle_lib.page_permutation(1000, 42).tolist()


# --- Kernel maths vs nested loops (tests/test_kernels.cu:126-304) -------------

def _bf16(x):
    return ck.float_to_bf16_bits(np.asarray(x, np.float32))


def test_rmsnorm_and_fused_residual(oracle_lib):
    rng = np.random.default_rng(20260904)
    x = _bf16(rng.normal(size=(5, 2048)))
    w = _bf16(rng.normal(0, 0.5, 2048))
    xf, wf = ck.bf16_bits_to_float(x), ck.bf16_bits_to_float(w)
    want = xf / np.sqrt((xf.astype(np.float64) ** 2).mean(1, keepdims=True) + 1e-5) * wf
    got = oracle_lib.rmsnorm(x, w, 1e-5, round_out=False)
    assert np.abs(got - want).max() <= 3e-2 * np.abs(want).max()
    d = _bf16(rng.normal(size=(5, 2048)))
    normed, xnew = oracle_lib.add_residual_rmsnorm(x, d, w, 1e-5)
    s = xf + ck.bf16_bits_to_float(d)
    assert np.array_equal(xnew, _bf16(s))


def test_attention_nested_loop_matches_softmax(oracle_lib):
    rng = np.random.default_rng(3)
    H, KV, D, P = 8, 2, 64, 37
    q = _bf16(rng.normal(size=H * D))
    k = _bf16(rng.normal(size=P * KV * D))
    v = _bf16(rng.normal(size=P * KV * D))
    out = oracle_lib.attention(q, k, v, H, KV, D, P)
    qf = ck.bf16_bits_to_float(q).reshape(H, D)
    kf = ck.bf16_bits_to_float(k).reshape(P, KV, D)
    vf = ck.bf16_bits_to_float(v).reshape(P, KV, D)
    for h in range(H):
        s = kf[:, h // 4] @ qf[h] / 8.0
        p = np.exp(s - s.max())
        p /= p.sum()
        assert np.allclose(out[h * D:(h + 1) * D], p @ vf[:, h // 4], atol=1e-5)


# --- The decode step vs transformers' fp32 Llama ------------------------------

@pytest.fixture(scope="module")
def tiny_fixture():
    return np.load(os.path.join(GOLDEN, "tiny_seed0_hf.npz"))


def test_decode_step_matches_transformers_fp32(oracle_lib, tiny_fixture):
    fx = tiny_fixture
    block = ck.cached(ck.TINY, 0)
    m = oracle_lib.Model(block, 64)
    prompt = fx["prompt"]
    assert prompt.tolist() == ck.prompt_ids(0, 32).tolist()
    for pos, tok in enumerate(prompt):
        out = m.decode(int(tok), pos, oracle_lib.MODE_FP32, taps=pos == len(prompt) - 1)
    logits, taps = out
    ref = fx["logits_first2"][0]
    assert np.abs(logits - ref).max() < 1e-4
    hf = fx["taps_prompt_last"]  # embed, layer_0, final norm
    assert np.abs(taps[0] - hf[0]).max() < 1e-6
    assert np.abs(taps[1] - hf[1]).max() < 1e-5
    assert np.abs(taps[-1] - hf[-1]).max() < 1e-4
    pos, toks = len(prompt), []
    for step in range(16):
        nxt = oracle_lib.argmax(logits)
        toks.append(nxt)
        np.testing.assert_array_equal(np.argsort(-logits, kind="stable")[:8], fx["top_ids"][step][:8])
        logits = m.decode(nxt, pos, oracle_lib.MODE_FP32)
        pos += 1
    assert toks == fx["greedy"].tolist()


def test_bf16_mode_close_to_fp32(oracle_lib):
    block = ck.cached(ck.TINY, 0)
    a, b = oracle_lib.Model(block, 16), oracle_lib.Model(block, 16)
    for pos, tok in enumerate(ck.prompt_ids(0, 8)):
        la = a.decode(int(tok), pos, oracle_lib.MODE_FP32)
        lb = b.decode(int(tok), pos, oracle_lib.MODE_BF16)
    assert np.abs(la - lb).max() < 3e-2
    assert float(la @ lb / np.linalg.norm(la) / np.linalg.norm(lb)) > 0.999


def test_weight_bytes_per_token(oracle_lib):
    g = ck.LLAMA_3_2_1B
    assert g.weight_bytes_per_token() == 2_471_628_800
    assert int(oracle_lib.lib().orc_weight_bytes_per_token(oracle_lib.config_of(g))) == 2_471_628_800
    assert g.kv_bytes_per_position() == 32_768


def test_bf16_reproducibility_floor_1b(oracle_lib):
    """Two summation orders of the same bf16-storage algorithm (the reference's)
    drift apart by more than the 3e-2 max-abs the tiny model meets: that spread
    is the floor any implementation sits on. The 1B GPU gates are therefore
    relative to it: cosine >= 0.999 (tools/validate_main.cu:149-153) and no
    further from fp32 than 1.5x the bf16-storage algorithm itself is."""
    block = ck.cached(ck.LLAMA_3_2_1B, 1)
    a, b, f = (oracle_lib.Model(block, 16) for _ in range(3))
    worst = 0.0
    for pos, tok in enumerate(ck.prompt_ids(1, 12)):
        la = a.decode(int(tok), pos, oracle_lib.MODE_BF16)
        lb = b.decode(int(tok), pos, oracle_lib.MODE_BF16_REORDERED)
        lf = f.decode(int(tok), pos, oracle_lib.MODE_FP32)
        worst = max(worst, float(np.abs(la - lb).max()))
        for l in (la, lb):
            rms = np.sqrt(np.mean((l - lf) ** 2)) / np.sqrt(np.mean(lf ** 2))
            assert rms <= 0.03  # the algorithm itself sits near 0.02 here
            assert float(l @ lf / np.linalg.norm(l) / np.linalg.norm(lf)) >= 0.999
    assert worst > 3e-2, worst


def test_chunk_prefill_matches_token_steps(oracle_lib):
    """orc_prefill (the chunked prefill, GEMMs over the chunk) computes what
    the token-by-token decode computes: fp32 to summation order, the bf16
    modes to the rounding of a few intermediate values (and, in the
    reference's bf16 mode, of the prefill's bf16 probabilities)."""
    block = ck.cached(ck.TINY, 0)
    prompt = ck.prompt_ids(0, 40)
    for mode, tol in ((oracle_lib.MODE_FP32, 1e-5), (oracle_lib.MODE_FP32_KV_BF16, 1e-3),
                      (oracle_lib.MODE_BF16, 2e-2)):
        a, b = oracle_lib.Model(block, 64), oracle_lib.Model(block, 64)
        for pos, tok in enumerate(prompt):
            la = a.decode(int(tok), pos, mode)
        b.prefill(prompt[:25], 0, mode, logits=False)
        lb = b.prefill(prompt[25:], 25, mode)
        assert np.abs(la - lb).max() <= tol, mode
        nxt = int(np.argmax(la))
        assert np.abs(a.decode(nxt, 40, mode) - b.decode(nxt, 40, mode)).max() <= tol, mode


def test_bf16_kv_cache_floor_1b(oracle_lib):
    """The committed configuration-2 fixture is the fp32 oracle's own output
    (reproduced here from its script's first step), and the oracle with fp32
    activations but the reference's bf16 KV cache sits about 0.033 from it:
    the floor of the cache format, above the north-star 3e-2 max-abs."""
    fx = np.load(os.path.join(os.path.dirname(__file__), "golden", "c2_fp32_1b.npz"))
    block = ck.cached(ck.LLAMA_3_2_1B, 1)
    assert np.array_equal(fx["prompt"], ck.prompt_ids(1, 128))
    f32 = oracle_lib.Model(block, 136).prefill(fx["prompt"], 0, oracle_lib.MODE_FP32)
    assert np.abs(f32 - fx["logits0"]).max() <= 1e-4
    assert int(np.argmax(f32)) == int(fx["ids"][0])
    kv16 = oracle_lib.Model(block, 136).prefill(fx["prompt"], 0, oracle_lib.MODE_FP32_KV_BF16)
    d = float(np.abs(kv16 - fx["logits0"]).max())
    assert 0.02 < d < 0.05, d

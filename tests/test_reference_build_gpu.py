"""The reference runtime itself on the GPU, built from its own sources by
baseline/Makefile (no reference files are read at run time: the binaries in
baseline/_ref travel with the repository):

* ref_bench_stock  -- the reference's Model, kernels and cuBLAS, unmodified;
* ref_bench_dropin -- the same Model with its kernel launchers forwarding to
  liblcr_b200 (baseline/kernels_b200.cu).

Both load the checkpoint this package writes (config.json +
model.safetensors through the reference's SafetensorsArchive). The drop-in
must reproduce the stock build within the north-star tolerance, the stock
build must agree with the fp32 oracle, and this library's own decode context
must produce the reference's greedy ids."""
import os
import subprocess

import numpy as np
import pytest

import oracle
from lcr_b200 import checkpoint as ck
from lcr_b200 import runtime as rt

pytestmark = pytest.mark.gpu

torch = pytest.importorskip("torch")
if not torch.cuda.is_available():
    pytest.skip("needs a CUDA device", allow_module_level=True)

REPO = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
BIN = os.path.join(REPO, "baseline", "_ref")
if not (os.path.exists(os.path.join(BIN, "ref_bench_stock")) and os.path.exists(os.path.join(BIN, "ref_bench_dropin"))):
    pytest.skip("the reference baseline binaries are not built (make -C baseline)", allow_module_level=True)

MAX_ABS = 3e-2
MIN_COS = 0.999


def cos(a, b):
    a, b = np.asarray(a, np.float64), np.asarray(b, np.float64)
    return float(a @ b / np.linalg.norm(a) / np.linalg.norm(b))


@pytest.fixture(scope="module")
def ckpt(tmp_path_factory):
    d = tmp_path_factory.mktemp("tiny_ckpt")
    block = ck.cached(ck.TINY, 0)
    ck.write_safetensors(str(d), block)
    prompt = ck.prompt_ids(0, 32)
    prompt.astype(np.int32).tofile(str(d / "prompt.bin"))
    return block, str(d), prompt


def run_ref(which, ckpt_dir, paged, steps=16):
    out = os.path.join(ckpt_dir, f"logits_{which}_{int(paged)}.bin")
    cmd = [os.path.join(BIN, f"ref_bench_{which}"), "--model", ckpt_dir, "--prompt",
           os.path.join(ckpt_dir, "prompt.bin"), "--steps", str(steps), "--max-seq", "64",
           "--warmup", "1", "--logits-out", out] + (["--paged"] if paged else [])
    r = subprocess.run(cmd, capture_output=True, text=True, timeout=300)
    assert r.returncode == 0, r.stderr[-2000:]
    import json

    rep = json.loads(r.stdout.strip().splitlines()[-1])
    return np.fromfile(out, dtype=np.float32), rep


@pytest.mark.parametrize("paged", [False, True])
def test_dropin_matches_stock_reference(ckpt, paged):
    block, d, prompt = ckpt
    stock, rs = run_ref("stock", d, paged)
    drop, rd = run_ref("dropin", d, paged)
    assert stock.size == block.geom.vocab_size
    assert np.abs(drop - stock).max() <= MAX_ABS and cos(drop, stock) >= MIN_COS
    assert rd["ids"] == rs["ids"]
    # the oracle restates the reference: the reference itself is within the
    # north-star gates of the fp32 evaluation, and of the bf16 one closely
    ref32, ref16 = oracle.Model(block, 64), oracle.Model(block, 64)
    l32 = ref32.prefill(prompt, 0, oracle.MODE_FP32)
    l16 = ref16.prefill(prompt, 0, oracle.MODE_BF16)
    tok16 = oracle.Model(block, 64)
    for pos, tok in enumerate(prompt):
        lt16 = tok16.decode(int(tok), pos, oracle.MODE_BF16)
    print(f"reference build (paged={paged}) vs oracle: fp32 {np.abs(stock - l32).max():.5f}, "
          f"bf16 chunk {np.abs(stock - l16).max():.5f}, bf16 per-token {np.abs(stock - lt16).max():.5f}")
    assert np.abs(stock - l32).max() <= MAX_ABS and cos(stock, l32) >= MIN_COS
    assert np.abs(stock - l16).max() <= 1e-2
    # and this library's decode context generates the reference's greedy ids
    m = rt.Model(block, max_seq=64, paged=paged, page_order_seed=3 if paged else 0)
    m.prefill(prompt)
    got = m.logits_to_host()
    assert np.abs(got - stock).max() <= MAX_ABS and cos(got, stock) >= MIN_COS
    first = int(np.argmax(got))
    ids = [first] + m.generate_greedy(first, len(rs["ids"]) - 1).tolist()
    assert ids == rs["ids"]

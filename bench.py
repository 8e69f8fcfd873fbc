"""Benchmark: Llama-3.2-1B bf16 batch-1 decode.

Workload (config 2): random-init Llama-3.2-1B geometry (seed 1), a 128-id
prompt, then greedy decode over positions 128..383 with a contiguous KV cache.
A step is one decoded token. The K timed steps cycle through that 256-token
window (the position is reset to 128 every 256 tokens; the prompt stays
cached). The decode step streams 2.47 GB of weights, far more than the 126 MB
L2, so no L2 flush is needed between steps.

  value  device throughput: tokens/s from CUDA events on the context's stream
         around graph launches of the step, token feedback on the device.
  e2e    the same through the C ABI with host buffers, one lcr_step_host call
         per step: the token and position go down from host memory, the step
         runs, the next token comes back with the status, synchronising each
         step (the reference's decode loop).
  roofline  decode_step_kernel, the dominant kernel (one persistent launch per
         token): algorithmic bytes per launch (weights + the KV read at the
         window's mean context) / the CUDA-event time per launch measured
         here, against MEASURED_PEAKS.json; traffic is the DRAM bytes of one
         launch from the committed ncu summary. The standalone streaming
         GEMV of each matrix is timed beside it (per_matrix_layer0).

Multi-GPU (torchrun): every rank decodes its own independent sequence on its
own GPU with its own weight replica -- the reference has no collective on this
path, so there is none; value = all ranks' tokens / the slowest rank's time.

batched  config 4 on the batched context in the same run:
         64 sequences kept in slots by continuous batching, tcgen05 projections;
         decode steps timed with CUDA events (see batched_bench).
prefill  config 5's 2048-token prefill chunk on tcgen05 (see prefill_bench).
long_context  config 3: bs1 decode after an 8192-id
         prompt over shuffled 16-position pages (see long_context_bench).

config5  BASELINE configs[4] at this run's GPU count: the 512-request set
         (lognormal contexts, median 2048, sigma 1.0, clipped to [512, 32768],
         seed 4) split over the ranks by longest-processing-time, each rank
         prefilling its prompts in 2048-token chunks and decoding 256 greedy
         tokens per request; aggregate tok/s over the slowest rank's
         CUDA-event time.
reference_gpu  the reference's own build (its src/ compiled unmodified for
         sm_100 with cuBLAS, baseline/Makefile) on the same GPU and config 2:
         a baseline, not the target. reference_dropin: the same Model with its
         kernel launchers forwarding to this library.

--impl reference: the reference has no CPU implementation of the decode step,
so its arm is the fp32 host evaluation (oracle port) of the same workload on
the host cores, rank 0 only.
"""
import argparse
import json
import os
import subprocess
import sys
import time

REPO = os.path.dirname(os.path.abspath(__file__))
sys.path.insert(0, REPO)
sys.path.insert(0, os.path.join(REPO, "llama-cuda-runtime_b200"))

import numpy as np  # noqa: E402

PROMPT = 128
WINDOW = 256
METRIC = "Llama-3.2-1B bf16 decode tok/s (bs1, config 2)"


def measured_peaks():
    try:
        with open(os.path.join(REPO, "MEASURED_PEAKS.json")) as f:
            p = json.load(f)
        return float(p["hbm_gbs"]), "measured"
    except Exception:
        return 6650.0, "fallback"


def profile_traffic():
    """DRAM bytes of one decode_step_kernel launch from the committed ncu summary."""
    path = os.path.join(REPO, "profiles", "decode_step_1b.md")
    try:
        for line in open(path):
            if line.startswith("traffic_bytes_per_launch:"):
                return int(line.split(":")[1].strip())
    except OSError:
        pass
    return None


class Clocks:
    """nvidia-smi clock samples during the timed region."""

    def __init__(self, index):
        self.index = index
        self.proc = None
        self.path = f"/tmp/lcr_clocks_{os.getpid()}.csv"

    def __enter__(self):
        try:
            self.proc = subprocess.Popen(
                ["nvidia-smi", f"--id={self.index}",
                 "--query-gpu=clocks.sm,clocks.max.sm,clocks_event_reasons.active,"
                 "clocks_event_reasons.hw_slowdown,clocks_event_reasons.hw_thermal_slowdown,"
                 "clocks_event_reasons.sw_thermal_slowdown,clocks_event_reasons.sw_power_cap",
                 "--format=csv,noheader,nounits", "-lms", "50"],
                stdout=open(self.path, "w"), stderr=subprocess.DEVNULL)
        except OSError:
            self.proc = None
        return self

    def __exit__(self, *exc):
        if self.proc is not None:
            self.proc.terminate()
            self.proc.wait()

    def summary(self):
        try:
            rows = [l.split(",") for l in open(self.path).read().strip().splitlines()]
        except OSError:
            return None
        rows = [[c.strip() for c in r] for r in rows if len(r) >= 7]
        if not rows:
            return None
        sm = [float(r[0]) for r in rows if r[0].replace(".", "").isdigit()]
        reasons = set()
        names = ["hw_slowdown", "hw_thermal_slowdown", "sw_thermal_slowdown", "sw_power_cap"]
        for r in rows:
            for n, v in zip(names, r[3:7]):
                if v.lower() == "active":
                    reasons.add(n)
        return {"sm_mhz": float(np.median(sm)) if sm else None,
                "sm_max_mhz": float(rows[0][1]) if rows[0][1].replace(".", "").isdigit() else None,
                "reasons": sorted(reasons), "samples": len(rows)}


def dist_setup(n_gpus, backend=None):
    """One process per GPU from the torchrun environment. NCCL on GPUs; gloo
    (host tensors) when asked for or when there is no GPU."""
    world = int(os.environ.get("WORLD_SIZE", "1"))
    rank = int(os.environ.get("RANK", "0"))
    local = int(os.environ.get("LOCAL_RANK", "0"))
    if world > 1:
        import datetime

        import torch
        import torch.distributed as dist

        backend = backend or ("nccl" if torch.cuda.is_available() else "gloo")
        kw = {}
        if backend == "nccl":
            torch.cuda.set_device(local)
            kw["device_id"] = torch.device(f"cuda:{local}")
        dist.init_process_group(backend, timeout=datetime.timedelta(seconds=300), **kw)
    return world, rank, local


def barrier(world):
    if world > 1:
        import torch.distributed as dist

        dist.barrier()


def reduce_max(world, value):
    """The largest `value` over all ranks (every rank takes part)."""
    if world == 1:
        return value
    import torch
    import torch.distributed as dist

    dev = "cuda" if dist.get_backend() == "nccl" else "cpu"
    t = torch.tensor([value], dtype=torch.float64, device=dev)
    dist.all_reduce(t, op=dist.ReduceOp.MAX)
    return float(t.item())


def reduce_sum(world, value):
    if world == 1:
        return value
    import torch
    import torch.distributed as dist

    dev = "cuda" if dist.get_backend() == "nccl" else "cpu"
    t = torch.tensor([value], dtype=torch.float64, device=dev)
    dist.all_reduce(t, op=dist.ReduceOp.SUM)
    return float(t.item())


def reduce_argmax(world, value):
    """The rank holding the largest `value` (every rank takes part)."""
    if world == 1:
        return 0
    import torch
    import torch.distributed as dist

    dev = "cuda" if dist.get_backend() == "nccl" else "cpu"
    t = torch.zeros(world, dtype=torch.float64, device=dev)
    t[dist.get_rank()] = value
    dist.all_reduce(t, op=dist.ReduceOp.SUM)
    return int(torch.argmax(t).item())


def aggregate(world, rank_ms, steps):
    """Whole-job throughput of `world` replicas that each decoded `steps`
    tokens: (slowest rank's ms, all ranks' tokens / that time)."""
    max_ms = reduce_max(world, rank_ms)
    return max_ms, world * steps / (max_ms / 1000.0)


def cpu_baseline(block, seconds=12.0, max_tokens=64):
    """The fp32 host evaluation (oracle port) on this host's cores at config
    2's positions: the prompt's first 127 ids prefilled as one chunk
    (untimed), then decode steps from position 127 on -- the prompt's last id,
    then the oracle's own greedy ids -- for about `seconds`."""
    import oracle

    from lcr_b200 import checkpoint as ck

    m = oracle.Model(block, PROMPT + max_tokens + 1)
    prompt = ck.prompt_ids(1, PROMPT)
    m.prefill(prompt[:-1], 0, oracle.MODE_FP32, logits=False)
    tok, pos = int(prompt[-1]), PROMPT - 1
    t0 = time.perf_counter()
    n = 0
    while n < max_tokens and time.perf_counter() - t0 < seconds:
        tok = oracle.argmax(m.decode(tok, pos, oracle.MODE_FP32))
        pos += 1
        n += 1
    dt = time.perf_counter() - t0
    return {"value": n / dt, "unit": "tok/s", "cores": os.cpu_count(), "kind": "port",
            "sample": f"{n} Llama-3.2-1B greedy decode steps of the fp32 host oracle at positions "
                      f"{PROMPT - 1}..{PROMPT - 2 + n} after the 127-id prompt prefix (config 2's positions; "
                      f"OpenMP over output rows, {os.cpu_count()} threads)"}


def run_reference(args, world, rank):
    if rank != 0:
        return
    from lcr_b200 import checkpoint as ck

    block = ck.generate(ck.LLAMA_3_2_1B, 1)
    budget = max(1, min(args.steps, 48))
    base = cpu_baseline(block, seconds=60.0, max_tokens=budget)
    line = {"metric": METRIC, "value": base["value"], "unit": "tok/s", "impl": "reference",
            "n_gpus": args.gpus, "steps": args.steps, "warmup": args.warmup,
            "ms_per_step": 1000.0 / base["value"], "higher_is_better": True,
            "scaling": "weak", "vs_baseline": None, "dtype": "f32", "data": "synthetic",
            "config": {"workload": "config2: Llama-3.2-1B geometry, bs1 greedy decode, 128-id "
                                   "prompt, positions 128..383, contiguous KV",
                       "note": "the reference has no CPU decode path; this arm is the fp32 host "
                               "evaluation (oracle port) of the same step"},
            "cpu_baseline": base,
            "e2e": {"value": base["value"], "unit": "tok/s", "h2d_bytes_per_step": 0,
                    "d2h_bytes_per_step": 0}}
    print(json.dumps(line))


BATCH = 64
BATCH_TARGET = 128
BATCH_MAX_CTX = 4096


def batched_bench(block, weights_dev, local, world, steps, warmup):
    """Config 4 on the batched context: 64 slots kept
    full by continuous batching -- initial contexts uniform in [128, 4096]
    (seed 3), Poisson(4) arrivals per step replacing finished sequences, 128
    tokens each, temperature 0.8 / top-k 50 / top-p 0.9 with per-sequence
    Philox seeds, paged KV (16-position pages, shuffled pool). Admitted
    contexts get synthetic KV (lcr_batch_fill_kv, untimed: config 4 measures
    decode; the prefill chunk is measured by prefill_bench); admissions
    happen between steps, and the timed unit is the decode step: CUDA events
    on the batch stream around each step."""
    import torch

    from lcr_b200 import checkpoint as ck
    from lcr_b200 import runtime as rt
    from lcr_b200 import scheduler as sch

    g = ck.LLAMA_3_2_1B
    max_seq = BATCH_MAX_CTX + BATCH_TARGET + 16
    per_seq = (max_seq + 15) // 16
    pool_pages = (BATCH + 4) * per_seq
    bt = rt.Batch(block, weights_dev, device=local, max_batch=BATCH, max_seq=max_seq, page_size=16,
                  pool_pages=pool_pages)
    cb = sch.ContinuousBatcher(bt, page_size=16, pool_pages=pool_pages, page_seed=3,
                               temperature=0.8, top_k=50, top_p=0.9)
    for q in sch.config4_workload(np.random.default_rng(3), BATCH, BATCH_TARGET, 128, BATCH_MAX_CTX):
        cb.submit(q)
    arrivals = np.random.default_rng(4003)
    next_sid = BATCH

    def admit():
        nonlocal next_sid
        new, next_sid = sch.config4_arrivals(arrivals, next_sid, 4.0, BATCH_TARGET, 128, BATCH_MAX_CTX)
        for q in new:
            cb.submit(q)
        cb.fill()

    for _ in range(warmup):
        admit()
        cb.step()
    bt.sync()
    stream = torch.cuda.ExternalStream(bt.stream, device=f"cuda:{local}")
    events, tokens, kv_positions = [], 0, 0
    barrier(world)
    torch.cuda.synchronize()
    for _ in range(steps):
        admit()
        n = cb.active()
        kv_positions += sum(cb.slots[b].position for b in range(n))
        e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        e0.record(stream)
        tokens += cb.step()
        e1.record(stream)
        events.append((e0, e1))
    bt.sync()
    torch.cuda.synchronize()
    barrier(world)
    ms = sum(a.elapsed_time(b) for a, b in events)
    max_ms = reduce_max(world, ms)
    per_step_ms = max_ms / steps
    bytes_step = g.weight_bytes_per_token() + (kv_positions / steps) * g.kv_bytes_per_position()
    peak, _ = measured_peaks()
    out = {
        "workload": "config4: Llama-3.2-1B, 64 slots, contexts U[128,4096] (seed 3), Poisson(4) "
                    "arrivals/step replace finished sequences, 128 tokens each, temp 0.8 top-k 50 "
                    "top-p 0.9, per-sequence Philox, paged KV 16 (shuffled pool)",
        "value": round(world * tokens / (max_ms / 1000.0), 1), "unit": "tok/s",
        "ms_per_step": round(per_step_ms, 4), "steps": steps, "warmup": warmup,
        "mean_context": round(kv_positions / max(1, steps * BATCH), 1),
        "bytes_per_step": int(bytes_step),
        "hbm_gbs": round(bytes_step / (per_step_ms / 1000) / 1e9, 1),
        "frac_of_peak": round(bytes_step / (per_step_ms / 1000) / 1e9 / peak, 4),
        "gpu_launches_per_step": bt.step_launches(BATCH),
        "finished_sequences": cb.finished,
        "note": "admitted contexts get synthetic KV (seeded fill, untimed); decode steps timed",
    }
    bt.close()
    return out


LONG_PROMPT = 8192
LONG_DECODE = 256


def long_context_bench(block, weights_dev, local, short_ms_per_step, warmup=16):
    """Config 3 on the bs1 persistent step: an 8192-id
    prompt (seed 2) through lcr_prefill (its first 8191 ids in four tcgen05
    chunks of up to 2048 rows), then 256 greedy tokens at positions
    8191..8446 over a paged KV cache of 16-position pages in a seeded shuffled
    physical order (seed 2). The 256 steps are timed with CUDA events on the
    context's stream after `warmup` steps from the same position. Bytes per
    step are the weights plus the KV read at the window's mean context
    (reference main.cu:195-220). `prefill_ms` is the median wall time of three
    further synchronous lcr_prefill calls of the same 8191 ids from position 0
    (host ids in, device logits out; the first call, which also builds the
    chunk engine, is not counted).

    The attention shares: by bytes, the KV read over the step's bytes; by
    time, the step time added over config 2's (whose context is ~32x shorter)
    over this step time -- an estimate from the two measurements, since the
    step is one persistent launch."""
    import torch

    from lcr_b200 import checkpoint as ck
    from lcr_b200 import runtime as rt

    g = ck.LLAMA_3_2_1B
    m = rt.Model(block, weights_dev, device=local, max_seq=LONG_PROMPT + LONG_DECODE + 16, paged=True,
                 page_size=16, page_order_seed=2)
    prompt = ck.prompt_ids(2, LONG_PROMPT)
    m.prefill(prompt[:-1])
    prefill_times = []
    for _ in range(3):
        m.reset()
        t0 = time.perf_counter()
        m.prefill(prompt[:-1])
        prefill_times.append((time.perf_counter() - t0) * 1000.0)
    prefill_ms = float(np.median(prefill_times))
    pinned = torch.empty(2, dtype=torch.int32, pin_memory=True)
    pinned[0] = int(prompt[-1])
    m.reserve_length(LONG_PROMPT + LONG_DECODE)  # every page the timed steps write, mapped up front
    m.set_token(pinned.data_ptr(), LONG_PROMPT - 1)
    m.enqueue_steps(warmup)
    m.sync()
    stream = torch.cuda.ExternalStream(m.stream, device=f"cuda:{local}")
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    torch.cuda.synchronize()
    m.set_token(pinned.data_ptr(), LONG_PROMPT - 1)
    e0.record(stream)
    m.enqueue_steps(LONG_DECODE)
    e1.record(stream)
    m.sync()
    torch.cuda.synchronize()
    ms = e0.elapsed_time(e1) / LONG_DECODE
    ctx_mean = LONG_PROMPT + (LONG_DECODE - 1) / 2
    kv_bytes = ctx_mean * g.kv_bytes_per_position()
    step_bytes = g.weight_bytes_per_token() + kv_bytes
    peak, kind = measured_peaks()
    gbs = step_bytes / (ms / 1000) / 1e9
    out = {"workload": f"config3: Llama-3.2-1B bs1 greedy, {LONG_PROMPT}-id prompt (seed 2), "
                       f"{LONG_DECODE} tokens at positions {LONG_PROMPT - 1}..{LONG_PROMPT + LONG_DECODE - 2}, "
                       "paged KV 16 (seeded shuffled page order)",
           "value": round(1000.0 / ms, 2), "unit": "tok/s", "ms_per_step": round(ms, 5),
           "steps": LONG_DECODE, "warmup": warmup,
           "bytes_per_step": int(step_bytes), "hbm_gbs": round(gbs, 1),
           "frac_of_peak": round(gbs / peak, 4), "peak_source": kind,
           "attention_byte_share": round(kv_bytes / step_bytes, 4),
           "attention_time_share_est": round(max(0.0, ms - short_ms_per_step) / ms, 4),
           "prefill_ms": round(prefill_ms, 3),
           "prefill_tokens_per_s": round((LONG_PROMPT - 1) / (prefill_ms / 1000.0), 1),
           "prefill_workload": f"lcr_prefill of {LONG_PROMPT - 1} ids at position 0 into the same paged cache: "
                               "4 tcgen05 chunks (2048, 2048, 2048, 2047 rows), wall time of the synchronous call, "
                               "median of 3"}
    m.close()
    return out


PREFILL_CHUNK = 2048


def measured_bf16_tflops():
    try:
        with open(os.path.join(REPO, "MEASURED_PEAKS.json")) as f:
            return float(json.load(f)["bf16_tflops"]), "measured"
    except Exception:
        return 1590.0, "fallback"


def prefill_bench(block, weights_dev, local, reps=5):
    """Config 5's prefill chunk on one GPU: 2048 prompt
    tokens (seed 5) into an empty paged sequence (16-position pages, shuffled)
    through lcr_batch_prefill -- tcgen05 projections over the 2048 rows,
    causal flash attention, the last row's lm_head and sample. FLOPs per
    chunk: 2 x (non-embedding weights) x 2048 for the projections plus
    4 x heads x head_dim x 2048 x 2049 / 2 per layer for causal QK^T and PV,
    plus the one-row lm_head. CUDA events on the batch stream around each
    chunk, after two warm-up chunks; the chunk rewrites the same pages."""
    import torch

    from lcr_b200 import checkpoint as ck
    from lcr_b200 import runtime as rt

    g = ck.LLAMA_3_2_1B
    P = PREFILL_CHUNK
    pages = P // 16
    bt = rt.Batch(block, weights_dev, device=local, max_batch=1, max_seq=P, page_size=16, pool_pages=pages)
    bt.set_pages(0, np.random.default_rng(5).permutation(pages).astype(np.int32))
    bt.set_sampling(0, 0.0)
    ids = ck.prompt_ids(5, P)
    for _ in range(2):
        bt.prefill(0, ids, 0)
    bt.sync()
    stream = torch.cuda.ExternalStream(bt.stream, device=f"cuda:{local}")
    times = []
    for _ in range(reps):
        e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        e0.record(stream)
        bt.prefill(0, ids, 0)
        e1.record(stream)
        times.append((e0, e1))
    bt.sync()
    torch.cuda.synchronize()
    ms = sorted(a.elapsed_time(b) for a, b in times)[len(times) // 2]
    h, f, q, kv = g.hidden_size, g.intermediate_size, g.q_dim, g.kv_dim
    layer_params = (q + 2 * kv) * h + h * q + 2 * f * h + f * h
    proj = 2.0 * layer_params * g.num_layers * P
    attn = 4.0 * g.num_heads * g.head_dim * P * (P + 1) / 2 * g.num_layers
    head = 2.0 * g.vocab_size * h
    flops = proj + attn + head
    peak, kind = measured_bf16_tflops()
    tflops = flops / (ms / 1000) / 1e12
    bt.close()
    return {"workload": f"config5 prefill chunk: {P} prompt tokens (seed 5), Llama-3.2-1B, empty paged "
                        "sequence (16-position pages, shuffled)",
            "ms_per_chunk": round(ms, 3), "tok_per_s": round(P / (ms / 1000), 1),
            "flops_per_chunk": flops, "tflops": round(tflops, 1),
            "peak_tflops": peak, "peak_source": kind, "frac_of_peak": round(tflops / peak, 4),
            "reps": reps, "statistic": "median"}


def reference_gpu_bench(block, which="stock", steps=WINDOW - 1):
    """The reference runtime's own Model on this GPU at config 2
    (baseline/_ref/ref_bench_<which>, built by baseline/Makefile from the
    reference's sources): the seed-1 checkpoint written as config.json +
    model.safetensors and read by the reference's SafetensorsArchive, the
    128-id prompt, then `steps` greedy steps timed by the reference's own
    per-step GPU timer. Bytes per token follow the reference's formula at its
    mean length (src/main.cu:195-220)."""
    import shutil
    import tempfile

    from lcr_b200 import checkpoint as ck

    exe = os.path.join(REPO, "baseline", "_ref", f"ref_bench_{which}")
    if not os.path.exists(exe):
        return {"unavailable": f"baseline/_ref/ref_bench_{which} is not built (make -C baseline REF=... JSON_INC=...)"}
    tmp = tempfile.mkdtemp(prefix="lcr_ref_")
    try:
        ck.write_safetensors(tmp, block)
        ids = os.path.join(tmp, "prompt.bin")
        ck.prompt_ids(1, PROMPT).astype(np.int32).tofile(ids)
        out = subprocess.run([exe, "--model", tmp, "--prompt", ids, "--steps", str(steps),
                              "--max-seq", str(PROMPT + WINDOW + 8), "--warmup", "2"],
                             capture_output=True, text=True, timeout=900)
        if out.returncode != 0:
            return {"unavailable": f"ref_bench_{which} exited {out.returncode}: {out.stderr.strip()[-300:]}"}
        r = json.loads(out.stdout.strip().splitlines()[-1])
    finally:
        shutil.rmtree(tmp, ignore_errors=True)
    g = block.geom
    mean_len = r["prompt_tokens"] + (r["decode_steps"] + 1) / 2.0
    bytes_tok = g.weight_bytes_per_token() + mean_len * g.kv_bytes_per_position()
    peak, kind = measured_peaks()
    ms = r["decode_ms"] / r["decode_steps"]
    return {"build": "the reference's src/ for sm_100, cuBLAS projections, its own kernels"
                     if which == "stock" else
                     "the reference's Model and cuBLAS projections, its kernel launchers forwarding "
                     "to liblcr_b200 (baseline/kernels_b200.cu)",
            "value": round(r["decode_tokens_per_s"], 2), "unit": "tok/s", "ms_per_step": round(ms, 5),
            "steps": r["decode_steps"], "prefill_ms": round(r["prefill_ms"], 3),
            "hbm_gbs": round(bytes_tok / (ms / 1000) / 1e9, 1),
            "frac_of_peak": round(bytes_tok / (ms / 1000) / 1e9 / peak, 4), "peak_source": kind,
            "timer": "the reference's per-step GPU timer (ForwardStats::last_decode_ms), sample + "
                     "D2H of the id outside it",
            "loop_tok_per_s": round(r["loop_tokens_per_s"], 2),
            "greedy_ids": r["ids"][:16]}


def config5_bench(block, weights_dev, local, world, rank):
    """BASELINE configs[4] on this run's ranks (lcr_b200.serve.config5): the
    512-request set split by longest-processing-time over the ranks, each
    rank serving its shard on its own GPU with no communication; the
    aggregate decode tok/s is all ranks' decoded tokens over the slowest
    rank's CUDA-event time."""
    import types

    from lcr_b200 import serve

    args = types.SimpleNamespace(sequences=512, sigma=1.0, decode_tokens=256, slots=128,
                                 shard=f"{rank}/{world}", device=local)
    r = serve.config5(block, weights_dev, args)
    total_s = reduce_max(world, r["seconds"])
    decode_s = reduce_max(world, r["decode_seconds"])
    decoded = reduce_sum(world, r["decode_tokens"])
    prompt_tokens = reduce_sum(world, r["prompt_tokens"])
    slowest = reduce_argmax(world, r["seconds"])
    return {"workload": "config5: 512 requests, contexts lognormal(median 2048, sigma 1.0) clipped to "
                        "[512, 32768] (seed 4), LPT-sharded over the ranks, prompts prefilled in 2048-token "
                        "chunks, 256 greedy tokens each, paged KV 16, 128 slots per GPU",
            "n_gpus": world, "requests": 512, "prompt_tokens": int(prompt_tokens),
            "decode_tokens": int(decoded), "seconds": round(total_s, 3),
            "decode_tok_per_s": round(decoded / total_s, 1),
            "decode_tok_per_s_in_steps": round(decoded / decode_s, 1),
            "run_tok_per_s": round((decoded + prompt_tokens) / total_s, 1),
            "slowest_rank": int(slowest), "timing": "CUDA events on each rank's batch stream, max over ranks"}


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=2560)
    ap.add_argument("--warmup", type=int, default=64)
    ap.add_argument("--impl", default="ours", choices=["ours", "reference"])
    ap.add_argument("--no-cpu-baseline", action="store_true")
    ap.add_argument("--no-batched", action="store_true", help="skip the config-4 batched measurement")
    ap.add_argument("--batched-steps", type=int, default=64)
    ap.add_argument("--no-long-context", action="store_true",
                    help="skip the config-3 long-context measurement")
    ap.add_argument("--no-config5", action="store_true", help="skip the config-5 request set")
    ap.add_argument("--no-reference-gpu", action="store_true",
                    help="skip the reference build's measurement on this GPU")
    ap.add_argument("--min-timed-s", type=float, default=1.0,
                    help="repeat the K-step measurement until the timed block lasts this long")
    args = ap.parse_args()
    args.warmup = max(args.warmup, 3)
    world, rank, local = dist_setup(args.gpus)
    if args.impl == "reference":
        run_reference(args, world, rank)
        if world > 1:
            import torch.distributed as dist

            dist.destroy_process_group()
        return

    import torch

    from lcr_b200 import checkpoint as ck
    from lcr_b200 import runtime as rt

    torch.cuda.set_device(local)
    g = ck.LLAMA_3_2_1B
    block = ck.generate(g, 1)
    prompt = ck.prompt_ids(1, PROMPT)
    m = rt.Model(block, device=local, max_seq=PROMPT + WINDOW + 8)
    m.prefill(prompt[:-1])
    first = int(prompt[-1])
    stream = torch.cuda.ExternalStream(m.stream, device=f"cuda:{local}")

    pinned = torch.empty(2, dtype=torch.int32, pin_memory=True)
    tok_ptr = pinned.data_ptr()
    pinned[0] = first

    def enqueue(steps):
        """`steps` device-resident greedy steps in windows of WINDOW tokens:
        each window restarts at position PROMPT - 1 from the same token (an
        8-byte async copy from pinned memory), so the context stays in
        128..383 however many steps run."""
        done = 0
        while done < steps:
            n = min(WINDOW, steps - done)
            m.set_token(tok_ptr, PROMPT - 1)
            m.enqueue_steps(n)
            done += n

    # warm-up (graph capture happens on first use)
    enqueue(args.warmup)
    m.sync()

    # The K timed steps, repeated until the timed block lasts --min-timed-s
    # (so the clock sampler sees it): the median repetition is the value.
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    e0.record(stream)
    enqueue(args.steps)
    e1.record(stream)
    torch.cuda.synchronize()
    reps = int(reduce_max(world, max(1, int(np.ceil(args.min_timed_s * 1000.0 / max(e0.elapsed_time(e1), 1e-3))))))
    barrier(world)
    torch.cuda.synchronize()
    rep_ms = []
    with Clocks(local) as clk:
        events = []
        for _ in range(reps):
            a, b = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
            a.record(stream)
            enqueue(args.steps)
            b.record(stream)
            events.append((a, b))
        torch.cuda.synchronize()
        rep_ms = [a.elapsed_time(b) for a, b in events]
    m.sync()
    barrier(world)
    max_ms, value = aggregate(world, float(np.median(rep_ms)), args.steps)

    # end to end: host token in, host token out, every step
    e2e_steps = min(args.steps, 1024)
    pinned[0] = first
    m.set_token(tok_ptr, PROMPT - 1)
    m.sync()
    barrier(world)
    torch.cuda.synchronize()
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    e0.record(stream)
    pos = PROMPT - 1
    tok = int(first)
    for i in range(e2e_steps):
        if pos >= PROMPT - 1 + WINDOW:
            pos = PROMPT - 1
        # one call per step (lcr_step_host): H2D token + position (8 B), the
        # step, D2H next token + status (16 B), synchronised
        tok = m.step_host(tok, pos)
        pos += 1
    e1.record(stream)
    torch.cuda.synchronize()
    e2e_ms = reduce_max(world, e0.elapsed_time(e1))
    e2e_value = world * e2e_steps / (e2e_ms / 1000.0)

    # roofline of the dominant kernel (decode_step_kernel, one launch per
    # token); the standalone GEMV of each layer-0 matrix beside it
    peak, peak_kind = measured_peaks()
    per_matrix = {}
    names = ["qkv", "o_proj", "gate_up", "down", "lm_head"]
    h, f, q, kv, v = g.hidden_size, g.intermediate_size, g.q_dim, g.kv_dim, g.vocab_size
    bytes_of = {"qkv": (q + 2 * kv) * h * 2, "o_proj": h * q * 2, "gate_up": 2 * f * h * 2,
                "down": h * f * 2, "lm_head": v * h * 2}
    for i, name in enumerate(names):
        m.time_gemv(i, 0, 3)  # first launch of a kernel loads its module
        ms = m.time_gemv(i, 0, 20)
        per_matrix[name] = {"us": round(ms * 1000, 2),
                            "gbs": round(bytes_of[name] / (ms / 1000) / 1e9, 1)}
    batched = prefill = None
    if not args.no_batched:
        batched = batched_bench(block, m.weights_dev, local, world, args.batched_steps,
                                max(3, args.warmup // 4))
        prefill = prefill_bench(block, m.weights_dev, local)

    ms_per_step = max_ms / args.steps
    config5 = None
    if not args.no_config5:
        config5 = config5_bench(block, m.weights_dev, local, world, rank)
    long_ctx = None
    if not args.no_long_context:
        long_ctx = long_context_bench(block, m.weights_dev, local, ms_per_step)
    # positions 127..382 read 128..383 cached positions: mean 255.5
    ctx_mean = PROMPT + (WINDOW - 1) / 2
    step_bytes = g.weight_bytes_per_token() + ctx_mean * g.kv_bytes_per_position()
    achieved = step_bytes / (ms_per_step / 1000) / 1e9
    ref_gpu = ref_dropin = None
    if rank == 0 and world == 1 and not args.no_reference_gpu:
        ref_gpu = reference_gpu_bench(block, "stock")
        ref_dropin = reference_gpu_bench(block, "dropin")
    if rank == 0:
        base = None if args.no_cpu_baseline or world > 1 else cpu_baseline(block)
        clocks = clk.summary()
        line = {
            "metric": METRIC, "value": round(value, 2), "unit": "tok/s", "n_gpus": world,
            "steps": args.steps, "warmup": args.warmup, "ms_per_step": round(ms_per_step, 5),
            "timed_repetitions": reps,
            "higher_is_better": True, "scaling": "weak", "vs_baseline": None, "dtype": "bf16",
            "data": "synthetic (random-init weights, seed 1; uniform prompt ids)",
            "config": {"workload": "config2: Llama-3.2-1B geometry, bs1 greedy decode, 128-id "
                                   "prompt, positions 128..383, contiguous KV",
                       "global_batch": world, "seq_len": PROMPT + WINDOW,
                       "parallelism": f"replicas x{world} (independent sequences)",
                       "l2": "no flush: each step streams 2.47 GB > 126 MB L2"},
            "hbm": {"bytes_per_token": int(step_bytes),
                    "achieved_gbs": round(step_bytes / (ms_per_step / 1000) / 1e9, 1),
                    "frac_of_peak": round(step_bytes / (ms_per_step / 1000) / 1e9 / peak, 4),
                    "peak_gbs": peak},
            "roofline": {"kernel": "decode_step_kernel<2048, 2048, 8192, 64, 4, 0, 0, 1> "
                                   "(persistent step, tagged-word exchange between phases, "
                                   "one launch per token)",
                         "bound": "hbm", "achieved": round(achieved, 1), "peak": peak,
                         "unit": "GB/s", "frac": round(achieved / peak, 4),
                         "traffic": profile_traffic(), "peak_source": peak_kind,
                         "algorithmic_bytes_per_launch": int(step_bytes),
                         "launch_us": round(ms_per_step * 1000, 2),
                         "per_matrix_layer0": per_matrix},
            "e2e": {"value": round(e2e_value, 2), "unit": "tok/s", "h2d_bytes_per_step": 8,
                    "d2h_bytes_per_step": 16, "steps": e2e_steps},
            "gpu_launches": reps * args.steps * m.step_launches(),
            "clocks": clocks,
            "cpu_baseline": base,
            "batched": batched,
            "prefill": prefill,
            "long_context": long_ctx,
            "config5": config5,
            "reference_gpu": ref_gpu,
            "reference_dropin": ref_dropin,
        }
        print(json.dumps(line))
    m.close()
    if world > 1:
        import torch.distributed as dist

        barrier(world)
        dist.destroy_process_group()


if __name__ == "__main__":
    main()

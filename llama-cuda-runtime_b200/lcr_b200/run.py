"""llama-run for the B200 build (the reference's src/main.cu CLI surface, on the
seeded random-init checkpoints or a safetensors checkpoint directory: there is
no tokenizer on this path, so the prompt is token ids).

  python -m lcr_b200.run --model 1b --prompt-len 128 --max-tokens 256 --bench
  python -m lcr_b200.run --model tiny --prompt 1,2,3 --max-tokens 16 --json
  python -m lcr_b200.run --model /path/to/checkpoint --prompt 1,2,3 --max-tokens 16

--bench / --json report the numbers of main.cu:195-334: decode tokens/s,
ms/token, bytes per token (weights + mean-length KV read) and the achieved
bandwidth against --peak-bandwidth (GB/s).
"""
from __future__ import annotations

import argparse
import json
import sys
import time

import numpy as np

from . import checkpoint as ck
from . import runtime as rt

MODELS = {"1b": ck.LLAMA_3_2_1B, "tiny": ck.TINY}


PHASES = ("qkv", "attn", "o", "gate_up", "down")


def print_trace(t: np.ndarray, layers: int, sm_mhz: float = 1965.0) -> None:
    """Phase timeline of one persistent decode step: per phase, the consumers'
    working time (previous barrier departure -> next barrier arrival) and the
    barrier wait, averaged over layers (mean / max over CTAs, microseconds);
    for the matrix phases also the time consumer thread 0 waited on weight
    stages to land and the producer waited on free ring slots (SM cycles at
    `sm_mhz`)."""
    t = t.astype(np.int64)
    t0 = t[:, 0].min()
    nbar = 5 * layers
    arrive = t[:, 1:2 * nbar:2]
    depart = t[:, 2:2 * nbar + 1:2]
    start = np.concatenate([t[:, :1], depart[:, :-1]], axis=1)
    work = (arrive - start) / 1e3
    wait = (depart - arrive) / 1e3
    prod = t[:, 256:256 + nbar + 1]
    pro = t[:, 163:163 + nbar]
    prologue = (pro - start) / 1e3
    cwait = t[:, 340:340 + nbar + 1] / sm_mhz
    pwait = t[:, 424:424 + nbar + 1] / sm_mhz
    print(f"{'phase':8s} {'work mean':>10s} {'work max':>9s} {'prologue':>9s} {'wait mean':>10s} "
          f"{'producer lead':>14s} {'data wait':>10s} {'slot wait':>10s}  (us)")
    for k, name in enumerate(PHASES):
        cols = list(range(k, nbar, 5))
        lead = (start[:, cols] - prod[:, cols]) / 1e3  # >0: producer started this phase earlier
        print(f"{name:8s} {work[:, cols].mean():10.2f} {work[:, cols].max(axis=0).mean():9.2f} "
              f"{prologue[:, cols].mean():9.2f} {wait[:, cols].mean():10.2f} {lead.mean():14.2f} "
              f"{cwait[:, cols].mean():10.2f} {pwait[:, cols].mean():10.2f}")
    lm = (t[:, 255] - depart[:, -1]) / 1e3
    total = (t[:, 255].max() - t0) / 1e3
    print(f"lm_head  {lm.mean():10.2f} {lm.max():9.2f} {'':9s} {'':10s} {'':14s} "
          f"{cwait[:, nbar].mean():10.2f} {pwait[:, nbar].mean():10.2f}")
    print(f"step (consumers start -> last CTA done): {total:.1f} us")


def main(argv=None) -> int:
    ap = argparse.ArgumentParser(prog="lcr_b200.run")
    ap.add_argument("--model", default="1b",
                    help="1b or tiny (seeded random-init checkpoints) or a checkpoint directory "
                         "(config.json + safetensors)")
    ap.add_argument("--seed", type=int, default=None, help="checkpoint seed (1b: 1, tiny: 0)")
    ap.add_argument("--prompt", default=None, help="comma-separated token ids")
    ap.add_argument("--prompt-len", type=int, default=128, help="uniform random prompt length")
    ap.add_argument("--max-tokens", type=int, default=128)
    ap.add_argument("--max-seq", type=int, default=0)
    ap.add_argument("--paged", action="store_true")
    ap.add_argument("--page-size", type=int, default=16)
    ap.add_argument("--page-order-seed", type=int, default=0)
    ap.add_argument("--splits", type=int, default=0)
    ap.add_argument("--device", type=int, default=0)
    ap.add_argument("--temperature", type=float, default=0.0)
    ap.add_argument("--top-k", type=int, default=0)
    ap.add_argument("--top-p", type=float, default=0.95)
    ap.add_argument("--peak-bandwidth", type=float, default=8000.0, help="GB/s")
    ap.add_argument("--bench", action="store_true")
    ap.add_argument("--json", action="store_true")
    ap.add_argument("--fp32-act", action="store_true",
                    help="persistent step with fp32 activations (default: the reference's "
                         "bf16 storage rounding)")
    ap.add_argument("--no-persistent", action="store_true",
                    help="the multi-kernel step instead of the persistent kernel")
    ap.add_argument("--cuda-core-attention", action="store_true",
                    help="persistent step's attention phase on CUDA cores instead of the tensor pipe")
    ap.add_argument("--grid-barriers", action="store_true",
                    help="persistent step's phases meet at grid barriers instead of exchanging tagged words")
    ap.add_argument("--per-token-prefill", action="store_true",
                    help="the prompt as decode steps instead of tcgen05 chunks")
    ap.add_argument("--trace", action="store_true",
                    help="per-phase timeline of the last decode step (persistent kernel)")
    ap.add_argument("--trace-out", default=None,
                    help="with --trace: also save the raw per-CTA timestamps (.npy)")
    args = ap.parse_args(argv)

    seed = args.seed if args.seed is not None else (1 if args.model == "1b" else 0)
    if args.model in MODELS:
        geom = MODELS[args.model]
        block = ck.generate(geom, seed)
    else:
        block = ck.load_checkpoint(args.model)
        geom = block.geom
    if args.prompt:
        prompt = np.array([int(t) for t in args.prompt.split(",")], np.int32)
    else:
        prompt = ck.prompt_ids(seed, args.prompt_len)
    max_seq = args.max_seq or (len(prompt) + args.max_tokens + 8)
    t0 = time.perf_counter()
    m = rt.Model(block, device=args.device, max_seq=max_seq, paged=args.paged,
                 page_size=args.page_size, attention_splits=args.splits,
                 page_order_seed=args.page_order_seed,
                 flags=(rt.FLAG_TRACE if args.trace else 0)
                 | (rt.FLAG_FP32_ACT if args.fp32_act else 0)
                 | (rt.FLAG_NO_PERSISTENT if args.no_persistent else 0)
                 | (rt.FLAG_CUDA_CORE_ATTENTION if args.cuda_core_attention else 0)
                 | (rt.FLAG_GRID_BARRIERS if args.grid_barriers else 0)
                 | (rt.FLAG_PER_TOKEN_PREFILL if args.per_token_prefill else 0))
    load_ms = (time.perf_counter() - t0) * 1000

    t0 = time.perf_counter()
    logits_ptr = m.prefill(prompt)
    prefill_ms = (time.perf_counter() - t0) * 1000
    tokens = []
    t0 = time.perf_counter()
    if args.temperature <= 0.0:
        first = int(np.argmax(m.logits_to_host()))
        tokens = [first] + m.generate_greedy(first, max(0, args.max_tokens - 1)).tolist()
    else:
        # The host draws the uniform, as main.cu:442-443 does with mt19937_64.
        rng = np.random.default_rng(seed)
        for _ in range(args.max_tokens):
            tok = m.sample(logits_ptr, args.temperature, args.top_k, args.top_p,
                           float(np.float32(rng.random())))
            tokens.append(tok)
            logits_ptr = m.decode(tok)
    decode_ms = (time.perf_counter() - t0) * 1000
    steps = max(1, args.max_tokens - 1)
    mean_len = len(prompt) + (steps + 1) / 2.0
    bytes_per_token = geom.weight_bytes_per_token() + mean_len * geom.kv_bytes_per_position()
    report = {
        "runtime": "llama-cuda-runtime_b200", "model": geom.name, "seed": seed,
        "load_ms": load_ms, "prompt_tokens": int(len(prompt)), "prefill_ms": prefill_ms,
        "decode_steps": steps, "decode_ms": decode_ms,
        "decode_ms_per_token": decode_ms / steps,
        "decode_tokens_per_second": steps / (decode_ms / 1000),
        "weight_bytes_per_token": geom.weight_bytes_per_token(),
        "kv_bytes_per_position": geom.kv_bytes_per_position(),
        "bytes_per_token": bytes_per_token,
        "achieved_bandwidth_bytes_per_second": bytes_per_token / (decode_ms / 1000 / steps),
        "peak_bandwidth_bytes_per_second": args.peak_bandwidth * 1e9,
        "kv_layout": "paged" if args.paged else "contiguous", "kv_page_size": args.page_size,
        "sequence_length": int(len(prompt) + args.max_tokens), "tokens": tokens[:32],
    }
    report["bandwidth_utilization"] = (report["achieved_bandwidth_bytes_per_second"]
                                       / report["peak_bandwidth_bytes_per_second"])
    if args.trace:
        t = m.trace()
        print_trace(t, geom.num_layers)
        if args.trace_out:
            np.save(args.trace_out, t)
    if args.json:
        print(json.dumps(report))
    elif args.bench:
        print(f"decode  {steps} steps in {decode_ms:.2f} ms ({decode_ms / steps:.3f} ms/token, "
              f"{report['decode_tokens_per_second']:.1f} tokens/s)")
        print(f"achieved {report['achieved_bandwidth_bytes_per_second'] / 1e9:.0f} GB/s, "
              f"{100 * report['bandwidth_utilization']:.1f}% of {args.peak_bandwidth:.0f} GB/s")
    else:
        print(" ".join(str(t) for t in tokens))
    m.close()
    return 0


if __name__ == "__main__":
    sys.exit(main())

"""Batched serving workloads on the B200 build: continuous-batching decode
(config 4 of the benchmark set) and chunked prefill (config 5's 2048-token
chunk), on the seeded random-init Llama-3.2-1B checkpoint.

  python -m lcr_b200.serve --steps 64                 # 64 slots, config-4 arrivals
  python -m lcr_b200.serve --prefill 2048 --reps 5    # one prompt chunk, 5 times
  python -m lcr_b200.serve --layers 2 --steps 4       # a 2-layer model, for profiling
  python -m lcr_b200.serve --config5 --sequences 512  # prefill + decode of a request set

The reference decodes one sequence at a time (src/main.cu:456-466); this is
the batched counterpart. Admitted contexts get synthetic KV (seeded, untimed):
the decode steps are what is timed. Times are wall-clock around synchronised
work; bench.py reports the CUDA-event numbers.
"""
from __future__ import annotations

import argparse
import dataclasses
import json
import sys
import time

import numpy as np

from . import checkpoint as ck
from . import runtime as rt
from . import scheduler as sch


def main(argv=None) -> int:
    ap = argparse.ArgumentParser()
    ap.add_argument("--layers", type=int, default=0, help="override the model's layer count (profiling)")
    ap.add_argument("--slots", type=int, default=64)
    ap.add_argument("--steps", type=int, default=32)
    ap.add_argument("--warmup", type=int, default=4)
    ap.add_argument("--max-ctx", type=int, default=4096)
    ap.add_argument("--target", type=int, default=128, help="tokens each sequence decodes")
    ap.add_argument("--prefill", type=int, default=0, help="time one prompt chunk of this many tokens instead")
    ap.add_argument("--reps", type=int, default=3)
    ap.add_argument("--device", type=int, default=0)
    ap.add_argument("--config5", action="store_true",
                    help="serve a request set: lognormal contexts prefilled in chunks, greedy decode")
    ap.add_argument("--sequences", type=int, default=512, help="config5: requests (this process's share)")
    ap.add_argument("--decode-tokens", type=int, default=256)
    ap.add_argument("--sigma", type=float, default=1.0, help="config5: lognormal sigma of the contexts")
    ap.add_argument("--shard", default="0/1", help="config5: this process's shard i/N of the request set")
    ap.add_argument("--json", action="store_true")
    args = ap.parse_args(argv)

    geom = ck.LLAMA_3_2_1B
    if args.layers:
        geom = dataclasses.replace(geom, num_layers=args.layers)
    block = ck.generate(geom, 1)
    wdev = rt.upload_block(block, args.device)
    if args.config5:
        report = config5(block, wdev, args)
    elif args.prefill:
        report = prefill(block, wdev, args)
    else:
        report = decode(block, wdev, args)
    print(json.dumps(report) if args.json else "\n".join(f"{k}: {v}" for k, v in report.items()))
    return 0


def prefill(block, wdev, args) -> dict:
    P = args.prefill
    pages = (P + 15) // 16
    bt = rt.Batch(block, wdev, device=args.device, max_batch=1, max_seq=pages * 16, page_size=16,
                  pool_pages=pages)
    bt.set_pages(0, np.random.default_rng(5).permutation(pages).astype(np.int32))
    bt.set_sampling(0, 0.0)
    ids = ck.prompt_ids(5, P)
    bt.prefill(0, ids, 0)
    bt.sync()
    t0 = time.perf_counter()
    for _ in range(args.reps):
        bt.prefill(0, ids, 0)
    bt.sync()
    ms = (time.perf_counter() - t0) * 1000 / args.reps
    next_id = int(bt.read(1)[0])
    bt.close()
    return {"workload": f"prefill chunk of {P} tokens", "layers": block.geom.num_layers,
            "ms_per_chunk": ms, "tokens_per_second": P / (ms / 1000), "next_id": next_id}


def config5_requests(total: int, sigma: float, seed: int = 4) -> np.ndarray:
    """Contexts of config 5's request set: lognormal with median 2048 and the
    given sigma, clipped to [512, 32768] (seeded, the whole set)."""
    rng = np.random.default_rng(seed)
    return np.clip(np.round(2048.0 * np.exp(sigma * rng.standard_normal(total))), 512, 32768).astype(np.int64)


def shard_requests(contexts: np.ndarray, shard: int, shards: int, decode_tokens: int) -> list:
    """Longest-processing-time split of the request set over `shards`
    processes by expected bytes (context + decode tokens): request indices of
    shard `shard`."""
    order = np.argsort(-(contexts + decode_tokens), kind="stable")
    load = np.zeros(shards)
    owner = np.zeros(len(contexts), dtype=np.int64)
    for i in order:
        k = int(np.argmin(load))
        owner[i] = k
        load[k] += contexts[i] + decode_tokens
    return [int(i) for i in np.nonzero(owner == shard)[0]]


def config5(block, wdev, args) -> dict:
    """Serves this shard of the request set on one GPU: up to --slots
    sequences in flight, each admitted with its prompt prefilled in 2048-token
    chunks (lcr_batch_prefill), then greedy decode of --decode-tokens tokens
    with continuous batching. Reports decode tokens per second over the whole
    run (prefill included) and over the decode steps alone, timed with CUDA
    events on the batch's stream."""
    import torch

    g = block.geom
    shard, shards = (int(x) for x in args.shard.split("/"))
    contexts = config5_requests(args.sequences, args.sigma)
    mine = shard_requests(contexts, shard, shards, args.decode_tokens)
    max_seq = int(contexts.max()) + args.decode_tokens + 16
    per_seq = (max_seq + 15) // 16
    slots = min(args.slots, max(1, len(mine)))
    # Pages for the largest requests in flight at once.
    need = sorted(((int(contexts[i]) + args.decode_tokens + 15) // 16 for i in mine), reverse=True)
    pool = sum(need[:slots]) + slots
    bt = rt.Batch(block, wdev, device=args.device, max_batch=slots, max_seq=max_seq, page_size=16,
                  pool_pages=pool)
    cb = sch.ContinuousBatcher(bt, page_size=16, pool_pages=pool, page_seed=4, temperature=0.0,
                               prefill_chunk=2048)
    for i in mine:
        prompt = ck.prompt_ids(10_000 + i, int(contexts[i])) % g.vocab_size
        cb.submit(sch.Sequence(sid=i, context=int(contexts[i]), target=args.decode_tokens, seed=i,
                               prompt=prompt.astype(np.int32)))
    stream = torch.cuda.ExternalStream(bt.stream, device=f"cuda:{args.device}")

    def event():
        e = torch.cuda.Event(enable_timing=True)
        e.record(stream)
        return e

    prompt_tokens = int(sum(int(contexts[i]) for i in mine))
    decoded = 0
    steps = 0
    step_events = []
    bt.sync()
    e_start = event()
    while cb.waiting or cb.active():
        cb.fill()
        e0 = event()
        done = cb.step()
        step_events.append((e0, event()))
        decoded += done
        steps += 1
    e_end = event()
    bt.sync()
    torch.cuda.synchronize()
    total = e_start.elapsed_time(e_end) / 1000.0
    t_decode = sum(a.elapsed_time(b) for a, b in step_events) / 1000.0
    bt.close()
    return {"workload": f"config5 shard {shard}/{shards}: {len(mine)} of {args.sequences} requests, contexts "
                        f"lognormal(median 2048, sigma {args.sigma}) in [512, 32768] (seed 4), prompts prefilled "
                        f"in 2048-token chunks, {args.decode_tokens} greedy tokens each, {slots} slots",
            "requests": len(mine), "prompt_tokens": prompt_tokens, "decode_tokens": decoded, "steps": steps,
            "seconds": total, "decode_seconds": t_decode,
            "decode_tokens_per_second": decoded / total,
            "decode_tokens_per_second_in_steps": decoded / t_decode,
            "prefill_tokens_per_second": prompt_tokens / max(1e-9, total - t_decode)}


def decode(block, wdev, args) -> dict:
    g = block.geom
    max_seq = args.max_ctx + args.target + 16
    per_seq = (max_seq + 15) // 16
    pool = (args.slots + 4) * per_seq
    bt = rt.Batch(block, wdev, device=args.device, max_batch=args.slots, max_seq=max_seq, page_size=16,
                  pool_pages=pool)
    cb = sch.ContinuousBatcher(bt, page_size=16, pool_pages=pool, page_seed=3)
    for q in sch.config4_workload(np.random.default_rng(3), args.slots, args.target, 128, args.max_ctx):
        cb.submit(q)
    arrivals = np.random.default_rng(4003)
    sid = args.slots
    tokens = 0
    positions = 0
    t_run = 0.0
    n = 0
    for i in range(args.warmup + args.steps):
        new, sid = sch.config4_arrivals(arrivals, sid, 4.0, args.target, 128, args.max_ctx)
        for q in new:
            cb.submit(q)
        cb.fill()
        bt.sync()
        timed = i >= args.warmup
        n = cb.active()
        if timed:
            positions += sum(cb.slots[b].position for b in range(n))
        t0 = time.perf_counter()
        done = cb.step()
        bt.sync()
        if timed:
            t_run += time.perf_counter() - t0
            tokens += done
    ms = t_run * 1000 / args.steps
    step_bytes = g.weight_bytes_per_token() + positions / args.steps * g.kv_bytes_per_position()
    report = {"workload": f"continuous batching, {args.slots} slots, contexts U[128, {args.max_ctx}]",
              "layers": g.num_layers, "steps": args.steps, "ms_per_step": ms,
              "tokens_per_second": tokens / t_run, "bytes_per_step": step_bytes,
              "achieved_gbs": step_bytes / (ms / 1000) / 1e9, "finished_sequences": cb.finished,
              "launches_per_step": bt.step_launches(n)}
    bt.close()
    return report


if __name__ == "__main__":
    sys.exit(main())

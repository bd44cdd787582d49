"""The reference's Triton paged attention and this repository's kernels on
the same inputs, on this machine.

Inputs follow the reference's own attention benchmark
(paged_attention_benchmark.py:48-197): bf16 K/V arenas with one private page
run per beam (block table = arange), every beam at the full history length,
N(0, 1) queries, keys and values; the causal case adds a valid current token
per beam, the readout case has `--query-length` queries per beam.  Both
implementations get the same tensors.  Each is timed two ways: the
reference's method (wall clock over `--repeats` calls after `--warmup`, one
synchronize at each end, launch overhead included) and CUDA events around
`--repeats` back-to-back calls (device time per call).  The maximum absolute
difference between the two outputs is reported.  Prints one JSON line per
case.

The reference is imported from ``baseline/_ref`` (or ``--reference``).
"""
from __future__ import annotations

import argparse
import json
import math
import sys
import time
from pathlib import Path

HERE = Path(__file__).resolve().parent
sys.path.insert(0, str(HERE.parent))

import torch  # noqa: E402


def wall_ms(fn, warmup: int, repeats: int) -> float:
    for _ in range(warmup):
        fn()
    torch.cuda.synchronize()
    started = time.perf_counter()
    for _ in range(repeats):
        fn()
    torch.cuda.synchronize()
    return 1e3 * (time.perf_counter() - started) / repeats


def event_ms(fn, warmup: int, repeats: int) -> float:
    for _ in range(warmup):
        fn()
    torch.cuda.synchronize()
    a, b = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    a.record()
    for _ in range(repeats):
        fn()
    b.record()
    torch.cuda.synchronize()
    return a.elapsed_time(b) / repeats


def case(ref_attention, ours, *, kind, batch, history, query_length, page, heads, hw,
         warmup, repeats, seed):
    torch.manual_seed(seed + batch)
    dev, dt = torch.device("cuda"), torch.bfloat16
    blocks = max(1, math.ceil(history / page))
    keys = torch.randn(batch * blocks, page, heads, hw, device=dev, dtype=dt)
    values = torch.randn_like(keys)
    table = torch.arange(batch * blocks, device=dev, dtype=torch.int32).view(batch, blocks)
    lengths = torch.full((batch,), history, device=dev, dtype=torch.int32)
    q = torch.randn(batch, heads, 1 if kind == "causal" else query_length, hw, device=dev,
                    dtype=dt)
    kw = {}
    if kind == "causal":
        kw = dict(current_key=torch.randn(batch, heads, hw, device=dev, dtype=dt),
                  current_value=torch.randn(batch, heads, hw, device=dev, dtype=dt),
                  current_valid=torch.ones(batch, device=dev, dtype=torch.bool))
    run_ref = lambda: ref_attention(q, keys, values, table, lengths, **kw)
    run_ours = lambda: ours(q, keys, values, table, lengths, **kw)
    diff = float((run_ref().float() - run_ours().float()).abs().max().item())
    kv_bytes = 2 * batch * history * heads * hw * 2
    line = {"case": kind, "batch": batch, "history": history, "queries": q.shape[2],
            "page": page, "heads": heads, "head_width": hw, "max_abs_diff": diff,
            "kv_bytes": kv_bytes}
    for name, fn in (("reference_triton", run_ref), ("b200", run_ours)):
        line[f"{name}_wall_ms"] = wall_ms(fn, warmup, repeats)
        line[f"{name}_device_ms"] = event_ms(fn, warmup, repeats)
    line["device_speedup"] = line["reference_triton_device_ms"] / line["b200_device_ms"]
    return line


def main() -> None:
    parser = argparse.ArgumentParser()
    parser.add_argument("--reference", type=Path, default=HERE / "_ref")
    parser.add_argument("--warmup", type=int, default=4)
    parser.add_argument("--repeats", type=int, default=50)
    parser.add_argument("--query-length", type=int, default=381)
    parser.add_argument("--seed", type=int, default=17)
    args = parser.parse_args()
    if not (args.reference / "paged_attention.py").exists():
        print(json.dumps({"unavailable": f"reference modules not found under {args.reference}"}))
        return
    sys.path.insert(0, str(args.reference))
    import paged_attention as ref
    from graph_rewrite_system_b200.paged_attention import paged_attention as ours

    shapes = [  # (batch, page, heads): the reference's published shape, then this path's
        (512, 8, 6), (1000, 8, 6), (512, 16, 8), (1000, 16, 8)]
    for kind in ("causal", "readout"):
        for batch, page, heads in shapes:
            print(json.dumps(case(ref.paged_attention, ours, kind=kind, batch=batch,
                                  history=64, query_length=args.query_length, page=page,
                                  heads=heads, hw=32, warmup=args.warmup,
                                  repeats=args.repeats, seed=args.seed)), flush=True)


if __name__ == "__main__":
    main()

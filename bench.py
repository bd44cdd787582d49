"""Benchmark of the B200 beam-search decode path (one JSON line on rank 0).

    python bench.py [--gpus N] [--steps K] [--warmup W] [--impl b200|reference]
                    [--workload rollout|decode-attention|update-gemm|graph-mlp|cache-churn]

Workloads (seeded synthetic inputs; the reference's hwb6 circuit, rule set
and checkpoint are not available):

* ``rollout`` (default): the full beam-search step - synthetic 6-qubit,
  259-gate circuit, width-256 / 8-head / 4 causal + 4 readout-graph-layer
  model with seeded random weights, bf16, beam 1000 per GPU, depth 64 (the
  metric's T), page 16, up to 2048 candidates per state ranked to 16 per
  parent and 16000 globally.  A step is one search level.  One whole untimed
  64-level search runs first; then a fresh 64-level search whose last K
  levels are timed (levels 65-K..64; the 64-K levels before them, at least
  W, are the untimed warm-up).  With N > 1 the beam is sharded (1000 beams
  per GPU, weak scaling).  The decode-attention microbenchmark below is
  measured in the same run and reported under ``paged_attention``.
* ``update-gemm``: the readout graph layers' update projection with its GELU
  as one tcgen05 tensor-core launch, GELU(x [300000, 512] @ W^T + b), against
  the library GEMM + bias+GELU pair on the same inputs.
* ``graph-mlp``: one readout graph layer's update MLP + residual + LayerNorm
  as one fused tensor-core launch (the GELU activation never leaves shared
  memory), M = 300000 rows, against the same layer as two GEMM launches.
* ``decode-attention``: the shared-prefix paged decode microbenchmark -
  512 beams, one query token each, 8 heads x 32, bf16, 381 shared s0 node
  keys, 64 action K/V entries per beam in pages of 16, block tables from a
  random prefix tree.  A step is one decode-attention launch over all beams.
* ``cache-churn``: the paged KV cache alone - 1000 live beams, 4 layers x 8
  heads x 32 bf16 K/V per action, page 16, depth 64; each level forks every
  beam into 5 children, keeps the top 1000 by seeded uniform scores, appends
  one token to each (copy-on-write of partial tail pages) and releases the
  previous level (refcount reclaim).  A step is one level; the L2 is flushed
  before each timed level.

Timing: each timed step is bracketed by CUDA events on the launching stream,
with barrier + synchronize around the timed region and the max over ranks.
Every workload reads inputs larger than L2 each step: the rollout's beam
state (hundreds of MB of bf16 activations per level), the decode benchmark's
16 rotating input sets, the GEMM's two rotating 307 MB inputs.  ``e2e`` runs
the workload through the public Python API with host inputs and host
results inside the timed region (the rollout: the same K levels of another
fresh search, each ``DeviceBeamSearch.step()`` plus the level's children
copied to pinned host memory; ``e2e_full_search`` adds the whole
``run()`` from the host circuit to the host beam summary).  Clocks are sampled with
nvidia-smi during the timed region.  ``--impl reference`` times the CPU
oracle (the reference's algorithm restated on the host) on the same workload.
"""
from __future__ import annotations

import argparse
import gc
import json
import os
from pathlib import Path
import statistics
import subprocess
import sys
import tempfile
import time

# grow the caching allocator's segments in place: the beam state tensors grow
# with the slot count level by level, and fresh cudaMalloc calls for them
# stall whole levels
os.environ.setdefault("PYTORCH_CUDA_ALLOC_CONF", "expandable_segments:True")

import torch  # noqa: E402

ROOT = Path(__file__).resolve().parent
sys.path.insert(0, str(ROOT))

METRIC = "beam-state decode steps/s at B=1000,T=64; paged-attn HBM GB/s vs peak"
PROBE_LEAD_US = 15.0                  # device busy time ahead of a probed launch
DECODE_INPUT_COPIES = 16              # 16 x ~11.2 MB = 180 MB > 126 MB L2
_SLEEP_RATE: list[float] = []


def sleep_cycles_per_us() -> float:
    """torch.cuda._sleep counts a device clock whose rate is not the SM
    clock's; measure it once against CUDA events (cycles per microsecond)."""
    if not _SLEEP_RATE:
        cycles = 2_000_000
        a, b = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        torch.cuda.synchronize()
        a.record()
        torch.cuda._sleep(cycles)
        b.record()
        torch.cuda.synchronize()
        _SLEEP_RATE.append(cycles / max(a.elapsed_time(b) * 1e3, 1e-3))
    return _SLEEP_RATE[0]


def device_sleep_us(us: float) -> None:
    """Keep the current stream busy for about `us` microseconds."""
    torch.cuda._sleep(max(1, int(us * sleep_cycles_per_us())))


def queue_ahead_us(steps: int) -> float:
    """Device sleep long enough for the host to enqueue `steps` API calls
    (~200 us each), at least 30 ms."""
    return max(30_000.0, steps * 200.0)

L2_FLUSH_BYTES = 256 << 20


def measured_peaks() -> dict:
    path = ROOT / "MEASURED_PEAKS.json"
    if path.exists():
        data = json.loads(path.read_text())
        return {"hbm_gbs": data["hbm_gbs"], "bf16_tflops": data["bf16_tflops"],
                "bf16_tflops_sustained": data.get("bf16_tflops_sustained"), "source": "measured"}
    return {"hbm_gbs": 6650.0, "bf16_tflops": 1590.0, "bf16_tflops_sustained": 1400.0,
            "source": "fallback"}


class KernelProbe:
    """Times every `every`-th call of one kernel wrapper of
    graph_rewrite_system_b200.kernels with CUDA events on the launching stream
    while active, and adds up those calls' algorithmic bytes and FLOPs
    (sampling keeps the probe's own device time out of most of the step)."""

    def __init__(self, name: str, work_fn, every: int = 4):
        self.name, self.work_fn, self.every = name, work_fn, every
        self.events, self.bytes, self.flops, self.calls = [], 0, 0, 0

    def __enter__(self):
        from graph_rewrite_system_b200 import kernels

        self.module, self.original = kernels, getattr(kernels, self.name)

        def timed(*a, **kw):
            # launches recorded into a CUDA graph are not timed (and the
            # probe's own sleep and events must not be captured with them)
            if torch.cuda.is_current_stream_capturing():
                return self.original(*a, **kw)
            self.calls += 1
            if self.calls % self.every:
                return self.original(*a, **kw)
            start = torch.cuda.Event(enable_timing=True)
            end = torch.cuda.Event(enable_timing=True)
            # keep the device busy while the host issues the launch, so the
            # events bracket the kernel and not the host call (~20 us)
            device_sleep_us(PROBE_LEAD_US)
            start.record()
            out = self.original(*a, **kw)
            end.record()
            self.events.append((start, end))
            nbytes, flops = self.work_fn(*a, **kw)
            self.bytes += nbytes
            self.flops += flops
            return out

        setattr(kernels, self.name, timed)
        return self

    def __exit__(self, *exc):
        setattr(self.module, self.name, self.original)

    def roofline(self, peaks: dict, kernel: str, traffic_ratio) -> dict | None:
        """Roofline of the sampled launches: their arithmetic intensity
        (algorithmic FLOPs / algorithmic bytes) against the ridge point of the
        measured peaks (sustained bf16 FLOP/s / HBM bytes/s) decides the
        bound, so `frac` is achieved / attainable; the other resource's
        fraction is reported beside it.  `traffic_ratio`: DRAM bytes /
        algorithmic bytes of this kernel from a committed ncu capture (None
        when absent)."""
        if not self.events:
            return None
        torch.cuda.synchronize()
        n = len(self.events)
        ms = sum(s.elapsed_time(e) for s, e in self.events) / n
        flops, nbytes = self.flops / n, self.bytes / n
        tflops = flops / (ms * 1e-3) / 1e12
        gbs = nbytes / (ms * 1e-3) / 1e9
        peak_tf = peaks["bf16_tflops_sustained"] or peaks["bf16_tflops"]
        peak_gbs = peaks["hbm_gbs"]
        intensity = flops / nbytes
        ridge = peak_tf * 1e12 / (peak_gbs * 1e9)
        memory_bound = intensity < ridge
        achieved, peak, unit = (gbs, peak_gbs, "GB/s") if memory_bound else \
            (tflops, peak_tf, "TFLOP/s")
        return {"bound": "hbm" if memory_bound else "tensor", "achieved": achieved,
                "peak": peak, "unit": unit, "frac": achieved / peak,
                "traffic": traffic_ratio * nbytes if traffic_ratio else None,
                "kernel": kernel, "launches": n, "sampled_every": self.every,
                "avg_launch_ms": ms, "algorithmic_flops_per_launch": flops,
                "algorithmic_bytes_per_launch": nbytes,
                "intensity_flop_per_byte": intensity, "ridge_flop_per_byte": ridge,
                "tensor_achieved_tflops": tflops, "tensor_frac": tflops / peak_tf,
                "hbm_achieved_gbs": gbs, "hbm_frac": gbs / peak_gbs,
                "peak_source": f"{peaks['source']} hbm_gbs; tensor: {peaks['source']} "
                               f"bf16_tflops_sustained (kernel timed inside the long search "
                               f"step)"}


def gemm_work(x, weight, bias=None, *, gelu=False, residual=None, zero_row=None, out=None,
              status=None):
    """Algorithmic bytes and FLOPs of one kernels.gemm call: read x, the
    weight, the bias and the residual once, write the output; 2 M N K."""
    m, k = x.shape
    n = weight.shape[0]
    nbytes = 2 * (m * k + n * k + m * n) + (4 * n if bias is not None else 0)
    nbytes += 2 * m * n if residual is not None else 0
    nbytes += m if zero_row is not None else 0
    return nbytes, 2.0 * m * n * k


def launch_count() -> int:
    """Kernels launched so far by libgrs_b200.so (its own launch counter)."""
    from graph_rewrite_system_b200 import _lib

    return int(_lib.lib().grs_launch_count())


def profiled_traffic(kernel: str) -> float | None:
    """DRAM bytes per launch of `kernel` from the committed ncu summary."""
    path = ROOT / "profiles" / "traffic.json"
    if not path.exists():
        return None
    return json.loads(path.read_text()).get(kernel)


class ClockSampler:
    FIELDS = ("index,clocks.sm,clocks.max.sm,power.draw,clocks_event_reasons.active,"
              "clocks_event_reasons.hw_slowdown,clocks_event_reasons.hw_thermal_slowdown,"
              "clocks_event_reasons.sw_thermal_slowdown,clocks_event_reasons.sw_power_cap")

    def __init__(self, device_index: int):
        self.device_index = device_index
        self.proc = None
        self.path = None

    def __enter__(self):
        fd, self.path = tempfile.mkstemp(suffix=".csv")
        os.close(fd)
        try:
            self.proc = subprocess.Popen(
                ["nvidia-smi", f"--id={self.device_index}", f"--query-gpu={self.FIELDS}",
                 "--format=csv,noheader,nounits", "-lms", "50"],
                stdout=open(self.path, "w"), stderr=subprocess.DEVNULL)
        except (FileNotFoundError, OSError):
            self.proc = None
        # the sampler's start-up (NVML initialisation) must be over before the
        # timed region opens: wait for its first sample
        deadline = time.time() + 10.0
        while self.proc is not None and time.time() < deadline:
            if os.path.getsize(self.path) > 0 and open(self.path).read().count("\n") >= 1:
                break
            time.sleep(0.02)
        time.sleep(0.06)
        self.window_start = time.time()
        return self

    def __exit__(self, *exc):
        self.window_end = time.time()
        if self.proc is not None:
            self.proc.terminate()
            try:
                self.proc.wait(timeout=5)
            except subprocess.TimeoutExpired:
                self.proc.kill()

    def summary(self) -> dict:
        rows = []
        if self.path and os.path.exists(self.path):
            for line in open(self.path):
                parts = [p.strip() for p in line.split(",")]
                if len(parts) >= 9:
                    rows.append(parts)
            os.unlink(self.path)
        if not rows:
            return {"sm_mhz": None, "sm_max_mhz": None, "reasons": ["unsampled"]}
        def num(x):
            try:
                return float(x)
            except ValueError:
                return None
        sm = [num(r[1]) for r in rows if num(r[1]) is not None]
        reasons = set()
        names = ("hw_slowdown", "hw_thermal_slowdown", "sw_thermal_slowdown", "sw_power_cap")
        for r in rows:
            for name, flag in zip(names, r[5:9]):
                if flag.lower() == "active":
                    reasons.add(name)
        return {"sm_mhz": statistics.median(sm) if sm else None,
                "sm_max_mhz": num(rows[0][2]), "reasons": sorted(reasons), "samples": len(rows)}


def dist_setup(n_gpus: int):
    world = int(os.environ.get("WORLD_SIZE", "1"))
    rank = int(os.environ.get("RANK", "0"))
    local = int(os.environ.get("LOCAL_RANK", "0"))
    if world > 1:
        import datetime
        import torch.distributed as dist

        torch.cuda.set_device(local)
        dist.init_process_group("nccl", timeout=datetime.timedelta(seconds=120),
                                device_id=torch.device("cuda", local))
    return world, rank, local


def barrier(world: int, device):
    if world > 1:
        import torch.distributed as dist

        dist.barrier(device_ids=[device.index])


def max_over_ranks(value: float, world: int, device) -> float:
    if world == 1:
        return value
    import torch.distributed as dist

    t = torch.tensor([value], device=device, dtype=torch.float64)
    dist.all_reduce(t, op=dist.ReduceOp.MAX)
    return float(t.item())


# ---------------------------------------------------------------------------
# decode-attention workload
# ---------------------------------------------------------------------------
def run_decode_attention(args, world, rank, device):
    from graph_rewrite_system_b200.paged_attention import paged_attention
    from graph_rewrite_system_b200.workloads import decode_attention_workload

    # independent input sets (own tables, arenas, queries) whose total is
    # larger than L2; step i uses set i % copies, so every step reads cold data
    copies = DECODE_INPUT_COPIES
    sets = [decode_attention_workload(device, seed=rank * 1000 + c) for c in range(copies)]
    w = sets[0]
    out = torch.empty_like(w.query)
    flush = torch.empty(L2_FLUSH_BYTES, dtype=torch.uint8, device=device)
    stream = torch.cuda.current_stream(device)

    def step(i):
        x = sets[i % copies]
        paged_attention(x.query, x.key_cache, x.value_cache, x.block_table, x.lengths,
                        shared_key=x.shared_key, shared_value=x.shared_value, out=out)

    for i in range(max(args.warmup, copies)):
        step(i)
    torch.cuda.synchronize(device)
    barrier(world, device)
    torch.cuda.synchronize(device)
    start, end = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    with ClockSampler(device.index) as clocks:
        # hold the device while the host enqueues the timed launches, so the
        # events bracket device time and not the Python call overhead
        device_sleep_us(queue_ahead_us(args.steps))
        launches0 = launch_count()
        start.record(stream)
        for i in range(args.steps):
            step(i)
        end.record(stream)
        launches = launch_count() - launches0
        torch.cuda.synchronize(device)
    barrier(world, device)
    kernel_ms = start.elapsed_time(end) / args.steps
    kernel_ms = max_over_ranks(kernel_ms, world, device)

    # the earlier 8-CTA cluster design on the same inputs, for comparison
    from graph_rewrite_system_b200 import _lib

    lib = _lib.lib()

    def step_cluster(i):
        x = sets[i % copies]
        q, kc = x.query, x.key_cache
        rc = lib.grs_decode_attention_shared_cluster(
            q.data_ptr(), q.stride(0), q.stride(1), kc.data_ptr(), x.value_cache.data_ptr(),
            kc.stride(0), kc.stride(1), kc.stride(2), x.block_table.data_ptr(),
            x.block_table.stride(0), x.block_table.shape[1], x.lengths.data_ptr(), kc.shape[0],
            None, None, 0, 0, None, x.shared_key.data_ptr(), x.shared_value.data_ptr(),
            x.shared_key.shape[0], out.data_ptr(), out.stride(0), out.stride(1), q.shape[0],
            q.shape[1], kc.shape[1], None, stream.cuda_stream)
        if rc != 0:
            raise RuntimeError(f"cluster decode returned {rc}")

    for i in range(copies):
        step_cluster(i)
    torch.cuda.synchronize(device)
    device_sleep_us(queue_ahead_us(args.steps))
    c0, c1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    c0.record(stream)
    for i in range(args.steps):
        step_cluster(i)
    c1.record(stream)
    torch.cuda.synchronize(device)
    cluster_ms = c0.elapsed_time(c1) / args.steps

    # the same launch alone after an L2 flush (launch latency included)
    single = []
    device_sleep_us(queue_ahead_us(args.steps))
    for i in range(args.steps):
        flush.zero_()
        a, b = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        a.record(stream)
        step(i)
        b.record(stream)
        single.append((a, b))
    torch.cuda.synchronize(device)
    single_ms = sorted(a.elapsed_time(b) for a, b in single)[len(single) // 2]

    # end to end through the public API with host buffers
    q_host = w.query.cpu().pin_memory()
    bt_host = w.block_table.cpu().pin_memory()
    len_host = w.lengths.cpu().pin_memory()
    out_host = torch.empty(out.shape, dtype=out.dtype, pin_memory=True)
    q_dev, bt_dev, len_dev = torch.empty_like(w.query), torch.empty_like(w.block_table), \
        torch.empty_like(w.lengths)

    def e2e_step():
        q_dev.copy_(q_host, non_blocking=True)
        bt_dev.copy_(bt_host, non_blocking=True)
        len_dev.copy_(len_host, non_blocking=True)
        paged_attention(q_dev, w.key_cache, w.value_cache, bt_dev, len_dev,
                        shared_key=w.shared_key, shared_value=w.shared_value, out=out)
        out_host.copy_(out, non_blocking=True)

    for _ in range(args.warmup):
        e2e_step()
    torch.cuda.synchronize(device)
    e2e_starts = [torch.cuda.Event(enable_timing=True) for _ in range(args.steps)]
    e2e_ends = [torch.cuda.Event(enable_timing=True) for _ in range(args.steps)]
    barrier(world, device)
    for i in range(args.steps):
        flush.zero_()
        e2e_starts[i].record(stream)
        e2e_step()
        e2e_ends[i].record(stream)
    torch.cuda.synchronize(device)
    e2e_ms = sum(s.elapsed_time(e) for s, e in zip(e2e_starts, e2e_ends)) / args.steps
    e2e_ms = max_over_ranks(e2e_ms, world, device)
    h2d = q_host.numel() * q_host.element_size() + bt_host.numel() * 4 + len_host.numel() * 4
    d2h = out_host.numel() * out_host.element_size()

    peaks = measured_peaks()
    step_bytes = sum(sets[i % copies].unique_bytes for i in range(args.steps)) / args.steps
    logical = sum(sets[i % copies].logical_bytes for i in range(args.steps)) / args.steps
    achieved = step_bytes / (kernel_ms * 1e-3) / 1e9
    line = {
        "metric": METRIC, "value": world * 1e3 / kernel_ms, "unit": "steps/s",
        "n_gpus": world, "steps": args.steps, "warmup": args.warmup,
        "ms_per_step": kernel_ms, "higher_is_better": True, "scaling": "weak",
        "vs_baseline": None, "dtype": "bf16", "data": "synthetic",
        "config": {"workload": "decode-attention: B=512 beams x 1 query, 8 heads x 32, "
                               "381 shared s0 keys + 64 paged action K/V (page 16), "
                               "prefix-tree block tables (branching 4)",
                   "beams": 512, "tokens": 64, "page_size": 16, "shared_keys": 381,
                   "l2": f"inputs larger than L2: {copies} independent input sets "
                         f"({copies * w.unique_bytes / 1e6:.0f} MB) used in rotation",
                   "timing": "launches back to back, queued ahead of the device",
                   "single_launch_after_l2_flush_ms": single_ms,
                   "cluster_kernel_ms": cluster_ms,
                   "parallelism": f"replicas x{world}"},
        "e2e": {"value": world * 1e3 / e2e_ms, "unit": "steps/s", "h2d_bytes_per_step": h2d,
                "d2h_bytes_per_step": d2h},
        "gpu_launches": launches,
        "roofline": {"bound": "hbm", "achieved": achieved, "peak": peaks["hbm_gbs"],
                     "unit": "GB/s", "frac": achieved / peaks["hbm_gbs"],
                     "traffic": profiled_traffic("decode_attention"),
                     "algorithmic_bytes": step_bytes,
                     "logical_bytes": logical,
                     "logical_gbs": logical / (kernel_ms * 1e-3) / 1e9,
                     "peak_source": f"{peaks['source']} hbm_gbs",
                     "kernel": "decode_group_kernel"},
        "clocks": clocks.summary(),
    }
    if rank == 0 and world == 1 and not args.no_cpu_baseline:
        line["cpu_baseline"] = cpu_decode_attention(w, device)
    return line


def cpu_decode_attention(w, device, *, sample_beams=64, repeats=None, budget_s=12.0):
    """The oracle (CPU restatement of the reference) on a bounded sample."""
    from oracle import paged_attention as oracle

    torch.set_num_threads(os.cpu_count() or 1)
    cache_k = w.key_cache.float().cpu()
    cache_v = w.value_cache.float().cpu()
    sk, sv = w.shared_key.float().cpu(), w.shared_value.float().cpu()
    q = w.query[:sample_beams].float().cpu()
    bt = w.block_table[:sample_beams].cpu()
    ln = w.lengths[:sample_beams].cpu()
    started = time.perf_counter()
    runs = 0
    while True:
        oracle.paged_attention(q, cache_k, cache_v, bt, ln, shared_key=sk, shared_value=sv)
        runs += 1
        elapsed = time.perf_counter() - started
        if (repeats and runs >= repeats) or (not repeats and elapsed > budget_s):
            break
    per_sample = elapsed / runs
    scale = w.query.shape[0] / sample_beams
    return {"value": 1.0 / (per_sample * scale), "unit": "steps/s",
            "cores": torch.get_num_threads(), "kind": "port",
            "sample": f"{sample_beams} of {w.query.shape[0]} beams, {runs} runs, "
                      f"scaled linearly to the full step"}


# ---------------------------------------------------------------------------
# rollout workload
# ---------------------------------------------------------------------------
def build_rollout(device, *, beam_size=1000, depth=64, seed=0, world=1, qubits=6, gates=259):
    """The full rollout workload: random-init rollout model, synthetic rules
    and circuit; `beam_size` beams per GPU (a sharded search over `world`
    GPUs when world > 1)."""
    from graph_rewrite_system_b200 import synthetic
    from graph_rewrite_system_b200.paged_model import PagedActionBindingModel
    from graph_rewrite_system_b200.rollout import DeviceBeamSearch
    from graph_rewrite_system_b200.sharded import ShardedBeamSearch
    from graph_rewrite_system_b200.synthetic import parameter_shapes

    rules = synthetic.synthetic_rules()
    cfg = synthetic.ROLLOUT_MODEL
    model = PagedActionBindingModel(
        rules, num_xfers=rules.num_xfers, width=cfg.width, retrieval_width=cfg.retrieval_width,
        graph_layers=cfg.graph_layers, action_layers=cfg.action_layers,
        action_heads=cfg.action_heads, max_sequence_length=cfg.max_sequence_length,
        readout_graph_layers=cfg.readout_graph_layers, dropout=0.0,
        compute_dtype=torch.bfloat16)
    state = model.state_dict()
    for name, value in synthetic.deterministic_parameters(parameter_shapes(cfg, rules),
                                                          seed).items():
        state[name] = torch.from_numpy(value)
    model.load_state_dict(state)
    model = model.to(device).eval()
    rc = synthetic.RolloutConfig(beam_size=beam_size * world, depth=depth, seed=seed,
                                 num_qubits=qubits, num_gates=gates)
    circuit = synthetic.random_circuit(rc.num_qubits, rc.num_gates, seed)
    if world > 1:
        return ShardedBeamSearch(model, rules, circuit, rc, device), rc
    return DeviceBeamSearch(model, rules, circuit, rc, device), rc


ROLLOUT_DEPTH = 64                      # the metric's T: every rollout search is 64 levels deep


def rollout_window(steps: int, warmup: int) -> tuple[int, int]:
    """(timed levels, first timed level) of the 64-level search: its last
    `steps` levels, after at least `warmup` untimed ones."""
    steps = max(1, min(steps, ROLLOUT_DEPTH - warmup))
    return steps, ROLLOUT_DEPTH - steps + 1


def warm_searches(search, depth: int, count: int = 2) -> None:
    """Untimed full searches until the caching allocator holds every block a
    search needs: the searches after them make no new device allocation."""
    for _ in range(count):
        search.run(depth)           # run() starts from reset()
    torch.cuda.synchronize()


def run_rollout(args, world, rank, device):
    from graph_rewrite_system_b200.rollout import StageTimer

    depth = ROLLOUT_DEPTH
    steps, first = rollout_window(args.steps, args.warmup)
    search, rc = build_rollout(device, beam_size=args.beam, depth=depth, seed=0, world=world,
                               qubits=args.qubits, gates=args.gates)
    stream = torch.cuda.current_stream(device)
    # two full untimed searches first (module load; the caching allocator and
    # NCCL meet every buffer size of the timed levels).  One is not enough:
    # the allocator's free blocks after it are split differently, and a search
    # that follows it still made one new device allocation at level 63, which
    # took 52 ms while the clock sampler's nvidia-smi was querying the driver
    warm_searches(search, depth)
    # the timed search: levels 1 .. first-1 untimed (they include the
    # warm-up), levels first .. 64 timed one by one
    search.reset()
    for _ in range(first - 1):
        if search.step() is None:
            raise RuntimeError(f"the search ended before level {first}")
    torch.cuda.synchronize(device)
    starts = [torch.cuda.Event(enable_timing=True) for _ in range(steps)]
    ends = [torch.cuda.Event(enable_timing=True) for _ in range(steps)]
    barrier(world, device)
    torch.cuda.synchronize(device)
    done = 0
    launches0 = launch_count()
    moved0 = (getattr(search, "moved_children", 0), getattr(search, "moved_bytes", 0))
    probe = KernelProbe("gemm", gemm_work)
    with ClockSampler(device.index) as clocks, probe:
        # every rank's sampler is up (their start-up times differ) before
        # any rank opens the window
        barrier(world, device)
        # NVTX range "timed_levels": lets a profiler restrict itself to the
        # timed window (ncu --nvtx --nvtx-include "timed_levels/")
        torch.cuda.nvtx.range_push("timed_levels")
        for i in range(steps):
            starts[i].record(stream)
            row = search.step()
            ends[i].record(stream)
            done += 1
            if row is None:
                break
        torch.cuda.nvtx.range_pop()
        torch.cuda.synchronize(device)
    launches = launch_count() - launches0
    moved = (getattr(search, "moved_children", 0) - moved0[0],
             getattr(search, "moved_bytes", 0) - moved0[1])
    barrier(world, device)
    step_ms = [s.elapsed_time(e) for s, e in zip(starts[:done], ends[:done])]
    total_ms = max_over_ranks(sum(step_ms), world, device)
    search.check()
    rows = search.rows
    last = rows[-1]
    window = f"{first}..{first + done - 1}"

    # end to end through the public API over the same window: a fresh search
    # (the host circuit uploaded at reset), the levels before the window
    # untimed, then every timed level is step() (with its host read of the
    # level summary) plus the level's children - parent, xfer, source and
    # destination slots, gate count - copied into pinned host memory
    search.reset()
    for _ in range(first - 1):
        search.step()
    torch.cuda.synchronize(device)
    barrier(world, device)
    e2e_start = torch.cuda.Event(enable_timing=True)
    e2e_end = torch.cuda.Event(enable_timing=True)
    d2h_actions = 0
    e2e_done = 0
    with ClockSampler(device.index):      # the same host conditions as the timed window
        search.level_actions_host()        # its pinned host buffers exist before the window
        barrier(world, device)             # all ranks open the window together
        e2e_start.record(stream)
        e2e_level_ms = []                  # host wall time per level (each ends in a host read)
        for _ in range(done):
            t_level = time.perf_counter()
            if search.step() is None:
                break
            d2h_actions += search.level_actions_host()["nbytes"]
            e2e_done += 1
            e2e_level_ms.append(round((time.perf_counter() - t_level) * 1e3, 3))
        e2e_end.record(stream)
        torch.cuda.synchronize(device)
    e2e_ms = max_over_ranks(e2e_start.elapsed_time(e2e_end), world, device)
    search.check()
    # where a level's time goes: CUDA events at the stage boundaries of the
    # same levels in one more search (kept out of the timed window)
    search.reset()
    for _ in range(first - 1):
        search.step()
    timer = StageTimer()
    search.timer = timer
    barrier(world, device)
    for _ in range(done):
        if search.step() is None:
            break
    torch.cuda.synchronize(device)
    timer.collect()
    search.timer = None
    search.check()
    summary_bytes = 12 * 8                 # the per-level summary words step() reads
    # the whole public call: host circuit in, 64 levels, beam summary out
    torch.cuda.synchronize(device)
    barrier(world, device)
    full_start = torch.cuda.Event(enable_timing=True)
    full_end = torch.cuda.Event(enable_timing=True)
    full_start.record(stream)
    search.run(depth)
    if world > 1:
        summary = {"gate_count": search.global_fingerprints()}
    else:
        summary = search.beam_summary()
    full_end.record(stream)
    torch.cuda.synchronize(device)
    full_ms = max_over_ranks(full_start.elapsed_time(full_end), world, device)
    full_h2d = (len(search.circuit.nodes) * 2 + len(search.circuit.edges) * 4) * 8
    stage_ms = {k: v / done for k, v in sorted(timer.totals.items())}
    stage_host_ms = {k: v / done for k, v in sorted(timer.host_totals.items())}
    stage_per_rank = None
    if world > 1:                           # every rank's device stage times
        import torch.distributed as dist

        stage_per_rank = [None] * world
        dist.all_gather_object(stage_per_rank, {k: round(v, 3) for k, v in stage_ms.items()})
    # whole-job throughput: each level advances world x beam beams, i.e.
    # `world * beam / 1000` levels of the B=1000 benchmark
    scale = world * args.beam / 1000
    line = {
        "metric": METRIC, "value": scale * done * 1e3 / total_ms, "unit": "steps/s",
        "n_gpus": world, "steps": done, "warmup": first - 1,
        "ms_per_step": total_ms / done, "higher_is_better": True, "scaling": "weak",
        "vs_baseline": None, "dtype": "bf16", "data": "synthetic",
        "config": {"workload": f"full rollout step: synthetic {args.qubits}-qubit "
                               f"{args.gates}-gate circuit, d_model 256, 8 heads, 4 causal + "
                               f"4 message-passing layers, random init, beam {args.beam} per "
                               f"GPU, depth {depth}, page 16, up to 2048 candidates per state "
                               f"-> 16 per parent -> 16000 proposals; levels {window} of the "
                               f"{depth}-level search timed",
                   "beam": rc.beam_size, "depth": depth, "timed_levels": window,
                   "untimed_levels_before_window": first - 1, "page_size": rc.page_size,
                   "level_ms": [round(x, 3) for x in step_ms],
                   "l2": "inputs larger than L2 (beam state ~0.2 GB bf16 per activation)",
                   "circuit": f"{args.qubits} qubits, {args.gates} gates",
                   "beam_per_gpu": args.beam,
                   "parallelism": (f"sharded beam over {world} GPUs: NCCL all-gather of ranked "
                                   f"records, identical global accept, all-to-all rebalance; "
                                   f"value counts B=1000-equivalent levels")
                                  if world > 1 else "single GPU"},
        "e2e": {"value": scale * e2e_done * 1e3 / e2e_ms, "unit": "steps/s",
                "level_ms": e2e_level_ms,
                "h2d_bytes_per_step": 0,
                "d2h_bytes_per_step": summary_bytes + d2h_actions // max(1, e2e_done),
                "timed_levels": f"{first}..{first + e2e_done - 1}",
                "scope": "DeviceBeamSearch.step() per level plus the level's children copied "
                         "to pinned host memory; the search state stays resident, its only "
                         "host input (the s0 circuit) is uploaded at reset, before the window"},
        "e2e_full_search": {"value": scale * depth * 1e3 / full_ms, "unit": "steps/s",
                            "levels": depth, "h2d_bytes": full_h2d,
                            "scope": "DeviceBeamSearch.run(): s0 circuit upload, all 64 "
                                     "levels, beam summary download"},
        "gpu_launches": launches,
        # traffic: the DRAM / algorithmic byte ratio ncu measured for the
        # store-epilogue GEMM on the update-projection shape (M = 300000),
        # applied to the probed launches' algorithmic bytes
        "roofline": probe.roofline(measured_peaks(),
                                   "tcgen05 store GEMMs (gemm_tc_kernel, gemm_bstat_kernel)",
                                   profiled_traffic("update_gemm_traffic_ratio")),
        "search": {"last_level": {k: getattr(last, k) for k in (
                       "step", "input_states", "output_states", "best_speculative_gate_count",
                       "predicted_actions", "eligible_actions_before_parent_cap",
                       "proposals_after_caps", "attempted_actions", "accepted_actions",
                       "invalid_structural_actions", "duplicate_speculative_successors",
                       "allocated_cache_pages", "logical_cache_pages")},
                   "stage_ms_per_step": stage_ms, "stage_host_ms_per_step": stage_host_ms,
                   "stage_ms_per_step_by_rank": stage_per_rank,
                   "children_changing_gpu_per_level": moved[0] / done,
                   "rebalance_mb_sent_per_level_rank0": moved[1] / done / 1e6},
        "clocks": clocks.summary(),
    }
    if rank == 0 and world == 1 and not args.no_cpu_baseline:
        base = cpu_rollout(done, first - 1, sample_beams=32)
        line["cpu_baseline"] = {k: base[k] for k in ("value", "unit", "cores", "kind", "sample")}
    return line


def run_sharded_config5(args, world, rank, device) -> dict:
    """The sharded-beam workload: synthetic 24-qubit, 2000-gate circuit, the
    same model, 1000 beams per GPU (global beam 1000 x GPUs), depth 64; one
    untimed search, then the last K levels of a second one timed like the
    headline (CUDA events per level, max over ranks)."""
    depth = ROLLOUT_DEPTH
    steps, first = rollout_window(args.steps, args.warmup)
    search, rc = build_rollout(device, beam_size=1000, depth=depth, seed=0, world=world,
                               qubits=24, gates=2000)
    stream = torch.cuda.current_stream(device)
    warm_searches(search, depth)
    search.reset()
    for _ in range(first - 1):
        if search.step() is None:
            raise RuntimeError(f"the search ended before level {first}")
    torch.cuda.synchronize(device)
    barrier(world, device)
    events = [(torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True))
              for _ in range(steps)]
    done = 0
    with ClockSampler(device.index) as clocks:
        barrier(world, device)             # all ranks open the window together
        for a, b in events:
            a.record(stream)
            row = search.step()
            b.record(stream)
            done += 1
            if row is None:
                break
        torch.cuda.synchronize(device)
    search.check()
    total_ms = max_over_ranks(sum(a.elapsed_time(b) for a, b in events[:done]), world, device)
    slots = search.slots
    del search
    torch.cuda.empty_cache()
    return {"workload": "sharded beam: synthetic 24-qubit 2000-gate circuit, same model, beam "
                        f"1000 per GPU ({1000 * world} global), depth {depth}, levels "
                        f"{first}..{first + done - 1} timed",
            "value": world * done * 1e3 / total_ms, "unit": "steps/s (B=1000-equivalent)",
            "ms_per_step": total_ms / done, "timed_levels": f"{first}..{first + done - 1}",
            "beam_per_gpu": 1000, "global_beam": 1000 * world, "slots": slots,
            "clocks": clocks.summary()}


def cpu_rollout(levels: int, warmup: int, sample_beams: int, full_beams: int = 1000):
    """The oracle beam search (the reference's loop restated on the host,
    fp32) on a bounded beam of the 64-level search: `warmup` untimed levels,
    then `levels` timed ones (the GPU arm's window); per-level time scaled
    linearly to full_beams."""
    from graph_rewrite_system_b200 import synthetic
    from oracle.model import OracleModel
    from oracle.rollout import OracleBeamSearch

    torch.set_num_threads(os.cpu_count() or 1)
    rules = synthetic.synthetic_rules()
    cfg = synthetic.ROLLOUT_MODEL
    params = synthetic.deterministic_parameters(synthetic.parameter_shapes(cfg, rules), 0)
    model = OracleModel({k: torch.from_numpy(v) for k, v in params.items()}, rules, cfg)
    rc = synthetic.RolloutConfig(beam_size=sample_beams, depth=ROLLOUT_DEPTH)
    circuit = synthetic.random_circuit(rc.num_qubits, rc.num_gates, 0)
    search = OracleBeamSearch(model, rules, circuit, rc, synthetic.SELECT_ALL_THRESHOLDS)
    search.reset()
    with torch.no_grad():
        for _ in range(warmup):
            search.step()
        started = time.perf_counter()
        done = 0
        for _ in range(levels):
            if search.step() is None:
                break
            done += 1
        elapsed = time.perf_counter() - started
    per_level = elapsed / max(done, 1) * (full_beams / sample_beams)
    return {"value": 1.0 / per_level, "unit": "steps/s", "cores": torch.get_num_threads(),
            "kind": "port",
            "sample": f"oracle beam search, beam {sample_beams} (of {full_beams}), levels "
                      f"{warmup + 1}..{warmup + done} of the {ROLLOUT_DEPTH}-level search "
                      f"(levels 1..{warmup} untimed), per-level time scaled x"
                      f"{full_beams / sample_beams:g}", "levels_timed": done,
            "timed_levels": f"{warmup + 1}..{warmup + done}"}


def run_reference(args, world, rank):
    """--impl reference: the CPU oracle on the same workload (rank 0 only)."""
    if rank != 0:
        return None
    if args.workload in ("update-gemm", "graph-mlp"):
        return {"impl": "reference", "unavailable": f"the {args.workload} microbenchmark has no "
                "CPU arm; the rollout workload's reference arm times the CPU oracle"}
    if args.workload == "cache-churn":
        started = time.perf_counter()
        levels = max(1, min(args.steps, CHURN["depth"] - args.warmup))
        base = cpu_cache_churn(levels)
        value = base["value"]
        return {
            "metric": "paged-cache churn levels/s (1000 beams, fork x5, top 1000, append, release)",
            "impl": "reference", "value": value, "unit": "levels/s", "n_gpus": world,
            "steps": levels, "warmup": CHURN["depth"] - levels, "ms_per_step": 1e3 / value,
            "higher_is_better": True, "scaling": "weak", "vs_baseline": None, "dtype": "bf16",
            "data": "synthetic",
            "config": {"workload": "cache churn (the oracle's sequential PagedKVCache): 1000 "
                                   "beams, 4 layers x 8 heads x 32, page 16, depth 64, 5 children",
                       "timed_levels": f"{CHURN['depth'] - levels + 1}..{CHURN['depth']}"},
            "cpu_baseline": {k: base[k] for k in ("value", "unit", "cores", "kind", "sample")},
            "e2e": {"value": value, "unit": "levels/s", "h2d_bytes_per_step": 0,
                    "d2h_bytes_per_step": 0},
            "wall_seconds": time.perf_counter() - started,
        }
    if args.workload == "rollout":
        started = time.perf_counter()
        steps, first = rollout_window(args.steps, args.warmup)
        base = cpu_rollout(steps, first - 1, sample_beams=64)
        value = base["value"]
        return {
            "metric": METRIC, "impl": "reference", "value": value, "unit": "steps/s",
            "n_gpus": world, "steps": base["levels_timed"], "warmup": first - 1,
            "ms_per_step": 1e3 / value, "higher_is_better": True, "scaling": "weak",
            "vs_baseline": None, "dtype": "f32", "data": "synthetic",
            "config": {"workload": "full rollout step (CPU oracle of the reference loop): "
                                   f"synthetic {args.qubits}-qubit {args.gates}-gate circuit, "
                                   f"depth {ROLLOUT_DEPTH}, levels {base['timed_levels']} timed, "
                                   "bounded beam scaled to beam 1000",
                       "depth": ROLLOUT_DEPTH, "timed_levels": base["timed_levels"],
                       "beam": 1000},
            "cpu_baseline": {k: base[k] for k in ("value", "unit", "cores", "kind", "sample")},
            "e2e": {"value": value, "unit": "steps/s", "h2d_bytes_per_step": 0,
                    "d2h_bytes_per_step": 0},
            "wall_seconds": time.perf_counter() - started,
        }
    device = torch.device("cpu")
    from graph_rewrite_system_b200.workloads import decode_attention_workload

    w = decode_attention_workload(device, seed=0, dtype=torch.float32)
    for _ in range(args.warmup):
        cpu_decode_attention(w, device, repeats=1)
    t0 = time.perf_counter()
    per = []
    for _ in range(args.steps):
        per.append(cpu_decode_attention(w, device, repeats=1)["value"])
    value = statistics.mean(per)
    base = cpu_decode_attention(w, device, repeats=1)
    return {
        "metric": METRIC, "impl": "reference", "value": value, "unit": "steps/s",
        "n_gpus": world, "steps": args.steps, "warmup": args.warmup,
        "ms_per_step": 1e3 / value, "higher_is_better": True, "scaling": "weak",
        "vs_baseline": None, "dtype": "f64", "data": "synthetic",
        "config": {"workload": "decode-attention (CPU oracle, 64-beam sample scaled)"},
        "cpu_baseline": {"value": value, "unit": "steps/s", "cores": base["cores"],
                         "kind": "port", "sample": base["sample"]},
        "e2e": {"value": value, "unit": "steps/s", "h2d_bytes_per_step": 0,
                "d2h_bytes_per_step": 0},
        "wall_seconds": time.perf_counter() - t0,
    }


def run_update_gemm(args, world, rank, device):
    """The readout graph layers' update projection as one tensor-core launch:
    GELU(x [300000, 512] @ u0^T [512 -> 512] + b), bf16 in and out, fp32
    accumulation (tcgen05 GEMM with the fused epilogue).  x rotates between two
    307 MB inputs (larger than L2); the library GEMM + separate bias+GELU pair
    is timed the same way for comparison."""
    from graph_rewrite_system_b200 import kernels as K

    m, k, n = 300000, 512, 512
    gen = torch.Generator(device=device).manual_seed(rank + 7)
    xs = [torch.randn(m, k, device=device, generator=gen).to(torch.bfloat16) for _ in range(2)]
    w = (torch.randn(n, k, device=device, generator=gen) / k ** 0.5).to(torch.bfloat16)
    w_t = w.t().contiguous()
    b = torch.randn(n, device=device, generator=gen)
    out = torch.empty(m, n, device=device, dtype=torch.bfloat16)
    status = torch.zeros(1, device=device, dtype=torch.int32)
    stream = torch.cuda.current_stream(device)
    flops = 2.0 * m * n * k

    def fused(i):
        code = K.gemm_bias_gelu(xs[i % 2], w, b, True, out, status)
        if code:
            raise RuntimeError(f"tensor-core GEMM refused the shape ({code})")

    def library(i):
        torch.mm(xs[i % 2], w_t, out=out)
        K.bias_gelu(out, b)

    def timed(fn, steps):
        for i in range(args.warmup):
            fn(i)
        torch.cuda.synchronize(device)
        barrier(world, device)
        events = [(torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True))
                  for _ in range(steps)]
        device_sleep_us(queue_ahead_us(steps))
        for i, (s0, s1) in enumerate(events):
            s0.record(stream)
            fn(i)
            s1.record(stream)
        torch.cuda.synchronize(device)
        return max_over_ranks(sum(a.elapsed_time(z) for a, z in events), world, device) / steps

    launches0 = launch_count()
    with ClockSampler(device.index) as clocks:
        ms = timed(fused, args.steps)
    launches = launch_count() - launches0
    lib_ms = timed(library, args.steps)
    if int(status.item()):
        raise RuntimeError(f"tensor-core GEMM reported status {int(status.item())}")
    # end to end: x from pinned host memory, one fused launch, the result back
    host_x = xs[0].cpu().pin_memory()
    host_out = torch.empty(m, n, dtype=torch.bfloat16).pin_memory()
    dev_x = torch.empty_like(xs[0])
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    e0.record(stream)
    for _ in range(3):
        dev_x.copy_(host_x, non_blocking=True)
        K.gemm_bias_gelu(dev_x, w, b, True, out, status)
        host_out.copy_(out, non_blocking=True)
    e1.record(stream)
    torch.cuda.synchronize(device)
    e2e_ms = max_over_ranks(e0.elapsed_time(e1) / 3, world, device)
    peaks = measured_peaks()
    achieved = flops / (ms * 1e-3) / 1e12
    traffic_ratio = profiled_traffic("update_gemm_traffic_ratio")
    algorithmic_bytes = 2.0 * (m * k + n * k + m * n) + 4 * n
    return {
        "metric": "update projection GEMM+GELU throughput", "value": world * achieved,
        "unit": "TFLOP/s", "n_gpus": world, "steps": args.steps, "warmup": args.warmup,
        "ms_per_step": ms, "higher_is_better": True, "scaling": "weak", "vs_baseline": None,
        "dtype": "bf16", "data": "synthetic",
        "config": {"workload": "update-gemm: GELU(x[300000,512] @ W[512,512]^T + b), bf16, "
                               "two rotating 307 MB inputs (larger than L2)",
                   "library_gemm_plus_bias_gelu_ms": lib_ms,
                   "speedup_vs_library_pair": lib_ms / ms},
        "e2e": {"value": world * flops / (e2e_ms * 1e-3) / 1e12, "unit": "TFLOP/s",
                "h2d_bytes_per_step": m * k * 2, "d2h_bytes_per_step": m * n * 2},
        "gpu_launches": launches,
        "roofline": {"bound": "tensor", "achieved": achieved, "peak": peaks["bf16_tflops"],
                     "unit": "TFLOP/s", "frac": achieved / peaks["bf16_tflops"],
                     "traffic": traffic_ratio * algorithmic_bytes if traffic_ratio else None,
                     "kernel": "gemm_tc_kernel", "algorithmic_bytes_per_launch": algorithmic_bytes,
                     "hbm_frac": algorithmic_bytes / (ms * 1e-3) / 1e9 / peaks["hbm_gbs"],
                     "peak_source": f"{peaks['source']} bf16_tflops (burst)"},
        "clocks": clocks.summary(),
    }


def run_graph_mlp(args, world, rank, device):
    """One readout graph layer's update as one tensor-core launch:
    LayerNorm(x + GELU([x | agg] U0^T + b0) U2^T + b2) * live over
    M = 300000 rows (beam 1000 x 300 slots), width 256, bf16; the [M, 512]
    GELU activation stays in shared memory.  Two rotating inputs of 307 MB
    (larger than L2).  The same layer as two tensor-core GEMMs with fused
    epilogues (GELU; residual + LayerNorm), which write and re-read the
    activation, is timed beside it."""
    from graph_rewrite_system_b200 import kernels as K

    m = 300000
    gen = torch.Generator(device=device).manual_seed(rank + 11)
    xs = [torch.randn(m, 512, device=device, generator=gen).to(torch.bfloat16) for _ in range(2)]
    u0 = (torch.randn(512, 512, device=device, generator=gen) / 512 ** 0.5).to(torch.bfloat16)
    u2 = (torch.randn(256, 512, device=device, generator=gen) / 512 ** 0.5).to(torch.bfloat16)
    b0 = torch.randn(512, device=device, generator=gen) * 0.1
    b2 = torch.randn(256, device=device, generator=gen) * 0.1
    gamma = 1 + 0.1 * torch.randn(256, device=device, generator=gen)
    beta = 0.1 * torch.randn(256, device=device, generator=gen)
    live = torch.rand(m, device=device, generator=gen) > 0.3
    out = torch.empty(m, 256, device=device, dtype=torch.bfloat16)
    hidden = torch.empty(m, 512, device=device, dtype=torch.bfloat16)
    status = torch.zeros(1, device=device, dtype=torch.int32)
    stream = torch.cuda.current_stream(device)
    flops = 2.0 * m * 512 * (512 + 256)

    def fused(i):
        x = xs[i % 2]
        K.graph_mlp(x, u0, b0, u2, b2, x[:, :256], gamma, beta, zero_row=live, out=out,
                    status=status)

    def two_gemms(i):
        x = xs[i % 2]
        K.gemm(x, u0, b0, gelu=True, out=hidden, status=status)
        K.gemm_layernorm(hidden, u2, b2, x[:, :256], gamma, beta, zero_row=live, out=out,
                         status=status)

    def timed(fn, steps):
        for i in range(args.warmup):
            fn(i)
        torch.cuda.synchronize(device)
        barrier(world, device)
        events = [(torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True))
                  for _ in range(steps)]
        device_sleep_us(queue_ahead_us(steps))
        for i, (s0, s1) in enumerate(events):
            s0.record(stream)
            fn(i)
            s1.record(stream)
        torch.cuda.synchronize(device)
        return max_over_ranks(sum(a.elapsed_time(z) for a, z in events), world, device) / steps

    launches0 = launch_count()
    with ClockSampler(device.index) as clocks:
        ms = timed(fused, args.steps)
    launches = launch_count() - launches0
    two_ms = timed(two_gemms, args.steps)
    if int(status.item()):
        raise RuntimeError(f"tensor-core kernel reported status {int(status.item())}")
    host_x = xs[0].cpu().pin_memory()
    host_out = torch.empty(m, 256, dtype=torch.bfloat16).pin_memory()
    dev_x = torch.empty_like(xs[0])
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    e0.record(stream)
    for _ in range(3):
        dev_x.copy_(host_x, non_blocking=True)
        K.graph_mlp(dev_x, u0, b0, u2, b2, dev_x[:, :256], gamma, beta, zero_row=live,
                    out=out, status=status)
        host_out.copy_(out, non_blocking=True)
    e1.record(stream)
    torch.cuda.synchronize(device)
    e2e_ms = max_over_ranks(e0.elapsed_time(e1) / 3, world, device)
    peaks = measured_peaks()
    achieved = flops / (ms * 1e-3) / 1e12
    traffic_ratio = profiled_traffic("graph_mlp_traffic_ratio")
    algorithmic_bytes = 2.0 * (m * 512 + 512 * 512 + 256 * 512 + m * 256) + m + 4 * 1280
    return {
        "metric": "graph-layer update (GELU MLP + residual + LayerNorm) throughput",
        "value": world * achieved, "unit": "TFLOP/s", "n_gpus": world, "steps": args.steps,
        "warmup": args.warmup, "ms_per_step": ms, "higher_is_better": True, "scaling": "weak",
        "vs_baseline": None, "dtype": "bf16", "data": "synthetic",
        "config": {"workload": "graph-mlp: LayerNorm(x + GELU([x|agg] U0^T + b0) U2^T + b2) * live, "
                               "M = 300000, width 256, bf16, two rotating 307 MB inputs "
                               "(larger than L2)",
                   "two_tensor_core_gemms_ms": two_ms, "speedup_vs_two_gemms": two_ms / ms},
        "e2e": {"value": world * flops / (e2e_ms * 1e-3) / 1e12, "unit": "TFLOP/s",
                "h2d_bytes_per_step": m * 512 * 2, "d2h_bytes_per_step": m * 256 * 2},
        "gpu_launches": launches,
        "roofline": {"bound": "tensor", "achieved": achieved, "peak": peaks["bf16_tflops"],
                     "unit": "TFLOP/s", "frac": achieved / peaks["bf16_tflops"],
                     "traffic": traffic_ratio * algorithmic_bytes if traffic_ratio else None,
                     "kernel": "graph_mlp_kernel", "algorithmic_bytes_per_launch": algorithmic_bytes,
                     "hbm_frac": algorithmic_bytes / (ms * 1e-3) / 1e9 / peaks["hbm_gbs"],
                     "peak_source": f"{peaks['source']} bf16_tflops (burst)"},
        "clocks": clocks.summary(),
    }


# cache-churn workload: 1000 live beams, 4 causal layers x 8 heads x 32 bf16
# K/V per action, page 16, depth 64, 5 children per beam
CHURN = dict(beams=1000, children=5, depth=64, layers=4, heads=8, head_width=32, width=256,
             page=16)


def churn_token_bytes(c=CHURN) -> int:
    """Bytes of one token row across every arena: K and V of each layer, the
    action state, the readout K and V (bf16)."""
    hd = c["heads"] * c["head_width"]
    return 2 * (2 * c["layers"] * hd + c["width"] + 2 * hd)


def churn_plan(seed: int, c=CHURN) -> list[torch.Tensor]:
    """Per level, the surviving children's parent rows: every beam forks into
    `children`, each child draws a seeded uniform score, the top `beams`
    (stable sort, ties by index) survive."""
    gen = torch.Generator().manual_seed(seed)
    plan, n = [], 1
    for _ in range(c["depth"]):
        scores = torch.rand(n * c["children"], generator=gen)
        parents = torch.sort(scores, descending=True, stable=True).indices[:c["beams"]]
        plan.append(parents // c["children"])
        n = plan[-1].numel()
    return plan


def churn_level_bytes(parent_lengths: list[int], parent_cols: int, n_prev: int,
                      c=CHURN) -> int:
    """Algorithmic HBM bytes of one churn level: every child writes its new
    token row; a child whose parent ends in a partial page copies that page's
    `length % page` rows to its own page (read + write); the parent block-table
    rows and lengths are read and the child rows written; the released rows
    are read once."""
    token = churn_token_bytes(c)
    rows = sum(1 + 2 * (length % c["page"]) for length in parent_lengths)
    n = len(parent_lengths)
    tables = 4 * (n * (parent_cols + 1) + n * (parent_cols + 2) + n_prev * (parent_cols + 1))
    return token * rows + tables


def cpu_cache_churn(levels: int, seed: int = 0) -> dict:
    """The oracle's PagedKVCache (the reference's sequential append/release
    loop restated) over the same churn: all 64 levels run, the last `levels`
    timed."""
    from oracle.paged_cache import OraclePagedKVCache

    c = CHURN
    cap = c["beams"] * (-(-c["depth"] // c["page"]) + 3)
    ref = OraclePagedKVCache(layers=c["layers"], capacity=cap, page_size=c["page"],
                             heads=c["heads"], head_width=c["head_width"],
                             model_width=c["width"], dtype=torch.bfloat16)
    gen = torch.Generator().manual_seed(seed + 1)
    handles = [ref.empty_handle()]
    first = c["depth"] - levels
    seconds = 0.0
    for level, parents in enumerate(churn_plan(seed)):
        n = parents.numel()
        kv = torch.randn(c["layers"], n, c["heads"], c["head_width"], generator=gen).bfloat16()
        act = torch.randn(n, c["width"], generator=gen).bfloat16()
        rk = torch.randn(n, c["heads"], c["head_width"], generator=gen).bfloat16()
        t0 = time.perf_counter()
        new = ref.append_batch([handles[p] for p in parents.tolist()], kv, kv, act, rk, rk)
        for h in handles:
            ref.release(h)
        handles = new
        if level >= first:
            seconds += time.perf_counter() - t0
    return {"value": levels / seconds, "unit": "levels/s", "cores": torch.get_num_threads(),
            "kind": "port", "sample": f"the oracle cache (sequential per-handle loop) over the "
                                      f"whole 64-level churn at 1000 beams, levels "
                                      f"{first + 1}..{c['depth']} timed, unscaled"}


def run_cache_churn(args, world, rank, device):
    """The paged-cache churn workload (1000 live beams, 4 layers x 8 heads x
    32 bf16 K/V per action, page 16, depth 64, 5 children per beam with
    seeded uniform scores, the top 1000 kept).  A step is one level on the
    device: the survivors' parent block-table rows are gathered, one token is
    appended to each (grs_cache_append: fork with copy-on-write of partial
    tail pages, then the token rows in every arena) and the previous level's
    rows are released (grs_cache_release: refcount reclaim in release order).
    The survivor choice (the search's ranking, not the cache's work) and the
    token contents are drawn before timing.  All 64 levels run; the last
    `steps` are timed, each after an L2 flush."""
    from graph_rewrite_system_b200 import kernels as K
    from graph_rewrite_system_b200.paged_cache import PagedKVCache

    c = CHURN
    levels = max(1, min(args.steps, c["depth"] - args.warmup))
    first = c["depth"] - levels
    cap = c["beams"] * (-(-c["depth"] // c["page"]) + 3)
    cache = PagedKVCache(layers=c["layers"], capacity=cap, page_size=c["page"],
                         heads=c["heads"], head_width=c["head_width"], model_width=c["width"],
                         device=device, dtype=torch.bfloat16)
    plan = [p.to(device) for p in churn_plan(rank)]
    gen = torch.Generator(device=device).manual_seed(rank + 1)
    hd = (c["heads"], c["head_width"])
    tokens = []
    for p in plan:
        n = p.numel()
        tokens.append(tuple(torch.randn(shape, device=device, generator=gen).bfloat16() for shape in
                            ((c["layers"], n) + hd, (c["layers"], n) + hd, (n, c["width"]),
                             (n,) + hd, (n,) + hd)))
    flush = torch.empty(L2_FLUSH_BYTES, dtype=torch.uint8, device=device)
    stream = torch.cuda.current_stream(device)

    def level(state, i, index=None):
        # every child of level i holds i + 1 tokens: its table row is exactly
        # ceil((i + 1) / page) pages wide
        table, lengths = state
        index = plan[i] if index is None else index
        n = index.numel()
        pt = torch.empty(n, table.shape[1], dtype=torch.int32, device=device)
        pl = torch.empty(n, dtype=torch.int32, device=device)
        K.gather_beams(table, index, pt)
        K.gather_beams(lengths, index, pl)
        ct, cl = cache.append_device(pt, pl, *tokens[i], child_cols=-(-(i + 1) // c["page"]))
        cache.release_device(table, lengths)
        return ct, cl

    def start():
        cache.reset()
        return (torch.zeros(1, 1, dtype=torch.int32, device=device),
                torch.zeros(1, dtype=torch.int32, device=device))

    # untimed pass: warm-up, and the algorithmic bytes of every timed level
    state = start()
    level_bytes = []
    for i in range(c["depth"]):
        if i >= first:
            lengths = state[1].index_select(0, plan[i]).tolist()
            level_bytes.append(churn_level_bytes(lengths, state[0].shape[1], state[1].numel()))
        state = level(state, i)
    cache.check_status()
    # timed pass
    state = start()
    for i in range(first):
        state = level(state, i)
    torch.cuda.synchronize(device)
    barrier(world, device)
    events = [(torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True))
              for _ in range(levels)]
    launches0 = launch_count()
    with ClockSampler(device.index) as clocks:
        for j, i in enumerate(range(first, c["depth"])):
            flush.fill_(j & 0xFF)
            events[j][0].record(stream)
            state = level(state, i)
            events[j][1].record(stream)
        torch.cuda.synchronize(device)
    launches = launch_count() - launches0
    cache.check_status()
    level_ms = [a.elapsed_time(b) for a, b in events]
    ms = max_over_ranks(sum(level_ms), world, device) / levels
    avg_bytes = sum(level_bytes) / levels
    # end to end: each level's token rows and survivor indices copied in from
    # pinned host memory, the child lengths and the status word read back
    host_tokens = [tuple(t.cpu().pin_memory() for t in tokens[i]) for i in range(first, c["depth"])]
    host_plan = [plan[i].cpu().pin_memory() for i in range(first, c["depth"])]
    host_lengths = torch.empty(c["beams"], dtype=torch.int32).pin_memory()
    host_status = torch.empty(1, dtype=torch.int32).pin_memory()
    dev_tokens = [torch.empty(t.shape, dtype=t.dtype, device=device) for t in host_tokens[0]]
    dev_plan = torch.empty(c["beams"], dtype=torch.int64, device=device)
    state = start()
    for i in range(first):
        state = level(state, i)
    torch.cuda.synchronize(device)
    barrier(world, device)
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    h2d = d2h = 0
    e0.record(stream)
    for j in range(levels):
        for dst, src in zip(dev_tokens, host_tokens[j]):
            dst.copy_(src, non_blocking=True)
            h2d += src.numel() * src.element_size()
        n = host_plan[j].numel()
        dev_plan[:n].copy_(host_plan[j], non_blocking=True)
        h2d += 8 * n
        i = first + j
        tokens_i, tokens[i] = tokens[i], tuple(dev_tokens)
        state = level(state, i, dev_plan[:n])
        tokens[i] = tokens_i
        ct, cl = state
        host_lengths[:n].copy_(cl, non_blocking=True)
        host_status.copy_(cache.status_tensor(), non_blocking=True)
        d2h += 4 * n + 4
        stream.synchronize()
        if int(host_status[0]):
            raise RuntimeError(f"cache kernel reported status {int(host_status[0])}")
    e1.record(stream)
    torch.cuda.synchronize(device)
    e2e_ms = max_over_ranks(e0.elapsed_time(e1), world, device) / levels
    peaks = measured_peaks()
    achieved = avg_bytes / (ms * 1e-3) / 1e9
    line = {
        "metric": "paged-cache churn levels/s (1000 beams, fork x5, top 1000, append, release)",
        "value": world * 1e3 / ms, "unit": "levels/s", "n_gpus": world, "steps": levels,
        "warmup": first, "ms_per_step": ms, "higher_is_better": True, "scaling": "weak",
        "vs_baseline": None, "dtype": "bf16", "data": "synthetic",
        "config": {"workload": "cache churn: 1000 live beams, 4 causal layers x 8 heads x 32 bf16 "
                               "K/V per action (+ action state, readout K/V), page 16, depth 64, "
                               "each level forks every beam into 5 children with seeded uniform "
                               "scores and keeps the top 1000; levels "
                               f"{first + 1}..{c['depth']} timed",
                   "timed_levels": f"{first + 1}..{c['depth']}", "beams_per_gpu": c["beams"],
                   "l2": "L2 flushed (256 MB write) before every timed level",
                   "parallelism": f"replicas x{world}" if world > 1 else "single GPU"},
        "e2e": {"value": world * 1e3 / e2e_ms, "unit": "levels/s",
                "h2d_bytes_per_step": h2d // levels, "d2h_bytes_per_step": d2h // levels,
                "scope": "PagedKVCache.append_device / release_device per level with the token "
                         "rows and survivor indices copied from pinned host memory and the "
                         "child lengths and status read back"},
        "gpu_launches": launches,
        "roofline": {"bound": "hbm", "achieved": achieved, "peak": peaks["hbm_gbs"],
                     "unit": "GB/s", "frac": achieved / peaks["hbm_gbs"],
                     "traffic": None, "kernel": "one churn level (append + release)",
                     "algorithmic_bytes_per_level": avg_bytes,
                     "level_ms": [round(x, 4) for x in level_ms],
                     "peak_source": f"{peaks['source']} hbm_gbs"},
        "clocks": clocks.summary(),
    }
    if rank == 0 and not args.no_cpu_baseline:
        line["cpu_baseline"] = cpu_cache_churn(levels)
    return line


def main() -> None:
    parser = argparse.ArgumentParser()
    parser.add_argument("--gpus", type=int, default=1)
    parser.add_argument("--steps", type=int, default=60)
    parser.add_argument("--warmup", type=int, default=4)
    parser.add_argument("--impl", choices=("b200", "reference"), default="b200")
    parser.add_argument("--workload", choices=("rollout", "decode-attention", "update-gemm",
                                               "graph-mlp", "cache-churn"), default="rollout")
    parser.add_argument("--no-cpu-baseline", action="store_true")
    parser.add_argument("--beam", type=int, default=1000,
                        help="rollout beam size (1000 is the benchmark configuration)")
    parser.add_argument("--no-attention", action="store_true",
                        help="rollout only: skip the paged-attention sub-benchmark")
    parser.add_argument("--no-config5", action="store_true",
                        help="rollout only: skip the sharded-beam (24-qubit, 2000-gate) block")
    parser.add_argument("--qubits", type=int, default=6,
                        help="rollout circuit qubits (24 with --gates 2000: the sharded config)")
    parser.add_argument("--gates", type=int, default=259, help="rollout circuit gates")
    args = parser.parse_args()
    if args.warmup < 3:
        args.warmup = 3
    world = int(os.environ.get("WORLD_SIZE", "1"))
    rank = int(os.environ.get("RANK", "0"))
    if args.impl == "reference":
        line = run_reference(args, world, rank)
        if line is not None:
            print(json.dumps(line), flush=True)
        return
    world, rank, local = dist_setup(args.gpus)
    device = torch.device("cuda", local)
    torch.cuda.set_device(device)
    sleep_cycles_per_us()            # calibrate the device sleep before any timed region
    # no cyclic-garbage collection pauses inside the measured levels (the
    # reference's benchmark loop disables the collector the same way,
    # paged_rollout_benchmark.py:886-887); reference counting still frees
    gc.collect()
    gc.disable()
    if args.workload == "rollout":
        line = run_rollout(args, world, rank, device)
        if not args.no_config5 and (args.qubits, args.gates) != (24, 2000):
            torch.cuda.empty_cache()
            line["sharded_config5"] = run_sharded_config5(args, world, rank, device)
        if not args.no_attention:
            attn_args = argparse.Namespace(steps=20, warmup=5, no_cpu_baseline=True)
            attention = run_decode_attention(attn_args, world, rank, device)
            line["paged_attention"] = {k: attention[k] for k in (
                "value", "unit", "ms_per_step", "roofline", "config")}
    elif args.workload == "update-gemm":
        line = run_update_gemm(args, world, rank, device)
    elif args.workload == "graph-mlp":
        line = run_graph_mlp(args, world, rank, device)
    elif args.workload == "cache-churn":
        line = run_cache_churn(args, world, rank, device)
    else:
        line = run_decode_attention(args, world, rank, device)
    if rank == 0:
        print(json.dumps(line), flush=True)
    if world > 1:
        import torch.distributed as dist

        dist.destroy_process_group()


if __name__ == "__main__":
    main()

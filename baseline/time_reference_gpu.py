"""Time the reference's own GPU search loop on this machine.

The reference's path for one search level, driven through its own stage
functions exactly as its benchmark loop composes them
(paged_rollout_benchmark.py:898-1093): ``paged_model_matches`` with
tensorized state batches and GPU proposals (paged_rollout_benchmark.py:243-388,
its paged readout on the Triton kernel of paged_attention.py),
``gpu_proposals.build_gpu_proposals`` with the effective per-parent cap, the
``lazy_rollout_benchmark.lazy_child`` accept loop (indexed topology, raw
dedup), the gate-count sort and ``advance_selected`` over the reference's
``PagedKVCache`` (paged_rollout_benchmark.py:390-556), on CUDA under the
reference's bf16 autocast (train.py:28-31) with a bf16 arena.

Workload: the rollout workload of ``bench.py`` (synthetic 6-qubit 259-gate
circuit, synthetic rule set, the rollout model at width 256 / 8 heads / 4
causal + 4 readout graph layers with the same seeded random weights, beam
1000, depth 64, page 16, the same candidate and proposal caps).  The
reference checkout has no trained checkpoint, calibration, ECC file or QASM
input here, so the Quartz-dependent parts of its entry script (QASM parsing,
exact refresh, audits) are not run; the stage loop above is the part the
B200 path replaces.

Each level is timed on the wall clock with a device synchronize at its end
(much of the reference's level is host Python).  Prints one JSON line.

The reference is imported from ``baseline/_ref`` (a ``pip install --target``
of the reference checkout; see the design notes), or from ``--reference``.
"""
from __future__ import annotations

import argparse
import json
import math
import os
import statistics
import sys
import time
from collections import defaultdict
from pathlib import Path

HERE = Path(__file__).resolve().parent
ROOT = HERE.parent
sys.path.insert(0, str(ROOT))

import torch  # noqa: E402


def main() -> None:
    parser = argparse.ArgumentParser()
    parser.add_argument("--reference", type=Path, default=HERE / "_ref")
    parser.add_argument("--device", default="cuda")
    parser.add_argument("--beam", type=int, default=1000)
    parser.add_argument("--depth", type=int, default=64)
    parser.add_argument("--timed", type=int, default=20, help="levels timed at the end")
    parser.add_argument("--small", action="store_true",
                        help="a tiny model and circuit (a quick check of the driver)")
    parser.add_argument("--budget-s", type=float, default=300.0,
                        help="stop after this much wall time and report the levels done")
    args = parser.parse_args()
    if not (args.reference / "paged_rollout_benchmark.py").exists():
        print(json.dumps({"impl": "reference-gpu",
                          "unavailable": f"reference modules not found under {args.reference}"}))
        return
    sys.path.insert(0, str(args.reference))

    import beam_search_benchmark as bsb
    import dataset as ref_dataset
    import gpu_proposals as gp
    import incremental_graph as ig
    import lazy_rollout_benchmark as lrb
    import paged_cache as ref_cache
    import paged_model as ref_model
    import paged_rollout_benchmark as prb
    from train import autocast_context, move_batch
    from graph_rewrite_system_b200 import synthetic

    device = torch.device(args.device)
    if args.small:
        cfg = synthetic.ModelConfig(width=32, retrieval_width=16, graph_layers=1,
                                    action_layers=2, action_heads=2, max_sequence_length=16,
                                    readout_graph_layers=1)
        rc = synthetic.RolloutConfig(beam_size=args.beam, depth=args.depth, num_qubits=4,
                                     num_gates=30, max_candidates_per_state=400,
                                     per_parent_cap=4, proposal_factor=4, page_size=4)
    else:
        cfg = synthetic.ROLLOUT_MODEL
        rc = synthetic.RolloutConfig(beam_size=args.beam, depth=args.depth)
    rules = synthetic.synthetic_rules()
    ref_rules = ref_dataset.RuleMetadata.from_payload({
        "source_patterns": list(rules.source_patterns),
        "xfer_to_source": list(rules.xfer_to_source),
        "xfer_sources": list(rules.xfer_sources),
        "xfer_destinations": list(rules.xfer_destinations)})
    model = ref_model.PagedActionBindingModel(
        ref_rules, num_xfers=rules.num_xfers, width=cfg.width,
        retrieval_width=cfg.retrieval_width, graph_layers=cfg.graph_layers,
        action_layers=cfg.action_layers, action_heads=cfg.action_heads,
        max_sequence_length=cfg.max_sequence_length,
        readout_graph_layers=cfg.readout_graph_layers, readout_attention_backend="paged",
        dropout=0.0)
    state = model.state_dict()
    for name, value in synthetic.deterministic_parameters(
            synthetic.parameter_shapes(cfg, rules), rc.seed).items():
        state[name] = torch.from_numpy(value)
    model.load_state_dict(state)
    model = model.to(device).eval()

    source_to_xfers = defaultdict(list)
    for xfer, source in enumerate(ref_rules.xfer_to_source):
        source_to_xfers[source].append(xfer)
    gate_deltas = [len(ref_rules.destination_gate_types[x])
                   - len(ref_rules.source_gate_types[ref_rules.xfer_to_source[x]])
                   for x in range(len(ref_rules.xfer_to_source))]
    rule_index = gp.GpuRuleIndex.build(source_to_xfers, gate_deltas,
                                       len(ref_rules.source_gate_types), rc.max_gate_increase,
                                       device)
    src_pat = tuple(ig.parse_pattern(p) for p in ref_rules.xfer_sources)
    dst_pat = tuple(ig.parse_pattern(p) for p in ref_rules.xfer_destinations)

    circuit = synthetic.random_circuit(rc.num_qubits, rc.num_gates, rc.seed)
    snapshot = circuit.snapshot()
    beam = [bsb.BeamState(graph=None, snapshot=snapshot, guid_to_slot={},
                          next_slot=rc.num_gates, last_touched={},
                          rewrite_distance={n[0]: 5 for n in snapshot["nodes"]},
                          previous_preferred=set(), local_streak=0, gate_count=rc.num_gates,
                          depth=0, history=(), topology_index=lrb.indexed_topology(snapshot))]
    with torch.no_grad(), autocast_context(device):
        slot_states, live, gate_types = model.initialize_incremental(
            move_batch(prb.initial_batch(snapshot), device))
        source_vectors = model.retrieval_source(model.source_representations())
    arena = ref_cache.PagedKVCache(
        layers=cfg.action_layers, capacity=rc.cache_pages, page_size=rc.page_size,
        heads=cfg.action_heads, head_width=cfg.width // cfg.action_heads,
        model_width=cfg.width, device=device,
        dtype=torch.bfloat16 if device.type == "cuda" else slot_states.dtype)
    handles = [arena.empty_handle()]
    seen = {lrb.raw_topology_hash(snapshot)}

    level_s, accepted_per_level = [], []
    started = time.perf_counter()
    for step in range(rc.depth):
        t0 = time.perf_counter()
        with torch.no_grad():
            candidates, _, _ = prb.paged_model_matches(
                beam, slot_states, live, gate_types, handles, arena, model, device,
                synthetic.SELECT_ALL_THRESHOLDS, source_vectors, rc.microbatch,
                rc.max_candidates_per_state, "tensorized", "gpu")
        cap = max(rc.per_parent_cap, math.ceil(rc.beam_size / max(1, len(beam))) * 2)
        proposals, _, _ = gp.build_gpu_proposals(candidates, beam, rule_index,
                                                 per_parent_cap=cap, global_cap=rc.global_cap)
        records = []
        for proposal in proposals:
            if len(records) >= rc.beam_size:
                break
            child, fingerprint, is_dup = lrb.lazy_child(beam[proposal.parent], proposal,
                                                        src_pat, dst_pat, False, "raw", seen,
                                                        "indexed")
            if is_dup or child is None:
                continue
            seen.add(fingerprint)
            records.append((child, proposal))
        if not records:
            break
        records.sort(key=lambda row: (row[0].gate_count, len(row[0].history)))
        records = records[:rc.beam_size]
        with torch.no_grad():
            slot_states, live, gate_types, handles, _, _ = prb.advance_selected(
                slot_states, live, gate_types, handles, records, ref_rules, arena, model,
                device, rc.microbatch)
        beam = [r[0] for r in records]
        if device.type == "cuda":
            torch.cuda.synchronize(device)
        level_s.append(time.perf_counter() - t0)
        accepted_per_level.append(len(records))
        if time.perf_counter() - started > args.budget_s:
            break

    done = len(level_s)
    first = max(0, rc.depth - args.timed) if done == rc.depth else max(0, done - args.timed)
    window = level_s[first:]
    value = len(window) / sum(window) if window else None
    line = {
        "impl": "reference-gpu",
        "metric": "beam-state decode steps/s at B=1000,T=64",
        "value": value, "unit": "steps/s",
        "timed_levels": f"{first + 1}..{done}", "levels_done": done, "depth": rc.depth,
        "median_level_s": statistics.median(window) if window else None,
        "level_s": [round(x, 4) for x in level_s],
        "accepted_per_level": accepted_per_level,
        "whole_search_s": sum(level_s),
        "device": torch.cuda.get_device_name(device) if device.type == "cuda" else "cpu",
        "host_cores": len(os.sched_getaffinity(0)),
        "config": {"workload": "reference stage loop (paged_model_matches, build_gpu_proposals, "
                               "lazy_child accept, gate-count sort, advance_selected), "
                               f"beam {rc.beam_size}, depth {rc.depth}, page {rc.page_size}, "
                               f"{rc.num_qubits}-qubit {rc.num_gates}-gate synthetic circuit, "
                               f"model width {cfg.width}, bf16 autocast"},
    }
    print(json.dumps(line))


if __name__ == "__main__":
    main()

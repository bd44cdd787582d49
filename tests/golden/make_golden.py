"""Generate the golden fixtures of tests/golden from the reference's own code.

Run where a checkout of the reference repository is available:

    python tests/golden/make_golden.py --reference <path to the reference checkout>

Each fixture stores seeded inputs and the outputs the reference's Python
implementation produced for them (CPU, fp32).  The tests pin the CPU oracle
against these files and compare the CUDA path with the oracle; nothing at
test time reads the reference.
"""
from __future__ import annotations

import argparse
import math
from pathlib import Path
import sys

import numpy as np
import torch

HERE = Path(__file__).resolve().parent
ROOT = HERE.parents[1]
sys.path.insert(0, str(ROOT))


def paged_attention_case(ref, with_current: bool):
    """The reference's own test case (test_paged_attention.py:8-60), fp32."""
    torch.manual_seed(7)
    b, cap, page, heads, hw, q = 5, 12, 8, 6, 32, 37
    keys = torch.randn(cap, page, heads, hw)
    values = torch.randn_like(keys)
    table = torch.tensor([[0, 6, 9], [1, 6, 8], [2, 7, 9], [0, 6, 8], [3, 4, 5]], dtype=torch.int32)
    lengths = torch.tensor([0, 3, 8, 9, 19], dtype=torch.int32)
    query = torch.randn(b, heads, q, hw)
    kwargs = {}
    if with_current:
        kwargs = dict(current_key=torch.randn(b, heads, hw), current_value=torch.randn(b, heads, hw),
                      current_valid=torch.tensor([True, True, False, True, True]))
    out = ref.paged_attention_reference(query, keys, values, table, lengths, **kwargs)
    arrays = dict(query=query, keys=keys, values=values, block_table=table, lengths=lengths,
                  output=out, **kwargs)
    return {k: v.numpy() for k, v in arrays.items()}


def cache_churn_case(paged_cache, *, seed: int, beams: int, depth: int, children: int,
                     page: int, layers: int = 2, heads: int = 2, hw: int = 4, width: int = 8):
    """Fork/COW/reclaim churn on the reference PagedKVCache (config-3 semantics:
    each step forks every beam into `children`, keeps the top `beams` by seeded
    uniform scores (stable, ties by index), appends one token per survivor and
    releases the old handles)."""
    g = torch.Generator().manual_seed(seed)
    capacity = beams * (math.ceil(depth / page) + 3)
    arena = paged_cache.PagedKVCache(layers=layers, capacity=capacity, page_size=page,
                                     heads=heads, head_width=hw, model_width=width,
                                     device=torch.device("cpu"), dtype=torch.float32)
    handles = [arena.empty_handle()]
    rec = {"capacity": np.int64(capacity), "page": np.int64(page), "layers": np.int64(layers),
           "heads": np.int64(heads), "hw": np.int64(hw), "width": np.int64(width)}
    for step in range(depth):
        scores = torch.rand(len(handles) * children, generator=g)
        order = torch.sort(scores, descending=True, stable=True).indices[:beams]
        parents = (order // children).tolist()
        n = len(parents)
        kv = torch.randn(layers, n, heads, hw, generator=g)
        vv = torch.randn(layers, n, heads, hw, generator=g)
        act = torch.randn(n, width, generator=g)
        rk = torch.randn(n, heads, hw, generator=g)
        rv = torch.randn(n, heads, hw, generator=g)
        new = arena.append_batch([handles[p] for p in parents], kv, vv, act, rk, rv)
        for h in handles:
            arena.release(h)
        handles = new
        cols = max(len(h.blocks) for h in handles)
        table = np.zeros((n, cols), np.int32)
        for i, h in enumerate(handles):
            table[i, : len(h.blocks)] = h.blocks
        rec[f"s{step}_parents"] = np.asarray(parents, np.int64)
        rec[f"s{step}_keys"] = kv.numpy(); rec[f"s{step}_values"] = vv.numpy()
        rec[f"s{step}_actions"] = act.numpy()
        rec[f"s{step}_rkeys"] = rk.numpy(); rec[f"s{step}_rvalues"] = rv.numpy()
        rec[f"s{step}_table"] = table
        rec[f"s{step}_lengths"] = np.asarray([h.length for h in handles], np.int32)
        rec[f"s{step}_refcounts"] = np.asarray(arena.refcounts, np.int32)
        rec[f"s{step}_free"] = np.asarray(arena.free, np.int32)
        # arena rows of every live handle token (valid positions only)
        _, values_g, actions_g, mask = arena.gather(handles)
        rec[f"s{step}_gather_values"] = values_g.numpy()
        rec[f"s{step}_gather_actions"] = actions_g.numpy()
    for h in handles:
        arena.release(h)
    rec["final_allocated"] = np.int64(arena.allocated_pages)
    rec["depth"] = np.int64(depth)
    return rec


def proposals_cases(gp, bsb, prb, ti):
    out = {}
    # 1. The reference test's hand-built case (test_gpu_proposals.py:27-91).
    beam = [bsb.BeamState(None, {"nodes": [], "edges": []}, {}, 0, {}, {}, set(), 0, g, 1, ())
            for g in (20, 18, 21)]
    s2x = {0: [0, 1], 1: [2], 2: [3, 4]}
    deltas = [0, -1, 1, 2, -2]
    rows = [[(0, 2, (2, 3), 0.7), (1, 4, (4,), 0.9)],
            [(2, 1, (1, 5), 0.8), (0, 3, (3, 7), 0.6)],
            [(1, 6, (6,), 0.95), (2, 8, (8,), 0.5)]]
    flat = [(b, s, a, bind, p) for b, r in enumerate(rows) for s, a, bind, p in r]
    bind = torch.full((len(flat), 2), -1, dtype=torch.long)
    for i, r in enumerate(flat):
        bind[i, : len(r[3])] = torch.tensor(r[3])
    cand = ti.CandidateTensors(torch.tensor([r[0] for r in flat]), torch.tensor([r[1] for r in flat]),
                               torch.tensor([r[2] for r in flat]), bind,
                               torch.tensor([r[4] for r in flat]))
    index = gp.GpuRuleIndex.build(s2x, deltas, 3, 1, torch.device("cpu"))
    props, metrics, _ = gp.build_gpu_proposals(cand, beam, index, per_parent_cap=2, global_cap=4)
    legacy, _ = prb.build_legacy_proposals(beam, rows, None, s2x, deltas, beam_size=2,
                                           max_actions_per_parent=2, exploration_actions_per_parent=0,
                                           proposal_factor=2, max_gate_increase=1)
    assert [(p.parent, p.xfer_id, p.anchor_slot, p.binding) for p in props] == \
        [(p.parent, p.xfer_id, p.anchor_slot, p.binding) for p in legacy]
    out["small"] = _pack_proposals(cand, [b.gate_count for b in beam], s2x, deltas, 3, 1, 2, 4,
                                   props, metrics)
    # 2. Seeded random case with ties in probability and gate counts.
    g = torch.Generator().manual_seed(11)
    num_parents, per, num_sources, num_xfers = 40, 30, 9, 17
    x2s = torch.randint(0, num_sources, (num_xfers,), generator=g).tolist()
    s2x = {}
    for x, s in enumerate(x2s):
        s2x.setdefault(s, []).append(x)
    deltas = torch.randint(-2, 3, (num_xfers,), generator=g).tolist()
    gates = torch.randint(50, 56, (num_parents,), generator=g).tolist()
    n = num_parents * per
    batch = torch.arange(num_parents).repeat_interleave(per)
    perm = torch.randperm(n, generator=g)
    batch = batch[perm]
    sources = torch.randint(0, num_sources, (n,), generator=g)
    anchors = torch.randint(0, 100, (n,), generator=g)
    bind = torch.randint(-1, 100, (n, 3), generator=g)
    probs = (torch.randint(0, 12, (n,), generator=g).float() / 16.0).sigmoid()  # many ties
    cand = ti.CandidateTensors(batch, sources, anchors, bind, probs)
    beam = [bsb.BeamState(None, {"nodes": [], "edges": []}, {}, 0, {}, {}, set(), 0, gg, 1, ())
            for gg in gates]
    index = gp.GpuRuleIndex.build(s2x, deltas, num_sources, 1, torch.device("cpu"))
    props, metrics, _ = gp.build_gpu_proposals(cand, beam, index, per_parent_cap=5, global_cap=120)
    out["random"] = _pack_proposals(cand, gates, s2x, deltas, num_sources, 1, 5, 120, props, metrics)
    return out


def _pack_proposals(cand, gates, s2x, deltas, num_sources, max_inc, cap, gcap, props, metrics):
    xfer_src = np.full(len(deltas), -1, np.int64)
    for s, xs in s2x.items():
        for x in xs:
            xfer_src[x] = s
    width = cand.bindings.shape[1]
    bind = np.full((len(props), width), -1, np.int64)
    for i, p in enumerate(props):
        bind[i, : len(p.binding)] = p.binding
    return dict(
        batch_ids=cand.batch_ids.numpy(), sources=cand.sources.numpy(), anchors=cand.anchors.numpy(),
        bindings=cand.bindings.numpy(), probabilities=cand.probabilities.numpy().astype(np.float32),
        parent_gates=np.asarray(gates, np.int64), xfer_to_source=xfer_src,
        gate_deltas=np.asarray(deltas, np.int64), num_sources=np.int64(num_sources),
        max_gate_increase=np.int64(max_inc), per_parent_cap=np.int64(cap), global_cap=np.int64(gcap),
        out_parent=np.asarray([p.parent for p in props], np.int64),
        out_xfer=np.asarray([p.xfer_id for p in props], np.int64),
        out_anchor=np.asarray([p.anchor_slot for p in props], np.int64),
        out_binding=bind,
        out_probability=np.asarray([p.probability for p in props], np.float64),
        out_next_gate=np.asarray([p.next_gate_count for p in props], np.int64),
        predicted=np.int64(metrics["predicted_actions"]), eligible=np.int64(metrics["eligible_actions"]),
    )


def topology_case(*, seed=0, beams=90, depth=7, qubits=4, gates=40, per_step=120):
    """Lazy topology + raw-fingerprint dedup through the reference's own
    lazy_child (indexed backend) and accept loop (paged_rollout_benchmark.py
    :1013-1046), on seeded proposals drawn from every structurally valid
    (source, anchor) of every parent, shuffled, with injected repeats
    (duplicates) and bindings through dead slots (invalid)."""
    import json
    import random

    import tempfile

    import beam_search_benchmark as bsb
    import incremental_graph as ig
    import lazy_rollout_benchmark as lrb
    import paged_rollout_benchmark as prb
    from graph_rewrite_system_b200 import synthetic

    rng = random.Random(seed)
    rules = synthetic.synthetic_rules()
    s2x, deltas = rules.source_to_xfers(), rules.gate_deltas()
    src_pat = tuple(ig.parse_pattern(p) for p in rules.xfer_sources)
    dst_pat = tuple(ig.parse_pattern(p) for p in rules.xfer_destinations)
    circuit = synthetic.random_circuit(qubits, gates, seed)
    snapshot = circuit.snapshot()
    beam = [bsb.BeamState(graph=None, snapshot=snapshot, guid_to_slot={}, next_slot=gates,
                          last_touched={}, rewrite_distance={n[0]: 5 for n in snapshot["nodes"]},
                          previous_preferred=set(), local_streak=0, gate_count=gates, depth=0,
                          history=(), topology_index=lrb.indexed_topology(snapshot))]
    seen = {lrb.raw_topology_hash(snapshot)}
    out = {"circuit_nodes": [list(n) for n in circuit.nodes],
           "circuit_edges": [list(e) for e in circuit.edges], "steps": []}
    for step in range(depth):
        proposals = []
        for parent, state in enumerate(beam):
            topo = state.topology_index
            inc = ig.IncrementalCircuit({"nodes": [(s_, t_, -1) for s_, t_ in topo.nodes.items()],
                                         "edges": list(topo.edges)})
            for source_id, pattern in enumerate(rules.source_patterns):
                ops = ig.parse_pattern(pattern)
                for anchor in sorted(topo.nodes):
                    binding = ig.structural_binding(inc, ops, anchor)
                    if binding is None:
                        continue
                    for xfer in s2x[source_id]:
                        if deltas[xfer] <= 1:
                            proposals.append(bsb.Proposal(parent, xfer, anchor, binding,
                                                          rng.random(),
                                                          state.gate_count + deltas[xfer]))
        rng.shuffle(proposals)
        proposals = proposals[:per_step]
        for _ in range(len(proposals) // 10):       # repeats -> duplicates
            proposals.insert(rng.randrange(len(proposals) + 1), rng.choice(proposals))
        for _ in range(len(proposals) // 20):       # dead slot -> invalid
            p = rng.choice(proposals)
            dead = rng.randrange(beam[p.parent].next_slot, beam[p.parent].next_slot + 50)
            binding = (dead,) + tuple(p.binding[1:])
            proposals.insert(rng.randrange(len(proposals) + 1),
                             bsb.Proposal(p.parent, p.xfer_id, p.anchor_slot, binding,
                                          p.probability, p.next_gate_count))
        records = []
        attempted = invalid = duplicates = 0
        for index, proposal in enumerate(proposals):
            if len(records) >= beams:
                break
            attempted += 1
            child, fingerprint, is_dup = lrb.lazy_child(beam[proposal.parent], proposal, src_pat,
                                                        dst_pat, False, "raw", seen, "indexed")
            if is_dup:
                duplicates += 1
                continue
            if child is None:
                invalid += 1
                continue
            seen.add(fingerprint)
            records.append((child, index))
        records.sort(key=lambda r: (r[0].gate_count, len(r[0].history)))
        records = records[:beams]
        children = []
        for child, index in records:
            topo = child.topology_index
            children.append({
                "proposal": index,
                "nodes": sorted([int(a), int(b)] for a, b in topo.nodes.items()),
                "edges": sorted(list(map(int, e)) for e in topo.edges),
                "next_slot": int(child.next_slot),
                "last_touched": [int(x) for x in child.last_touched],
                "rewrite_distance": [int(x) for x in child.rewrite_distance],
                "previous_preferred": sorted(int(x) for x in child.previous_preferred),
                "local_streak": int(child.local_streak), "gate_count": int(child.gate_count),
                "depth": int(child.depth)})
        beam = [r[0] for r in records]
        # the reference's own beam-level dump line for the new beam
        # (paged_rollout_benchmark.py:213-239)
        with tempfile.TemporaryDirectory() as tmp:
            dump = Path(tmp) / "levels.jsonl"
            prb.append_beam_level(dump, step + 1, beam)
            level_line = dump.read_text()
        out["steps"].append({
            "proposals": [[p.parent, p.xfer_id, p.anchor_slot, list(p.binding),
                           p.next_gate_count] for p in proposals],
            "attempted": attempted, "invalid": invalid, "duplicates": duplicates,
            "children": children, "beam_level_line": level_line})
    return {"json": np.array(json.dumps(out))}


def main() -> None:
    parser = argparse.ArgumentParser()
    parser.add_argument("--reference", type=Path, required=True,
                        help="path of the reference repository checkout (imported read-only)")
    parser.add_argument("--only", default="")
    args = parser.parse_args()
    sys.path.insert(0, str(args.reference))
    import paged_attention as ref_attention
    import paged_cache as ref_cache
    import gpu_proposals as ref_proposals
    import beam_search_benchmark as ref_bsb
    import paged_rollout_benchmark as ref_prb
    import threshold_inference as ref_ti

    only = set(filter(None, args.only.split(",")))
    if not only or "attention" in only:
        np.savez_compressed(HERE / "paged_attention_history.npz", **paged_attention_case(ref_attention, False))
        np.savez_compressed(HERE / "paged_attention_current.npz", **paged_attention_case(ref_attention, True))
    if not only or "cache" in only:
        np.savez_compressed(HERE / "paged_cache_churn_p4.npz",
                            **cache_churn_case(ref_cache, seed=3, beams=8, depth=11, children=3, page=4))
        np.savez_compressed(HERE / "paged_cache_churn_p3.npz",
                            **cache_churn_case(ref_cache, seed=5, beams=13, depth=9, children=5, page=3))
    if not only or "proposals" in only:
        for name, case in proposals_cases(ref_proposals, ref_bsb, ref_prb, ref_ti).items():
            np.savez_compressed(HERE / f"proposals_{name}.npz", **case)
    if not only or "model" in only:
        np.savez_compressed(HERE / "model_cpu_equivalence.npz", **model_case(args.reference))
    if not only or "topology" in only:
        np.savez_compressed(HERE / "topology_accept.npz", **topology_case())
    if not only or "exploration" in only:
        np.savez_compressed(HERE / "proposals_exploration.npz",
                            **exploration_cases(ref_prb, ref_bsb))
    if not only or "checkpoint" in only:
        np.savez_compressed(HERE / "checkpoint_tiny.npz", **checkpoint_case(args.reference))
    if not only or "rollout" in only:
        np.savez_compressed(HERE / "rollout_reference_loop.npz", **rollout_case())
    print("golden fixtures written to", HERE)




def random_prefixes(ref_graph, circuit_snapshot, rules, num_beams, num_actions, seed):
    """Seeded valid action prefixes: at each step pick uniformly among every
    (source, anchor) whose structural binding exists in the current graph
    (the reference's incremental_graph.structural_binding), then a uniform
    xfer of that source; destination slots continue the slot counter."""
    import random

    rng = random.Random(seed)
    s2x = rules.source_to_xfers()
    samples = []
    for beam in range(num_beams):
        circuit = ref_graph.IncrementalCircuit(circuit_snapshot)
        next_slot = max(n[0] for n in circuit_snapshot["nodes"]) + 1
        actions = []
        for _ in range(num_actions):
            options = []
            for source_id, pattern in enumerate(rules.source_patterns):
                ops = ref_graph.parse_pattern(pattern)
                for anchor in sorted(circuit.nodes):
                    binding = ref_graph.structural_binding(circuit, ops, anchor)
                    if binding is not None:
                        options.append((source_id, binding))
            source_id, binding = options[rng.randrange(len(options))]
            xfer = rng.choice(s2x[source_id])
            dst = ref_graph.parse_pattern(rules.xfer_destinations[xfer])
            dst_slots = tuple(range(next_slot, next_slot + len(dst)))
            circuit.apply(ref_graph.parse_pattern(rules.xfer_sources[xfer]), dst, binding, dst_slots)
            next_slot += len(dst)
            actions.append({"xfer_id": xfer, "source_id": source_id,
                            "binding_slots": list(binding), "dst_slots": list(dst_slots)})
        samples.append({"initial_graph": circuit_snapshot, "actions": actions, "matches": [],
                        "prefix_length": num_actions, "local_streak": 0, "previous_action": None,
                        "previous_delta": None, "previous_local_streak": 0})
    return samples


def model_case(reference: Path, *, seed=1, beams=16, actions=8, dag_nodes=64):
    """Full-prefix encode, one-token paged decode, paged readout, match logits,
    structural decode and threshold candidates of the reference model
    (CPU equivalence configuration, seeded weights): 16 beams with an
    8-action prefix each over a random 64-node DAG, page size 4."""
    import dataset as ref_dataset
    import incremental_graph as ref_graph
    import paged_cache as ref_cache
    import paged_model as ref_model
    import threshold_inference as ref_ti
    from graph_rewrite_system_b200 import synthetic
    from oracle.model import parameter_shapes

    rules = synthetic.small_rules()
    cfg = synthetic.CPU_EQUIVALENCE_MODEL
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
        dropout=0.0).eval()
    shapes = parameter_shapes(cfg, rules)
    params = synthetic.deterministic_parameters(shapes, seed)
    state = model.state_dict()
    names = {n for n, _ in model.named_parameters()}
    assert names == set(shapes), (names ^ set(shapes))
    for k, v in params.items():
        assert tuple(state[k].shape) == v.shape, k
        state[k] = torch.from_numpy(v)
    model.load_state_dict(state)

    circuit = synthetic.random_dag(dag_nodes, 8, seed + 1)
    snapshot = circuit.snapshot()
    samples = random_prefixes(ref_graph, snapshot, rules, beams, actions, seed + 2)
    batch = ref_dataset.collate_prefixes(samples, ref_rules)
    out = {}
    for key in ("initial_types", "edge_batch", "edge_src", "edge_dst", "edge_relation",
                "current_types", "current_edge_batch", "current_edge_src", "current_edge_dst",
                "current_edge_relation", "action_xfers", "action_sources", "binding_slots",
                "destination_slots", "destination_types", "current_rewrite_distance"):
        out["batch_" + key] = batch[key].numpy()
    with torch.no_grad():
        full_states, full_live, full_types = model.encode(batch)
        out["encode_states"] = full_states.numpy()
        out["encode_live"] = full_live.numpy()
        out["encode_types"] = full_types.numpy()
        # one-token paged decode, then the paged readout
        s0 = {k: batch[k] for k in ("initial_types", "edge_batch", "edge_src", "edge_dst",
                                    "edge_relation")}
        states, live, types = model.initialize_incremental(s0)
        out["initial_states"] = states.numpy()
        arena = ref_cache.PagedKVCache(layers=cfg.action_layers, capacity=64, page_size=4,
                                       heads=cfg.action_heads,
                                       head_width=cfg.width // cfg.action_heads,
                                       model_width=cfg.width, device=torch.device("cpu"),
                                       dtype=torch.float32)
        handles = [arena.empty_handle()] * beams
        tokens, keys0 = [], []
        for a in range(actions):
            table, lengths = arena.block_table(handles)
            res = model.advance_incremental(
                states, live, types, None, None,
                states.new_empty((beams, 0, cfg.width)), torch.empty((beams, 0), dtype=torch.bool),
                xfer_ids=batch["action_xfers"][:, a], source_ids=batch["action_sources"][:, a],
                source_slots=batch["binding_slots"][:, a],
                destination_slots=batch["destination_slots"][:, a],
                destination_types=batch["destination_types"][:, a],
                paged_key_cache=arena.keys, paged_value_cache=arena.values,
                block_table=table, past_lengths=lengths)
            states, live, types, new_k, new_v, action, _ = res
            rk, rv = model.project_action_readout_kv(action)
            new_handles = arena.append_batch(handles, new_k, new_v, action, rk, rv)
            for h in handles:
                arena.release(h)
            handles = new_handles
            tokens.append(action.numpy())
            keys0.append(new_k[0].numpy())
        out["advance_tokens"] = np.stack(tokens)
        out["advance_keys_layer0"] = np.stack(keys0)
        out["advance_states"] = states.numpy()
        out["advance_live"] = live.numpy()
        out["advance_types"] = types.numpy()
        table, lengths = arena.block_table(handles)
        readout, _, _ = model.readout_incremental(
            states, live, types, states.new_empty((beams, 0, cfg.width)),
            torch.empty((beams, 0), dtype=torch.bool), batch,
            readout_key_cache=arena.readout_keys, readout_value_cache=arena.readout_values,
            block_table=table, lengths=lengths)
        out["readout_states"] = readout.numpy()
        logits, eligible = model.match_logits(readout, live, types)
        out["logits"] = logits.numpy()
        out["eligible"] = eligible.numpy()
        config = {"groups": {g: {"scale": 1.0, "bias": 0.0, "raw_threshold": -1e9}
                             for g in ("near", "far")}}
        cand = ref_ti.threshold_candidate_tensors(model, batch, logits, eligible, config,
                                                  max_candidates_per_state=24)
        for k in ("batch_ids", "sources", "anchors", "bindings", "probabilities"):
            out["candidates_" + k] = getattr(cand, k).numpy()
        # structural decode of every (slot, source) pair with an eligible anchor
        bi, sl, so = eligible.nonzero(as_tuple=True)
        bindings, valid = model.structural_decode(batch, types, live, bi, so, sl)
        out["decode_batch"], out["decode_sources"], out["decode_anchors"] = bi.numpy(), so.numpy(), sl.numpy()
        out["decode_bindings"], out["decode_valid"] = bindings.numpy(), valid.numpy()
    out["seed"] = np.int64(seed)
    return out


def exploration_cases(ref_prb, ref_bsb):
    """build_legacy_proposals (paged_rollout_benchmark.py:101-210) with a
    second model's candidates and an exploration quota, on seeded candidate
    lists: the exploration model re-predicts about half of the primary
    (source, anchor, binding) candidates with its own probabilities and adds
    its own.  Cases: a regular quota, no quota (the cap is checked after an
    append), a quota equal to the cap, and one wide parent (a search's first
    level, where the effective cap is 2 x beam)."""
    import json
    import random

    from graph_rewrite_system_b200 import synthetic

    rules = synthetic.synthetic_rules()
    s2x, deltas = rules.source_to_xfers(), rules.gate_deltas()
    out = {}
    for name, (seed, parents, per_state, beam_size, cap, quota) in {
            "regular": (11, 6, 12, 6, 8, 3), "no_quota": (12, 5, 10, 5, 6, 0),
            "full_quota": (13, 4, 9, 4, 5, 5), "wide": (14, 1, 300, 120, 16, 6)}.items():
        rng = random.Random(seed)
        f32 = lambda: float(np.float32(rng.random()))
        beam = [ref_bsb.BeamState(graph=None, snapshot=None, guid_to_slot={}, next_slot=0,
                                  last_touched={}, rewrite_distance={}, previous_preferred=set(),
                                  local_streak=0, gate_count=rng.randrange(90, 96), depth=0,
                                  history=()) for _ in range(parents)]
        predicted, explored = [], []
        for _ in range(parents):
            rows, seen = [], set()
            while len(rows) < per_state:
                source = rng.randrange(rules.num_sources)
                anchor = rng.randrange(60)
                if (source, anchor) in seen:
                    continue
                seen.add((source, anchor))
                width = len(rules.source_gate_types[source])
                binding = tuple([anchor] + [rng.randrange(60) for _ in range(width - 1)])
                rows.append((source, anchor, binding, f32()))
            extra = []
            for source, anchor, binding, _ in rows:
                if rng.random() < 0.5:
                    extra.append((source, anchor, binding, f32()))
            while len(extra) < per_state:
                source, anchor = rng.randrange(rules.num_sources), 60 + rng.randrange(40)
                if (source, anchor) in seen:
                    continue
                seen.add((source, anchor))
                width = len(rules.source_gate_types[source])
                extra.append((source, anchor,
                              tuple([anchor] + [rng.randrange(60) for _ in range(width - 1)]), f32()))
            rng.shuffle(extra)
            predicted.append(rows)
            explored.append(extra)
        proposals, metrics = ref_prb.build_legacy_proposals(
            beam, predicted, explored, s2x, deltas, beam_size=beam_size,
            max_actions_per_parent=cap, exploration_actions_per_parent=quota,
            proposal_factor=4, max_gate_increase=1)
        out[name] = {
            "gate_counts": [b.gate_count for b in beam],
            "predicted": [[list(r[:2]) + [list(r[2]), r[3]] for r in rows] for rows in predicted],
            "exploration_predicted": [[list(r[:2]) + [list(r[2]), r[3]] for r in rows]
                                      for rows in explored],
            "beam_size": beam_size, "cap": cap, "quota": quota, "proposal_factor": 4,
            "proposals": [[q.parent, q.xfer_id, q.anchor_slot, list(q.binding), q.probability,
                           q.next_gate_count] for q in proposals],
            "metrics": {k: v for k, v in metrics.items() if not k.endswith("_seconds")}}
    return {"json": np.array(json.dumps(out))}


def checkpoint_case(reference: Path, *, seed=4, beams=3, actions=4):
    """A trainer-style checkpoint payload of a tiny reference model built by
    the reference's own build_model (model_factory.py:7-41), saved the way
    train.py:482-490 saves it, with the reference model's full-prefix encode
    of a small seeded batch (paged_model.py:657-777)."""
    import dataset as ref_dataset
    import incremental_graph as ref_graph
    import model_factory as ref_factory
    from graph_rewrite_system_b200 import synthetic

    rules = synthetic.small_rules()
    ref_rules = ref_dataset.RuleMetadata.from_payload({
        "source_patterns": list(rules.source_patterns),
        "xfer_to_source": list(rules.xfer_to_source),
        "xfer_sources": list(rules.xfer_sources),
        "xfer_destinations": list(rules.xfer_destinations)})
    args = {"architecture": "paged_action", "width": 32, "retrieval_width": 16,
            "graph_layers": 1, "action_layers": 1, "action_heads": 2,
            "max_sequence_length": 16, "readout_graph_layers": 1,
            "readout_attention_backend": "sdpa", "lr": 3e-4}
    model = ref_factory.build_model(ref_rules, rules.num_xfers, args).eval()
    g = torch.Generator().manual_seed(seed)
    state = model.state_dict()
    for name, value in state.items():
        if value.is_floating_point():
            state[name] = torch.randn(value.shape, generator=g) * 0.1 + (
                1.0 if name.endswith("norm.weight") else 0.0)
    model.load_state_dict(state)
    circuit = synthetic.random_dag(32, 8, seed)
    samples = random_prefixes(ref_graph, circuit.snapshot(), rules, beams, actions, seed + 1)
    batch = ref_dataset.collate_prefixes(samples, ref_rules)
    with torch.no_grad():
        states, live, types = model.encode(batch)
    payload = {"model": model.state_dict(), "args": args, "metrics": {"loss": 0.0},
               "format": "paged_action_binding"}
    torch.save(payload, HERE / "checkpoint_tiny.pt")
    out = {"batch_" + k: batch[k].numpy() for k in (
        "initial_types", "edge_batch", "edge_src", "edge_dst", "edge_relation",
        "current_types", "current_edge_batch", "current_edge_src", "current_edge_dst",
        "current_edge_relation", "action_xfers", "action_sources", "binding_slots",
        "destination_slots", "destination_types")}
    out.update(encode_states=states.numpy(), encode_live=live.numpy(), encode_types=types.numpy())
    return out


def rollout_case(*, seed=7, beam_size=12, depth=6, qubits=4, gates=30):
    """Six levels of the reference's own search loop on the CPU (fp32):
    paged_model_matches with tensorized state batches and threshold candidate
    tensors, build_gpu_proposals with the effective parent cap, the lazy_child
    accept loop (indexed topology, raw dedup), the gate-count sort and
    advance_selected over a PagedKVCache (paged_rollout_benchmark.py:243-556,
    898-1093).  Seeded weights (synthetic.deterministic_parameters), the
    synthetic rule set and a seeded random circuit."""
    import json
    import math
    from collections import defaultdict

    import beam_search_benchmark as bsb
    import dataset as ref_dataset
    import gpu_proposals as gp
    import incremental_graph as ig
    import lazy_rollout_benchmark as lrb
    import paged_cache as ref_cache
    import paged_model as ref_model
    import paged_rollout_benchmark as prb
    from graph_rewrite_system_b200 import synthetic
    from oracle.model import parameter_shapes

    cfg = synthetic.ModelConfig(**ROLLOUT_GOLDEN_MODEL)
    rc = synthetic.RolloutConfig(**ROLLOUT_GOLDEN_SEARCH)
    assert (rc.beam_size, rc.depth) == (beam_size, depth)
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
        dropout=0.0).eval()
    state = model.state_dict()
    for k, v in synthetic.deterministic_parameters(parameter_shapes(cfg, rules), seed).items():
        assert tuple(state[k].shape) == v.shape, k
        state[k] = torch.from_numpy(v)
    model.load_state_dict(state)
    device = torch.device("cpu")

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

    circuit = synthetic.random_circuit(qubits, gates, seed + 1)
    snapshot = circuit.snapshot()
    beam = [bsb.BeamState(graph=None, snapshot=snapshot, guid_to_slot={}, next_slot=gates,
                          last_touched={}, rewrite_distance={n[0]: 5 for n in snapshot["nodes"]},
                          previous_preferred=set(), local_streak=0, gate_count=gates, depth=0,
                          history=(), topology_index=lrb.indexed_topology(snapshot))]
    with torch.no_grad():
        slot_states, live, gate_types = model.initialize_incremental(prb.initial_batch(snapshot))
        source_vectors = model.retrieval_source(model.source_representations())
    arena = ref_cache.PagedKVCache(layers=cfg.action_layers, capacity=rc.cache_pages,
                                   page_size=rc.page_size, heads=cfg.action_heads,
                                   head_width=cfg.width // cfg.action_heads,
                                   model_width=cfg.width, device=device, dtype=torch.float32)
    handles = [arena.empty_handle()]
    seen = {lrb.raw_topology_hash(snapshot)}
    out = {"circuit_nodes": [list(n) for n in circuit.nodes],
           "circuit_edges": [list(e) for e in circuit.edges], "levels": [],
           "model": ROLLOUT_GOLDEN_MODEL, "search": ROLLOUT_GOLDEN_SEARCH, "seed": seed,
           "qubits": qubits, "gates": gates}
    states_out = {}
    for step in range(depth):
        with torch.no_grad():
            candidates, _, _ = prb.paged_model_matches(
                beam, slot_states, live, gate_types, handles, arena, model, device,
                synthetic.SELECT_ALL_THRESHOLDS, source_vectors, rc.microbatch,
                rc.max_candidates_per_state, "tensorized", "gpu")
        cap = max(rc.per_parent_cap, math.ceil(rc.beam_size / max(1, len(beam))) * 2)
        proposals, metrics, _ = gp.build_gpu_proposals(candidates, beam, rule_index,
                                                       per_parent_cap=cap,
                                                       global_cap=rc.global_cap)
        records = []
        attempted = invalid = duplicates = 0
        for proposal in proposals:
            if len(records) >= rc.beam_size:
                break
            attempted += 1
            child, fingerprint, is_dup = lrb.lazy_child(beam[proposal.parent], proposal, src_pat,
                                                        dst_pat, False, "raw", seen, "indexed")
            if is_dup:
                duplicates += 1
                continue
            if child is None:
                invalid += 1
                continue
            seen.add(fingerprint)
            records.append((child, proposal))
        level = {"input_states": len(beam), "proposals_after_caps": len(proposals),
                 "predicted_actions": int(metrics["predicted_actions"]),
                 "eligible_actions": int(metrics["eligible_actions"]),
                 "attempted": attempted, "invalid": invalid, "duplicates": duplicates}
        if not records:
            out["levels"].append(level | {"children": []})
            break
        records.sort(key=lambda row: (row[0].gate_count, len(row[0].history)))
        records = records[:rc.beam_size]
        with torch.no_grad():
            slot_states, live, gate_types, handles, _, _ = prb.advance_selected(
                slot_states, live, gate_types, handles, records, ref_rules, arena, model,
                device, rc.microbatch)
        beam = [r[0] for r in records]
        level["children"] = [[int(p.parent), int(p.xfer_id), int(p.anchor_slot),
                              [int(x) for x in p.binding], int(c.gate_count)]
                             for c, p in records]
        level["candidate_count"] = int(candidates.batch_ids.numel())
        out["levels"].append(level)
        states_out[f"states_{step}"] = slot_states.numpy()
        states_out[f"live_{step}"] = live.numpy()
        states_out[f"types_{step}"] = gate_types.numpy()
    return {"json": np.array(json.dumps(out)), **states_out}


# The model and search settings of the reference-loop fixture (rollout_case);
# the oracle test rebuilds the same model from the same seed.
ROLLOUT_GOLDEN_MODEL = dict(width=32, retrieval_width=16, graph_layers=1, action_layers=2,
                            action_heads=2, max_sequence_length=16, readout_graph_layers=1)
ROLLOUT_GOLDEN_SEARCH = dict(beam_size=12, depth=6, page_size=4, max_candidates_per_state=400,
                             per_parent_cap=4, proposal_factor=4)


if __name__ == "__main__":
    main()

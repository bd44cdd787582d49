"""Pin the oracle lazy topology + accept loop against the reference's decisions."""
from __future__ import annotations

import json

import numpy as np

from conftest import load_golden
from graph_rewrite_system_b200 import synthetic
from oracle import topology as T


def topology_golden():
    return json.loads(str(load_golden("topology_accept.npz")["json"]))


def rule_patterns():
    rules = synthetic.synthetic_rules()
    src = [synthetic.parse_pattern(p) for p in rules.xfer_sources]
    dst = [synthetic.parse_pattern(p) for p in rules.xfer_destinations]
    return rules, src, dst


def check_children(records, step, slots):
    assert len(records) == len(step["children"])
    for (child, index), exp in zip(records, step["children"]):
        assert index == exp["proposal"]
        assert sorted([s, t] for s, t in child.topology.nodes.items()) == exp["nodes"]
        assert sorted(list(e) for e in child.topology.edges) == exp["edges"]
        assert child.next_slot == exp["next_slot"]
        n = len(exp["last_touched"])
        assert child.last_touched[:n].tolist() == exp["last_touched"]
        assert (child.last_touched[n:] == -1).all()
        m = len(exp["rewrite_distance"])
        assert child.rewrite_distance[:m].tolist() == exp["rewrite_distance"]
        assert sorted(child.previous_preferred) == exp["previous_preferred"]
        assert child.local_streak == exp["local_streak"]
        assert child.gate_count == exp["gate_count"] and child.depth == exp["depth"]


def test_oracle_accept_loop_matches_reference():
    g = topology_golden()
    rules, src, dst = rule_patterns()
    nodes = {s: t for s, t in g["circuit_nodes"]}
    slots = 64 + 3 * len(g["steps"]) + 64
    beam = [T.initial_beam(nodes, [tuple(e) for e in g["circuit_edges"]], slots)]
    seen = {beam[0].topology.fingerprint}
    for step in g["steps"]:
        proposals = [(p, x, a, tuple(b), ng) for p, x, a, b, ng in step["proposals"]]
        records, metrics = T.accept(beam, proposals, src, dst, seen, 90, slots)
        assert metrics == {"attempted": step["attempted"], "invalid": step["invalid"],
                           "duplicates": step["duplicates"]}
        check_children(records, step, slots)
        beam = [r[0] for r in records]


def test_fingerprint_is_order_independent():
    edges = [(0, 1, 0, 0), (1, 2, 0, 1), (3, 2, 0, 0)]
    a = T.indexed_topology({0: 1, 1: 2, 2: 6, 3: 0}, edges)
    b = T.indexed_topology({3: 0, 2: 6, 1: 2, 0: 1}, edges[::-1])
    assert a.fingerprint == b.fingerprint
    c = T.indexed_topology({0: 1, 1: 2, 2: 6, 3: 0}, edges[:2])
    assert a.fingerprint != c.fingerprint


def test_beam_level_lines_match_reference_bytes():
    """The history exporter's JSONL line for each accepted level equals,
    byte for byte, the line the reference's append_beam_level wrote for the
    same beam (paged_rollout_benchmark.py:213-239)."""
    from graph_rewrite_system_b200.history import beam_level_line

    g = topology_golden()
    rules, src, dst = rule_patterns()
    nodes = {s: t for s, t in g["circuit_nodes"]}
    slots = 64 + 3 * len(g["steps"]) + 64
    beam = [T.initial_beam(nodes, [tuple(e) for e in g["circuit_edges"]], slots)]
    seen = {beam[0].topology.fingerprint}
    for depth, step in enumerate(g["steps"], 1):
        proposals = [(p, x, a, tuple(b), ng) for p, x, a, b, ng in step["proposals"]]
        records, _ = T.accept(beam, proposals, src, dst, seen, 90, slots)
        beam = [r[0] for r in records]
        line = beam_level_line(depth, [(n.gate_count, n.history) for n in beam])
        assert line == step["beam_level_line"], depth


TINY = dict(width=32, retrieval_width=16, graph_layers=1, action_layers=1, action_heads=2,
            max_sequence_length=16, readout_graph_layers=1)


def test_reference_checkpoint_loads_and_reproduces_its_encode():
    """tests/golden/checkpoint_tiny.pt was saved from a reference model built
    by the reference's build_model, in its trainer's payload layout; the
    loaded weights drive the oracle to the reference model's own full-prefix
    encode of the recorded batch (fp32, 2e-5)."""
    import torch

    from conftest import GOLDEN, load_golden
    from graph_rewrite_system_b200.model_factory import load_checkpoint
    from oracle.model import OracleModel

    rules = synthetic.small_rules()
    model = load_checkpoint(GOLDEN / "checkpoint_tiny.pt", rules, device="cpu",
                            compute_dtype=torch.float32)
    assert (model.width, model.action_heads, model.action_layers_count) == (32, 2, 1)
    params = {k: v for k, v in model.state_dict().items() if k in dict(model.named_parameters())}
    oracle = OracleModel(params, rules, synthetic.ModelConfig(**TINY))
    g = load_golden("checkpoint_tiny.npz")
    batch = {k[len("batch_"):]: torch.from_numpy(v) for k, v in g.items() if k.startswith("batch_")}
    states, live, types = oracle.encode(batch)
    np.testing.assert_allclose(states.numpy(), g["encode_states"], rtol=2e-5, atol=2e-5)
    assert np.array_equal(live.numpy(), g["encode_live"])
    assert np.array_equal(types.numpy(), g["encode_types"])


def test_checkpoint_payload_builds_the_reference_architecture(tmp_path):
    """A trainer-style payload ({'model', 'args', 'metrics', 'format'}) loads
    through load_checkpoint into a model with the reference's argument
    mapping; every parameter round-trips."""
    import torch

    from graph_rewrite_system_b200.model_factory import build_model, load_checkpoint
    from oracle.model import parameter_shapes

    rules = synthetic.small_rules()
    cfg = synthetic.CPU_EQUIVALENCE_MODEL
    args = {"architecture": "paged_action", "width": cfg.width,
            "retrieval_width": cfg.retrieval_width, "graph_layers": cfg.graph_layers,
            "action_layers": cfg.action_layers, "action_heads": cfg.action_heads,
            "max_sequence_length": cfg.max_sequence_length,
            "readout_graph_layers": cfg.readout_graph_layers,
            "readout_attention_backend": "sdpa"}
    params = synthetic.deterministic_parameters(parameter_shapes(cfg, rules), 4)
    model = build_model(rules, rules.num_xfers, args, compute_dtype=torch.float32)
    state = model.state_dict()
    for k, v in params.items():
        state[k] = torch.from_numpy(v)
    path = tmp_path / "ckpt.pt"
    torch.save({"model": state, "args": args, "metrics": {}, "format": "paged_action"}, path)
    loaded = load_checkpoint(path, rules, device="cpu", compute_dtype=torch.float32)
    assert loaded.readout_attention_backend == "paged" and not loaded.training
    got = loaded.state_dict()
    for k, v in params.items():
        assert torch.equal(got[k], torch.from_numpy(v)), k
    import pytest

    with pytest.raises(NotImplementedError):
        build_model(rules, rules.num_xfers, dict(args, architecture="legacy"))
    with pytest.raises(ValueError):
        load_checkpoint({"model": state}, rules, device="cpu")

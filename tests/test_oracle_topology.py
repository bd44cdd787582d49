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

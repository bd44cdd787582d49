"""CUDA expansion/ranking vs the reference's recorded proposals (bit-exact)."""
from __future__ import annotations

import numpy as np
import pytest
import torch

from conftest import load_golden

pytestmark = pytest.mark.gpu


def _device_proposals(g, dev):
    from graph_rewrite_system_b200.gpu_proposals import GpuRuleIndex, build_gpu_proposals
    from graph_rewrite_system_b200.types import BeamState, CandidateTensors

    s2x = {}
    for x, s in enumerate(g["xfer_to_source"].tolist()):
        s2x.setdefault(s, []).append(x)
    index = GpuRuleIndex.build(s2x, g["gate_deltas"].tolist(), int(g["num_sources"]),
                               int(g["max_gate_increase"]), dev)
    t = lambda k: torch.from_numpy(g[k]).to(dev)
    cand = CandidateTensors(t("batch_ids"), t("sources"), t("anchors"), t("bindings"),
                            t("probabilities"))
    beam = [BeamState(None, None, {}, 0, {}, {}, set(), 0, int(x), 1, ())
            for x in g["parent_gates"]]
    return build_gpu_proposals(cand, beam, index, per_parent_cap=int(g["per_parent_cap"]),
                               global_cap=int(g["global_cap"]))


@pytest.mark.parametrize("name", ["proposals_small.npz", "proposals_random.npz"])
def test_golden(cuda_device, name):
    g = load_golden(name)
    props, metrics, _ = _device_proposals(g, cuda_device)
    assert [p.parent for p in props] == g["out_parent"].tolist()
    assert [p.xfer_id for p in props] == g["out_xfer"].tolist()
    assert [p.anchor_slot for p in props] == g["out_anchor"].tolist()
    assert [p.next_gate_count for p in props] == g["out_next_gate"].tolist()
    for p, row in zip(props, g["out_binding"]):
        assert list(p.binding) == [int(b) for b in row if b >= 0]
    np.testing.assert_allclose([p.probability for p in props], g["out_probability"], atol=1e-7)
    assert metrics == {"predicted_actions": int(g["predicted"]),
                       "eligible_actions": int(g["eligible"])}


@pytest.mark.parametrize("seed", [0, 1, 2])
def test_random_vs_oracle(cuda_device, seed):
    """Config-4 shaped: 1000 parents x 80 candidates, cap 16, global 16000."""
    from graph_rewrite_system_b200.gpu_proposals import GpuRuleIndex, rank_proposals_device
    from graph_rewrite_system_b200.synthetic import synthetic_rules
    from oracle import proposals as oracle

    rules = synthetic_rules()
    rng = np.random.default_rng(seed)
    parents, per = 1000, 80
    batch = np.repeat(np.arange(parents), per)
    sources = rng.integers(0, rules.num_sources, batch.size)
    probs = (1 / (1 + np.exp(-rng.integers(-40, 40, batch.size) / 8.0))).astype(np.float32)
    gates = rng.integers(255, 262, parents)
    s2x, deltas = rules.source_to_xfers(), rules.gate_deltas()
    index_o = oracle.build_rule_index(s2x, deltas, rules.num_sources, 1)
    sel, metrics = oracle.rank_proposals(batch, sources, np.zeros(batch.size, np.int64),
                                         np.zeros((batch.size, 1), np.int64), probs, gates,
                                         index_o, per_parent_cap=16, global_cap=16000)
    index = GpuRuleIndex.build(s2x, deltas, rules.num_sources, 1, cuda_device)
    d = lambda a: torch.from_numpy(np.asarray(a)).to(cuda_device)
    ranked = rank_proposals_device(d(batch), d(sources), d(probs), d(gates), index,
                                   per_parent_cap=16, global_cap=16000)
    count = int(ranked.count.item())
    assert int(ranked.status.item()) == 0
    assert count == len(sel["row"])
    np.testing.assert_array_equal(ranked.rows[:count].cpu().numpy(), sel["candidate"])
    np.testing.assert_array_equal(ranked.xfer_ids[:count].cpu().numpy(), sel["xfer"])
    np.testing.assert_array_equal(ranked.next_gate[:count].cpu().numpy(), sel["next_gate"])
    assert ranked.metrics.tolist() == [metrics["predicted_actions"], metrics["eligible_actions"]]


@pytest.mark.parametrize("seed,k,cap", [(0, 80, 16), (1, 300, 5), (2, 2048, 16), (3, 7, 2000)])
def test_grouped_matches_general(cuda_device, seed, k, cap):
    """Padded parent-grouped layout: the shared-memory per-parent path equals
    the general expansion + stable radix sort path, bit for bit."""
    from graph_rewrite_system_b200.gpu_proposals import (GpuRuleIndex, rank_proposals_device,
                                                         rank_proposals_grouped)
    from graph_rewrite_system_b200.synthetic import synthetic_rules

    rules = synthetic_rules()
    rng = np.random.default_rng(seed)
    parents = 120
    n = parents * k
    sources = rng.integers(0, rules.num_sources, n)
    sources[rng.random(n) < 0.6] = -1                           # absent rows
    probs = (1 / (1 + np.exp(-rng.integers(-20, 20, n) / 4.0))).astype(np.float32)  # ties
    gates = rng.integers(250, 256, parents)
    batch = np.repeat(np.arange(parents), k)
    index = GpuRuleIndex.build(rules.source_to_xfers(), rules.gate_deltas(), rules.num_sources, 1,
                               cuda_device)
    d = lambda a: torch.from_numpy(np.asarray(a)).to(cuda_device)
    general = rank_proposals_device(d(batch), d(sources), d(probs), d(gates), index,
                                    per_parent_cap=cap, global_cap=1500)
    grouped = rank_proposals_grouped(d(sources), d(probs), k, d(gates), index,
                                     per_parent_cap=cap, global_cap=1500)
    assert int(general.status.item()) == 0 and int(grouped.status.item()) == 0
    c = int(general.count.item())
    assert int(grouped.count.item()) == c
    assert torch.equal(grouped.rows[:c], general.rows[:c])
    assert torch.equal(grouped.xfer_ids[:c], general.xfer_ids[:c])
    assert torch.equal(grouped.next_gate[:c], general.next_gate[:c])
    assert torch.equal(grouped.metrics, general.metrics)


def _exploration_random_case(seed, parents, per_state, maxp, rules):
    """Two models' candidate tables over the same slots: the exploration
    model repeats about half of the primary (source, anchor, binding)
    candidates with its own probabilities and adds its own."""
    g = np.random.default_rng(seed)

    def rows_for(parent, pairs):
        out = []
        for source, anchor in pairs:
            width = len(rules.source_gate_types[source])
            binding = [anchor] + [int(v) for v in g.integers(0, 200, width - 1)]
            out.append((parent, source, anchor, binding + [-1] * (maxp - width),
                        float(np.float32(g.random()))))
        return out

    prim, expl = [], []
    for b in range(parents):
        pairs = set()
        while len(pairs) < per_state:
            pairs.add((int(g.integers(rules.num_sources)), int(g.integers(0, 200))))
        pairs = sorted(pairs)
        p_rows = rows_for(b, pairs)
        shared = [(r[1], r[2], r[3]) for r in p_rows if g.random() < 0.5]
        e_rows = [(b, s, a, bd, float(np.float32(g.random()))) for s, a, bd in shared]
        extra = set()
        while len(extra) < per_state // 2:
            pair = (int(g.integers(rules.num_sources)), int(g.integers(200, 300)))
            extra.add(pair)
        e_rows += rows_for(b, sorted(extra))
        g.shuffle(e_rows)
        prim += p_rows
        expl += e_rows

    def table(rows):
        return {"batch_ids": np.asarray([r[0] for r in rows], np.int64),
                "sources": np.asarray([r[1] for r in rows], np.int64),
                "anchors": np.asarray([r[2] for r in rows], np.int64),
                "bindings": np.asarray([r[3] for r in rows], np.int64).reshape(-1, maxp),
                "probabilities": np.asarray([r[4] for r in rows], np.float32)}

    return table(prim), table(expl), g.integers(100, 104, parents).astype(np.int64)


def test_exploration_ranking_matches_oracle(cuda_device):
    """grs_proposals_rank_exploration = the oracle's restatement of
    build_legacy_proposals with a second model (pinned to the reference's
    own outputs on CPU): same proposals in the same order, same metrics."""
    from test_oracle_golden import exploration_golden, exploration_inputs
    from graph_rewrite_system_b200 import synthetic
    from graph_rewrite_system_b200.gpu_proposals import GpuRuleIndex, rank_proposals_exploration
    from oracle import proposals as P

    rules = synthetic.synthetic_rules()
    maxp = max(map(len, rules.source_gate_types))
    index_o = P.build_rule_index(rules.source_to_xfers(), rules.gate_deltas(), rules.num_sources, 1)
    index = GpuRuleIndex.build(rules.source_to_xfers(), rules.gate_deltas(), rules.num_sources, 1,
                               cuda_device)
    cases = []
    for case in exploration_golden().values():
        primary, explored, gates, cap, gcap = exploration_inputs(case, maxp)
        cases.append((primary, explored, gates, cap, case["quota"], gcap))
    for seed, parents, per_state, cap, quota in [(1, 40, 30, 16, 4), (2, 25, 24, 12, 0),
                                                 (3, 30, 20, 10, 10), (4, 1, 900, 600, 50)]:
        primary, explored, gates = _exploration_random_case(seed, parents, per_state, maxp, rules)
        cases.append((primary, explored, gates, cap, quota, max(parents * 16, parents * cap)))
    dev = lambda t: {k: torch.from_numpy(v).to(cuda_device) for k, v in t.items()}
    for primary, explored, gates, cap, quota, gcap in cases:
        sel, metrics = P.rank_proposals_exploration(primary, explored, gates, index_o,
                                                    per_parent_cap=cap,
                                                    exploration_per_parent=quota, global_cap=gcap)
        ranked, m = rank_proposals_exploration(dev(primary), dev(explored),
                                               torch.from_numpy(gates).to(cuda_device), index,
                                               per_parent_cap=cap, exploration_per_parent=quota,
                                               global_cap=gcap)
        count = int(ranked.count.item())
        assert int(ranked.status.item()) == 0
        rows = ranked.rows[:count].cpu().numpy()
        table = {k: np.concatenate((primary[k], explored[k])) for k in primary}
        got = [(int(table["batch_ids"][r]), int(x), int(table["anchors"][r]),
                tuple(int(v) for v in table["bindings"][r] if v >= 0), int(n))
               for r, x, n in zip(rows, ranked.xfer_ids[:count].tolist(),
                                  ranked.next_gate[:count].tolist())]
        exp = [(int(p), int(x), int(a), tuple(b), int(n)) for p, x, a, b, n in zip(
            sel["parent"], sel["xfer"], sel["anchor"], sel["binding"], sel["next_gate"])]
        assert got == exp, (cap, quota)
        assert m.tolist() == [metrics["predicted_actions"], metrics["eligible_actions"],
                              metrics["exploration_predicted_actions"],
                              metrics["exploration_eligible_actions"],
                              metrics["selected_exploration_proposals"]]

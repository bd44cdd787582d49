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

"""Pin the CPU oracle against vectors produced by the reference's own code.

The fixtures (tests/golden/*.npz) were written by tests/golden/make_golden.py
from the reference implementation; the oracle must reproduce them exactly
(integer state) or within fp32 tolerance (attention).
"""
from __future__ import annotations

import numpy as np
import torch

from conftest import load_golden
from oracle import paged_attention as oracle_attention
from oracle.paged_cache import OraclePagedKVCache
from oracle import proposals as oracle_proposals


def _attention_case(name, with_current):
    g = load_golden(name)
    kwargs = {}
    if with_current:
        kwargs = dict(current_key=torch.from_numpy(g["current_key"]),
                      current_value=torch.from_numpy(g["current_value"]),
                      current_valid=torch.from_numpy(g["current_valid"]))
    out = oracle_attention.paged_attention(
        torch.from_numpy(g["query"]), torch.from_numpy(g["keys"]), torch.from_numpy(g["values"]),
        torch.from_numpy(g["block_table"]), torch.from_numpy(g["lengths"]), **kwargs)
    np.testing.assert_allclose(out.numpy(), g["output"], rtol=1e-5, atol=1e-5)
    if not with_current:
        assert not out[0].any()


def test_oracle_attention_history_only():
    _attention_case("paged_attention_history.npz", False)


def test_oracle_attention_with_current():
    _attention_case("paged_attention_current.npz", True)


def replay_churn(g, make_cache, check):
    """Replay a recorded churn sequence on a cache built by make_cache(); call
    check(step, cache, handles) after every step."""
    cache = make_cache(g)
    handles = [cache.empty_handle()]
    for step in range(int(g["depth"])):
        parents = g[f"s{step}_parents"].tolist()
        new = cache.append_batch([handles[p] for p in parents],
                                 torch.from_numpy(g[f"s{step}_keys"]),
                                 torch.from_numpy(g[f"s{step}_values"]),
                                 torch.from_numpy(g[f"s{step}_actions"]),
                                 torch.from_numpy(g[f"s{step}_rkeys"]),
                                 torch.from_numpy(g[f"s{step}_rvalues"]))
        for h in handles:
            cache.release(h)
        handles = new
        check(step, cache, handles)
    for h in handles:
        cache.release(h)
    return cache


def _oracle_cache(g):
    return OraclePagedKVCache(layers=int(g["layers"]), capacity=int(g["capacity"]),
                              page_size=int(g["page"]), heads=int(g["heads"]),
                              head_width=int(g["hw"]), model_width=int(g["width"]))


def _check_churn_step(g, step, cache, handles):
    table = g[f"s{step}_table"]
    for i, h in enumerate(handles):
        assert list(h.blocks) == [int(p) for p in table[i, : len(h.blocks)]]
    assert [h.length for h in handles] == g[f"s{step}_lengths"].tolist()
    assert cache.refcounts == g[f"s{step}_refcounts"].tolist()
    assert cache.free == g[f"s{step}_free"].tolist()
    _, values, actions, mask = cache.gather(handles)
    np.testing.assert_array_equal(values.numpy(), g[f"s{step}_gather_values"])
    np.testing.assert_array_equal(actions.numpy(), g[f"s{step}_gather_actions"])


def test_oracle_cache_churn():
    for name in ("paged_cache_churn_p4.npz", "paged_cache_churn_p3.npz"):
        g = load_golden(name)
        cache = replay_churn(g, _oracle_cache, lambda s, c, h: _check_churn_step(g, s, c, h))
        assert cache.allocated_pages == int(g["final_allocated"]) == 0


def test_oracle_cache_errors():
    cache = OraclePagedKVCache(layers=1, capacity=2, page_size=2, heads=1, head_width=2,
                               model_width=2)
    root = cache.empty_handle()
    kv = torch.zeros(1, 3, 1, 2)
    try:
        cache.append_batch([root] * 3, kv, kv, torch.zeros(3, 2))
        raise AssertionError("expected exhaustion")
    except RuntimeError as exc:
        assert "exhausted" in str(exc)


def proposals_from_golden(g):
    s2x = {}
    for x, s in enumerate(g["xfer_to_source"].tolist()):
        s2x.setdefault(s, []).append(x)
    index = oracle_proposals.build_rule_index(s2x, g["gate_deltas"].tolist(), int(g["num_sources"]),
                                              int(g["max_gate_increase"]))
    return oracle_proposals.rank_proposals(
        g["batch_ids"], g["sources"], g["anchors"], g["bindings"], g["probabilities"],
        g["parent_gates"], index, per_parent_cap=int(g["per_parent_cap"]),
        global_cap=int(g["global_cap"]))


def test_oracle_proposals():
    for name in ("proposals_small.npz", "proposals_random.npz"):
        g = load_golden(name)
        sel, metrics = proposals_from_golden(g)
        np.testing.assert_array_equal(sel["parent"], g["out_parent"])
        np.testing.assert_array_equal(sel["xfer"], g["out_xfer"])
        np.testing.assert_array_equal(sel["anchor"], g["out_anchor"])
        np.testing.assert_array_equal(sel["next_gate"], g["out_next_gate"])
        bind = np.where(sel["binding"] >= 0, sel["binding"], -1)
        for i in range(len(bind)):
            row = [b for b in bind[i] if b >= 0]
            assert row == [b for b in g["out_binding"][i] if b >= 0]
        np.testing.assert_allclose(sel["probability"], g["out_probability"], rtol=0, atol=1e-7)
        assert metrics == {"predicted_actions": int(g["predicted"]),
                           "eligible_actions": int(g["eligible"])}


def exploration_golden():
    import json

    return json.loads(str(load_golden("proposals_exploration.npz")["json"]))


def exploration_inputs(case, max_pattern):
    """The golden case's per-state candidate lists as padded candidate tables."""
    import math

    def table(per_state):
        batch, sources, anchors, bindings, probs = [], [], [], [], []
        for parent, rows in enumerate(per_state):
            for source, anchor, binding, prob in rows:
                batch.append(parent)
                sources.append(source)
                anchors.append(anchor)
                bindings.append(list(binding) + [-1] * (max_pattern - len(binding)))
                probs.append(prob)
        return {"batch_ids": np.asarray(batch, np.int64), "sources": np.asarray(sources, np.int64),
                "anchors": np.asarray(anchors, np.int64),
                "bindings": np.asarray(bindings, np.int64).reshape(-1, max_pattern),
                "probabilities": np.asarray(probs, np.float32)}

    parents = len(case["gate_counts"])
    cap = max(case["cap"], math.ceil(case["beam_size"] / max(1, parents)) * 2)
    return (table(case["predicted"]), table(case["exploration_predicted"]),
            np.asarray(case["gate_counts"], np.int64), cap,
            case["beam_size"] * case["proposal_factor"])


def test_oracle_exploration_quota_matches_reference():
    """build_legacy_proposals with a second model's candidates and an
    exploration quota (paged_rollout_benchmark.py:101-210): the oracle
    selects the reference's proposals in the reference's order."""
    from graph_rewrite_system_b200 import synthetic
    from oracle import proposals as P

    rules = synthetic.synthetic_rules()
    index = P.build_rule_index(rules.source_to_xfers(), rules.gate_deltas(), rules.num_sources, 1)
    maxp = max(map(len, rules.source_gate_types))
    for name, case in exploration_golden().items():
        primary, explored, gates, cap, global_cap = exploration_inputs(case, maxp)
        sel, metrics = P.rank_proposals_exploration(
            primary, explored, gates, index, per_parent_cap=cap,
            exploration_per_parent=case["quota"], global_cap=global_cap)
        got = [[int(p), int(x), int(a), list(b), int(n)] for p, x, a, b, n in zip(
            sel["parent"], sel["xfer"], sel["anchor"], sel["binding"], sel["next_gate"])]
        exp = [[p, x, a, b, n] for p, x, a, b, _, n in case["proposals"]]
        assert got == exp, name
        assert metrics == case["metrics"], name

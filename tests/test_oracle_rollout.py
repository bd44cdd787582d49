"""The oracle beam search against the reference's own search loop.

tests/golden/rollout_reference_loop.npz holds six levels of the reference's
loop run on the CPU in fp32 (paged_model_matches -> build_gpu_proposals ->
lazy_child accept loop -> gate-count sort -> advance_selected,
paged_rollout_benchmark.py:243-556, 898-1093) over seeded weights, the
synthetic rule set and a seeded circuit.  The oracle loop (oracle/rollout.py)
must take the same decisions at every level (every accepted child's parent,
xfer, anchor binding and gate count, in order; attempted / duplicate /
invalid counts; proposal and expansion metrics) and reach the same slot
states (fp32, 1e-4).
"""
from __future__ import annotations

import json

import numpy as np
import torch

from conftest import load_golden


def test_oracle_loop_matches_reference_loop():
    from graph_rewrite_system_b200 import synthetic
    from oracle.model import OracleModel, parameter_shapes
    from oracle.rollout import OracleBeamSearch

    g = load_golden("rollout_reference_loop.npz")
    spec = json.loads(str(g["json"]))
    cfg = synthetic.ModelConfig(**spec["model"])
    rc = synthetic.RolloutConfig(**spec["search"])
    rules = synthetic.synthetic_rules()
    params = synthetic.deterministic_parameters(parameter_shapes(cfg, rules), spec["seed"])
    model = OracleModel({k: torch.from_numpy(v) for k, v in params.items()}, rules, cfg)
    circuit = synthetic.random_circuit(spec["qubits"], spec["gates"], spec["seed"] + 1)
    assert [list(n) for n in circuit.nodes] == spec["circuit_nodes"]
    assert [list(e) for e in circuit.edges] == spec["circuit_edges"]

    search = OracleBeamSearch(model, rules, circuit, rc, synthetic.SELECT_ALL_THRESHOLDS)
    search.reset()
    duplicates = 0
    for step, level in enumerate(spec["levels"]):
        row = search.step()
        assert row is not None
        assert row["input_states"] == level["input_states"]
        assert row["proposals_after_caps"] == level["proposals_after_caps"]
        assert row["predicted_actions"] == level["predicted_actions"]
        assert row["eligible_actions_before_parent_cap"] == level["eligible_actions"]
        assert row["attempted_actions"] == level["attempted"]
        assert row["invalid_structural_actions"] == level["invalid"]
        assert row["duplicate_speculative_successors"] == level["duplicates"]
        duplicates += level["duplicates"]
        expected = [(c[0], c[1], tuple(c[3])) for c in level["children"]]
        assert row["children"] == expected, step
        assert [n.gate_count for n in search.beam] == [c[4] for c in level["children"]]
        live = g[f"live_{step}"]
        s = live.shape[1]
        assert np.array_equal(search.primary.live[:, :s].numpy(), live)
        assert not search.primary.live[:, s:].any()
        assert np.array_equal(search.primary.types[:, :s].numpy(), g[f"types_{step}"])
        got = search.primary.states[:, :s].numpy() * live[..., None]
        want = g[f"states_{step}"] * live[..., None]
        np.testing.assert_allclose(got, want, rtol=1e-4, atol=1e-4)
    assert duplicates > 0          # the fixture exercises the dedup path

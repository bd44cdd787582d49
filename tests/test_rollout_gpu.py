"""Device beam search vs the oracle beam search (the reference loop restated).

fp32: the per-level decisions (every accepted child's parent, xfer and
binding, in order), the accept/duplicate/invalid counts, the proposal and
expansion metrics, the final 64-bit topology fingerprints and the exported
beam-level history lines must match exactly.  bf16 at the rollout model's shape: the search runs, the device
topology types equal the model's live-slot types, every invariant holds and
the cache returns every page.
"""
from __future__ import annotations

import numpy as np
import pytest
import torch

pytestmark = pytest.mark.gpu


def _setup(dev, dtype, cfg, seed, qubits, gates, rollout):
    from graph_rewrite_system_b200 import synthetic
    from oracle.model import OracleModel, parameter_shapes
    from test_paged_model_gpu import build_model

    rules = synthetic.synthetic_rules()
    model = build_model(dev, dtype, rules, cfg, seed)
    params = synthetic.deterministic_parameters(parameter_shapes(cfg, rules), seed)
    oracle = OracleModel({k: torch.from_numpy(v) for k, v in params.items()}, rules, cfg)
    circuit = synthetic.random_circuit(qubits, gates, seed + 1)
    return rules, model, oracle, circuit


SMALL = dict(width=64, retrieval_width=32, graph_layers=1, action_layers=2, action_heads=2,
             max_sequence_length=64, readout_graph_layers=2)


@pytest.mark.parametrize("seed", [3, 4])
def test_fp32_rollout_matches_oracle(cuda_device, seed):
    from graph_rewrite_system_b200 import synthetic
    from graph_rewrite_system_b200.history import BeamHistoryRecorder, beam_level_line
    from graph_rewrite_system_b200.rollout import DeviceBeamSearch
    from oracle.rollout import OracleBeamSearch
    from oracle.topology import node_component  # noqa: F401  (same hash family)

    cfg = synthetic.ModelConfig(**SMALL)
    rc = synthetic.RolloutConfig(beam_size=12, depth=6, page_size=4, max_candidates_per_state=400,
                                 per_parent_cap=4, proposal_factor=4)
    rules, model, oracle_model, circuit = _setup(cuda_device, torch.float32, cfg, seed, 4, 30, rc)
    oracle = OracleBeamSearch(oracle_model, rules, circuit, rc, synthetic.SELECT_ALL_THRESHOLDS)
    oracle.reset()
    search = DeviceBeamSearch(model, rules, circuit, rc, cuda_device)
    search.reset()
    recorder = BeamHistoryRecorder(search)
    for _ in range(rc.depth):
        exp = oracle.step()
        got = search.step()
        if exp is None:
            assert got is None
            break
        assert got is not None
        # the exported JSONL line of the level equals the oracle beam's
        recorder.record()
        assert beam_level_line(recorder.depth, recorder.states()) == beam_level_line(
            got.step, [(n.gate_count, n.history) for n in oracle.beam])
        for key in ("accepted_actions", "attempted_actions", "invalid_structural_actions",
                    "duplicate_speculative_successors", "proposals_after_caps",
                    "predicted_actions", "eligible_actions_before_parent_cap"):
            assert getattr(got, key) == exp[key], (got.step, key, getattr(got, key), exp[key])
        assert search.last_children() == exp["children"], got.step
        assert torch.equal(search.types, search.topo.types)
        fps = [int(x) & ((1 << 64) - 1) for x in search.topo.fingerprint.tolist()]
        assert fps == [n.topology.fingerprint for n in oracle.beam]
        assert search.topo.gate.tolist() == [n.gate_count for n in oracle.beam]
        assert search.topo.streak.tolist() == [n.local_streak for n in oracle.beam]
        s = search.slots
        dist = search.topo.distance.cpu().numpy()
        touched = search.topo.touched.cpu().numpy()
        for i, n in enumerate(oracle.beam):
            assert (dist[i] == n.rewrite_distance[:s]).all()
            assert (touched[i] == n.last_touched[:s]).all()
        # model states agree with the oracle's dense-history recomputation
        np.testing.assert_allclose(search.states.float().cpu().numpy()[:, : oracle.states.shape[1]],
                                   oracle.states.numpy(), rtol=1e-4, atol=1e-4)
    search.check()


def test_bf16_rollout_model_shape_invariants(cuda_device):
    from graph_rewrite_system_b200 import synthetic
    from graph_rewrite_system_b200.rollout import DeviceBeamSearch

    cfg = synthetic.ROLLOUT_MODEL
    rc = synthetic.RolloutConfig(beam_size=96, depth=6, page_size=16, max_candidates_per_state=80,
                                 per_parent_cap=16, proposal_factor=16)
    rules, model, _, circuit = _setup(cuda_device, torch.bfloat16, cfg, 0, 6, 259, rc)
    search = DeviceBeamSearch(model, rules, circuit, rc, cuda_device)
    rows = search.run()
    assert len(rows) == rc.depth and all(r.accepted_actions > 0 for r in rows)
    for r in rows:
        assert r.accepted_actions <= rc.beam_size
        assert r.attempted_actions == (r.accepted_actions + r.invalid_structural_actions
                                       + r.duplicate_speculative_successors)
        assert r.proposals_after_caps <= min(rc.global_cap, r.eligible_actions_before_parent_cap)
    assert torch.equal(search.types, search.topo.types)
    gates = search.topo.gate.tolist()
    assert gates == sorted(gates)                      # records sorted by gate count
    live = (search.types >= 0).sum(1).tolist()
    assert live == gates                               # gate count == live nodes
    fps = search.topo.fingerprint.tolist()
    assert len(set(fps)) == len(fps)                   # raw dedup: all distinct
    search.cache.release_device(search.block_table, search.lengths)
    search.check()
    assert search.cache.allocated_pages == 0


@pytest.mark.parametrize("quota,until", [(2, 2), (3, 0), (0, 3)])
def test_fp32_rollout_with_exploration_model_matches_oracle(cuda_device, quota, until):
    """A second (exploration) model searched alongside the primary one
    (paged_rollout_benchmark.py:724-758, 917-961, 1071-1091): per level the
    same children in the same order, the same proposal and exploration
    metrics and fingerprints as the oracle search; the second model leaves
    the search at level `until` (0: stays)."""
    from graph_rewrite_system_b200 import synthetic
    from graph_rewrite_system_b200.history import BeamHistoryRecorder, beam_level_line
    from graph_rewrite_system_b200.rollout import DeviceBeamSearch
    from oracle.model import OracleModel, parameter_shapes
    from oracle.rollout import OracleBeamSearch
    from test_paged_model_gpu import build_model

    cfg = synthetic.ModelConfig(**SMALL)
    rc = synthetic.RolloutConfig(beam_size=12, depth=5, page_size=4, max_candidates_per_state=400,
                                 per_parent_cap=4, proposal_factor=4)
    rules, model, oracle_model, circuit = _setup(cuda_device, torch.float32, cfg, 3, 4, 30, rc)
    x_model = build_model(cuda_device, torch.float32, rules, cfg, 9)
    x_params = synthetic.deterministic_parameters(parameter_shapes(cfg, rules), 9)
    x_oracle = OracleModel({k: torch.from_numpy(v) for k, v in x_params.items()}, rules, cfg)
    oracle = OracleBeamSearch(oracle_model, rules, circuit, rc, synthetic.SELECT_ALL_THRESHOLDS,
                              exploration_model=x_oracle, exploration_per_parent=quota,
                              exploration_until_depth=until)
    oracle.reset()
    search = DeviceBeamSearch(model, rules, circuit, rc, cuda_device, exploration_model=x_model,
                              exploration_per_parent=quota, exploration_until_depth=until)
    search.reset()
    recorder = BeamHistoryRecorder(search)
    for level in range(rc.depth):
        exp = oracle.step()
        got = search.step()
        if exp is None:
            assert got is None
            break
        for key in ("accepted_actions", "attempted_actions", "invalid_structural_actions",
                    "duplicate_speculative_successors", "proposals_after_caps",
                    "predicted_actions", "eligible_actions_before_parent_cap",
                    "exploration_predicted_actions", "exploration_eligible_actions",
                    "selected_exploration_proposals"):
            assert getattr(got, key) == exp.get(key, 0), (got.step, key)
        assert search.last_children() == exp["children"], got.step
        fps = [int(x) & ((1 << 64) - 1) for x in search.topo.fingerprint.tolist()]
        assert fps == [n.topology.fingerprint for n in oracle.beam]
        recorder.record()
        assert beam_level_line(recorder.depth, recorder.states()) == beam_level_line(
            got.step, [(n.gate_count, n.history) for n in oracle.beam])
        assert search.exploring == (until == 0 or level < until)
    if until and rc.depth > until:
        assert search.exploration_cache.allocated_pages == 0     # released when it left
    search.check()


def test_fp32_device_search_matches_reference_loop(cuda_device):
    """The device search against the reference's own loop, recorded in
    tests/golden/rollout_reference_loop.npz (six CPU fp32 levels of
    paged_model_matches -> build_gpu_proposals -> lazy_child -> advance_selected,
    paged_rollout_benchmark.py:243-556, 898-1093): every level's children,
    counts and metrics equal, slot states within 1e-4."""
    import json

    from conftest import load_golden
    from graph_rewrite_system_b200 import synthetic
    from graph_rewrite_system_b200.rollout import DeviceBeamSearch
    from test_paged_model_gpu import build_model

    g = load_golden("rollout_reference_loop.npz")
    spec = json.loads(str(g["json"]))
    cfg = synthetic.ModelConfig(**spec["model"])
    rc = synthetic.RolloutConfig(**spec["search"])
    rules = synthetic.synthetic_rules()
    model = build_model(cuda_device, torch.float32, rules, cfg, spec["seed"])
    circuit = synthetic.random_circuit(spec["qubits"], spec["gates"], spec["seed"] + 1)
    search = DeviceBeamSearch(model, rules, circuit, rc, cuda_device)
    search.reset()
    for step, level in enumerate(spec["levels"]):
        got = search.step()
        assert got is not None
        assert got.input_states == level["input_states"]
        assert got.proposals_after_caps == level["proposals_after_caps"]
        assert got.predicted_actions == level["predicted_actions"]
        assert got.eligible_actions_before_parent_cap == level["eligible_actions"]
        assert got.attempted_actions == level["attempted"]
        assert got.invalid_structural_actions == level["invalid"]
        assert got.duplicate_speculative_successors == level["duplicates"]
        assert search.last_children() == [(c[0], c[1], tuple(c[3])) for c in level["children"]]
        assert search.topo.gate.tolist() == [c[4] for c in level["children"]]
        live = g[f"live_{step}"]
        s = live.shape[1]
        assert np.array_equal(search.live[:, :s].cpu().numpy(), live)
        assert not search.live[:, s:].any()
        assert np.array_equal(search.types[:, :s].cpu().numpy(), g[f"types_{step}"])
        got_states = search.states[:, :s].float().cpu().numpy() * live[..., None]
        np.testing.assert_allclose(got_states, g[f"states_{step}"] * live[..., None],
                                   rtol=1e-4, atol=1e-4)

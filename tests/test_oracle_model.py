"""Pin the oracle model against the reference model's outputs (fp32, CPU)."""
from __future__ import annotations

import numpy as np
import torch

from conftest import load_golden
from graph_rewrite_system_b200 import synthetic
from oracle.candidates import threshold_candidates
from oracle.model import OracleModel, parameter_shapes

TOL = dict(rtol=2e-5, atol=2e-5)


def golden_model():
    g = load_golden("model_cpu_equivalence.npz")
    rules, cfg = synthetic.small_rules(), synthetic.CPU_EQUIVALENCE_MODEL
    params = synthetic.deterministic_parameters(parameter_shapes(cfg, rules), int(g["seed"]))
    model = OracleModel({k: torch.from_numpy(v) for k, v in params.items()}, rules, cfg)
    batch = {k[len("batch_"):]: torch.from_numpy(v) for k, v in g.items() if k.startswith("batch_")}
    return g, model, batch


def test_oracle_encode_matches_reference():
    g, model, batch = golden_model()
    states, live, types = model.encode(batch)
    np.testing.assert_allclose(states.numpy(), g["encode_states"], **TOL)
    assert np.array_equal(live.numpy(), g["encode_live"])
    assert np.array_equal(types.numpy(), g["encode_types"])


def test_oracle_stepwise_decode_readout_logits():
    g, model, batch = golden_model()
    states, live, types = model.initial_state(batch["initial_types"], batch["edge_batch"],
                                              batch["edge_src"], batch["edge_dst"],
                                              batch["edge_relation"])
    np.testing.assert_allclose(states.numpy(), g["initial_states"], **TOL)
    past_k = past_v = None
    tokens, rks, rvs = [], [], []
    for a in range(batch["action_xfers"].shape[1]):
        states, live, types, nk, nv, token = model.advance(
            states, live, types, past_k, past_v, a, xfer_ids=batch["action_xfers"][:, a],
            source_ids=batch["action_sources"][:, a], source_slots=batch["binding_slots"][:, a],
            destination_slots=batch["destination_slots"][:, a],
            destination_types=batch["destination_types"][:, a])
        np.testing.assert_allclose(token.numpy(), g["advance_tokens"][a], **TOL)
        np.testing.assert_allclose(nk[0].numpy(), g["advance_keys_layer0"][a], **TOL)
        past_k = nk.unsqueeze(3) if past_k is None else torch.cat((past_k, nk.unsqueeze(3)), 3)
        past_v = nv.unsqueeze(3) if past_v is None else torch.cat((past_v, nv.unsqueeze(3)), 3)
        rk, rv = model.project_readout_kv(token)
        rks.append(rk)
        rvs.append(rv)
    np.testing.assert_allclose(states.numpy(), g["advance_states"], **TOL)
    assert np.array_equal(live.numpy(), g["advance_live"])
    assert np.array_equal(types.numpy(), g["advance_types"])
    hk = torch.stack(rks, 2)
    hv = torch.stack(rvs, 2)
    lengths = torch.full((states.shape[0],), hk.shape[2])
    readout = model.fuse_action_history(states, live, hk, hv, lengths)
    readout = model.fuse_readout_graph(readout, live, batch["current_edge_batch"],
                                       batch["current_edge_src"], batch["current_edge_dst"],
                                       batch["current_edge_relation"])
    np.testing.assert_allclose(readout.numpy(), g["readout_states"], **TOL)
    logits, eligible = model.match_logits(readout, live, types)
    np.testing.assert_allclose(logits.numpy(), g["logits"], **TOL)
    assert np.array_equal(eligible.numpy(), g["eligible"])


def test_oracle_structural_decode_and_candidates():
    g, model, batch = golden_model()
    types = torch.from_numpy(g["advance_types"])
    live = torch.from_numpy(g["advance_live"])
    edges = (batch["current_edge_batch"], batch["current_edge_src"], batch["current_edge_dst"],
             batch["current_edge_relation"])
    bindings, valid = model.structural_decode(
        types, live, edges, torch.from_numpy(g["decode_batch"]),
        torch.from_numpy(g["decode_sources"]), torch.from_numpy(g["decode_anchors"]))
    assert np.array_equal(bindings.numpy(), g["decode_bindings"])
    assert np.array_equal(valid.numpy(), g["decode_valid"])
    assert valid.any() and (~valid).any()
    cand = threshold_candidates(model, types, live, batch["current_rewrite_distance"], edges,
                                torch.from_numpy(g["logits"]), torch.from_numpy(g["eligible"]),
                                synthetic.SELECT_ALL_THRESHOLDS, max_candidates_per_state=24)
    for k in ("batch_ids", "sources", "anchors", "bindings"):
        assert np.array_equal(cand[k].numpy(), g["candidates_" + k]), k
    np.testing.assert_allclose(cand["probabilities"].numpy(), g["candidates_probabilities"], **TOL)

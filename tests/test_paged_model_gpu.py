"""CUDA paged model vs the reference model's recorded outputs.

fp32 (the CPU-equivalence configuration): within 2e-5, the reference's own
full-prefix vs paged tolerance (test_paged_model.py:167-171).  bf16: relative
Frobenius error within 2e-2 against the same fp32 reference values.
"""
from __future__ import annotations

import numpy as np
import pytest
import torch

from conftest import load_golden

pytestmark = pytest.mark.gpu

TOL = dict(rtol=2e-5, atol=2e-5)


def build_model(dev, dtype, rules, cfg, seed):
    from graph_rewrite_system_b200.paged_model import PagedActionBindingModel
    from graph_rewrite_system_b200.synthetic import deterministic_parameters
    from oracle.model import parameter_shapes

    model = PagedActionBindingModel(
        rules, num_xfers=rules.num_xfers, width=cfg.width, retrieval_width=cfg.retrieval_width,
        graph_layers=cfg.graph_layers, action_layers=cfg.action_layers,
        action_heads=cfg.action_heads, max_sequence_length=cfg.max_sequence_length,
        readout_graph_layers=cfg.readout_graph_layers, dropout=0.0, compute_dtype=dtype)
    state = model.state_dict()
    params = deterministic_parameters(parameter_shapes(cfg, rules), seed)
    assert {n for n, _ in model.named_parameters()} == set(params)
    for k, v in params.items():
        state[k] = torch.from_numpy(v)
    model.load_state_dict(state)
    return model.to(dev).eval()


def run_golden(dev, dtype):
    from graph_rewrite_system_b200 import synthetic
    from graph_rewrite_system_b200.paged_cache import PagedKVCache

    g = load_golden("model_cpu_equivalence.npz")
    rules, cfg = synthetic.small_rules(), synthetic.CPU_EQUIVALENCE_MODEL
    model = build_model(dev, dtype, rules, cfg, int(g["seed"]))
    batch = {k[len("batch_"):]: torch.from_numpy(v).to(dev) for k, v in g.items()
             if k.startswith("batch_")}
    out = {}
    states, live, types = model.initialize_incremental(batch)
    out["initial_states"] = states
    beams = states.shape[0]
    arena = PagedKVCache(layers=cfg.action_layers, capacity=64, page_size=4,
                         heads=cfg.action_heads, head_width=cfg.width // cfg.action_heads,
                         model_width=cfg.width, device=dev, dtype=dtype)
    handles = [arena.empty_handle()] * beams
    tokens, keys0 = [], []
    for a in range(batch["action_xfers"].shape[1]):
        table, lengths = arena.block_table(handles)
        states, live, types, nk, nv, action, _ = model.advance_incremental(
            states, live, types, xfer_ids=batch["action_xfers"][:, a],
            source_ids=batch["action_sources"][:, a], source_slots=batch["binding_slots"][:, a],
            destination_slots=batch["destination_slots"][:, a],
            destination_types=batch["destination_types"][:, a], paged_key_cache=arena.keys,
            paged_value_cache=arena.values, block_table=table, past_lengths=lengths)
        rk, rv = model.project_action_readout_kv(action)
        new = arena.append_batch(handles, nk, nv, action, rk, rv)
        for h in handles:
            arena.release(h)
        handles = new
        tokens.append(action)
        keys0.append(nk[0])
    out["advance_tokens"] = torch.stack(tokens)
    out["advance_keys_layer0"] = torch.stack(keys0)
    out["advance_states"], out["advance_live"], out["advance_types"] = states, live, types
    table, lengths = arena.block_table(handles)
    readout, _, _ = model.readout_incremental(
        states, live, types, batch=batch, readout_key_cache=arena.readout_keys,
        readout_value_cache=arena.readout_values, block_table=table, lengths=lengths)
    out["readout_states"] = readout
    out["logits"], out["eligible"] = model.match_logits(readout, live, types)
    for h in handles:
        arena.release(h)
    assert arena.allocated_pages == 0
    return g, out


def test_paged_model_fp32_matches_reference(cuda_device):
    g, out = run_golden(cuda_device, torch.float32)
    for key in ("initial_states", "advance_tokens", "advance_keys_layer0", "advance_states",
                "readout_states", "logits"):
        np.testing.assert_allclose(out[key].float().cpu().numpy(), g[key], err_msg=key, **TOL)
    for key in ("advance_live", "advance_types", "eligible"):
        assert np.array_equal(out[key].cpu().numpy(), g[key]), key


def _rel(a, b):
    a = a.float().cpu().numpy().astype(np.float64)
    return np.linalg.norm(a - b) / max(np.linalg.norm(b), 1e-12)


def test_paged_model_bf16_within_tolerance(cuda_device):
    g, out = run_golden(cuda_device, torch.bfloat16)
    for key in ("initial_states", "advance_tokens", "advance_keys_layer0", "advance_states",
                "readout_states"):
        assert _rel(out[key], g[key]) < 2e-2, (key, _rel(out[key], g[key]))
    eligible = g["eligible"]
    logits = out["logits"].cpu().numpy()
    assert np.array_equal(out["eligible"].cpu().numpy(), eligible)
    assert np.linalg.norm(logits[eligible] - g["logits"][eligible]) / \
        np.linalg.norm(g["logits"][eligible]) < 2e-2
    for key in ("advance_live", "advance_types"):
        assert np.array_equal(out[key].cpu().numpy(), g[key]), key


def test_structural_decode_and_candidates_match_reference(cuda_device):
    from graph_rewrite_system_b200 import synthetic
    from graph_rewrite_system_b200.threshold_inference import threshold_candidate_tensors

    g = load_golden("model_cpu_equivalence.npz")
    rules, cfg = synthetic.small_rules(), synthetic.CPU_EQUIVALENCE_MODEL
    model = build_model(cuda_device, torch.float32, rules, cfg, int(g["seed"]))
    batch = {k[len("batch_"):]: torch.from_numpy(v).to(cuda_device) for k, v in g.items()
             if k.startswith("batch_")}
    types = torch.from_numpy(g["advance_types"]).to(cuda_device)
    live = torch.from_numpy(g["advance_live"]).to(cuda_device)
    d = lambda k: torch.from_numpy(g[k]).to(cuda_device)
    bindings, valid = model.structural_decode(batch, types, live, d("decode_batch"),
                                              d("decode_sources"), d("decode_anchors"))
    assert np.array_equal(bindings.cpu().numpy(), g["decode_bindings"])
    assert np.array_equal(valid.cpu().numpy(), g["decode_valid"])
    cand = threshold_candidate_tensors(model, batch, d("logits"), d("eligible"),
                                       synthetic.SELECT_ALL_THRESHOLDS,
                                       max_candidates_per_state=24)
    for k in ("batch_ids", "sources", "anchors", "bindings"):
        assert np.array_equal(getattr(cand, k).cpu().numpy(), g["candidates_" + k]), k
    np.testing.assert_allclose(cand.probabilities.cpu().numpy(), g["candidates_probabilities"],
                               rtol=1e-6, atol=1e-7)


@pytest.mark.parametrize("k,s,ns", [(1, 97, 13), (7, 97, 13), (80, 97, 13), (500, 97, 13),
                                    (7, 96, 31), (500, 96, 31), (2048, 96, 31)])
def test_select_candidates_topk_with_ties(cuda_device, k, s, ns):
    """Random bf16-rounded logits (many exact ties) vs the oracle's stable order;
    96 x 31 items per row take the 8-item vector loads of the first pass."""
    from graph_rewrite_system_b200 import kernels as K
    from graph_rewrite_system_b200.synthetic import SELECT_ALL_THRESHOLDS

    gen = torch.Generator().manual_seed(k + s)
    b = 6
    logits = torch.randn(b, s, ns, generator=gen).bfloat16().float()
    eligible = torch.rand(b, s, ns, generator=gen) > 0.4
    eligible[2] = False
    logits = logits.masked_fill(~eligible, -1e4)
    distance = torch.randint(0, 6, (b, s), generator=gen, dtype=torch.int32)
    flat = logits.flatten(1).masked_fill(~eligible.flatten(1), -torch.inf)
    order = torch.argsort(flat, dim=1, descending=True, stable=True)[:, :k]
    scores = torch.gather(flat, 1, order)
    dev = cuda_device
    n = b * k
    outs = [torch.empty(n, device=dev, dtype=torch.int64) for _ in range(3)]
    prob = torch.empty(n, device=dev)
    K.select_candidates(logits.to(dev), eligible.to(dev), distance.to(dev), k,
                        SELECT_ALL_THRESHOLDS["groups"], *outs, prob)
    _, src, anc = (o.cpu().view(b, k) for o in outs)
    present = scores.isfinite()
    assert torch.equal(src >= 0, present)
    assert torch.equal(anc[present] * ns + src[present], order[present])
    np.testing.assert_allclose(prob.cpu().view(b, k)[present].numpy(),
                               scores[present].sigmoid().numpy(), rtol=1e-6)

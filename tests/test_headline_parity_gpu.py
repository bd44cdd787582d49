"""Parity at the rollout model's own shape: the bf16 device model against the
fp32 oracle on the same beam states.

The model is the rollout workload's (width 256, 8 heads x 32, 4 causal
layers, 4 readout graph layers, seeded random weights, bf16) on the 6-qubit
259-gate synthetic circuit, beam 64, so a level's per-slot GEMMs have
B x S >= 4096 rows; every projection runs on the tcgen05 GEMMs (plain and
LayerNorm epilogues, the fused graph-layer MLP, the match-logits GEMM: the
test checks that each ran).  After
three levels of the device search:

* one-token advance of level 3: the children's next states from the
  parents' level-2 states and cached K/V (paged_model.py:444-613) vs the
  oracle's dense-history advance;
* node readout over the paged readout K/V plus the readout graph
  (paged_model.py:615-655), match logits (model.py:375-389) vs the oracle;
* per-state top-80 candidates with structural decode
  (threshold_inference.py:208-297): every candidate whose oracle score is
  clear of the 80th score by more than the measured logit error is selected
  on both sides with identical bindings.

bf16 tolerance: 2e-2 relative (Frobenius norm of the difference over the
norm of the fp32 oracle values, and per element against the row scale).
"""
from __future__ import annotations

import pytest
import torch

pytestmark = pytest.mark.gpu

TOL = 2e-2


def _rel(a: torch.Tensor, b: torch.Tensor) -> float:
    a, b = a.double(), b.double()
    return float((a - b).norm() / b.norm().clamp_min(1e-12))


def _assert_close_rows(a: torch.Tensor, b: torch.Tensor, what: str) -> None:
    """Frobenius-relative error <= TOL and every element within TOL of the
    oracle row's RMS (or of its own magnitude)."""
    assert _rel(a, b) < TOL, (what, _rel(a, b))
    a, b = a.double(), b.double()
    scale = b.pow(2).mean(-1, keepdim=True).sqrt().clamp_min(1e-6)
    err = (a - b).abs() / torch.maximum(scale, b.abs())
    assert float(err.max()) < 4 * TOL, (what, float(err.max()))


def _edges(topo):
    from oracle.device_views import port_edges

    return port_edges(topo.out_node, topo.out_port)


def _dense_history(pages, table, lengths):
    from oracle.device_views import dense_history

    return dense_history(pages, table, lengths)


@pytest.fixture(scope="module")
def rollout(cuda_device):
    import bench
    from graph_rewrite_system_b200 import kernels as K
    from graph_rewrite_system_b200 import synthetic
    from oracle.model import OracleModel

    search, rc = bench.build_rollout(cuda_device, beam_size=64, depth=3)
    rules, cfg = synthetic.synthetic_rules(), synthetic.ROLLOUT_MODEL
    params = synthetic.deterministic_parameters(synthetic.parameter_shapes(cfg, rules), 0)
    oracle = OracleModel({k: torch.from_numpy(v) for k, v in params.items()}, rules, cfg)
    names = ("gemm", "gemm_layernorm", "graph_mlp", "match_logits_gemm")
    calls = dict.fromkeys(names, 0)
    originals = {n: getattr(K, n) for n in names}

    def counting(name):
        def call(*a, **kw):
            calls[name] += 1
            return originals[name](*a, **kw)
        return call

    for n in names:
        setattr(K, n, counting(n))
    try:
        search.reset()
        for _ in range(2):
            assert search.step() is not None
        # the parents of level 3 as the oracle needs them (their pages are
        # released by level 3's step)
        cache = search.cache
        parents = dict(states=search.states.float().cpu(), live=search.live.cpu(),
                       types=search.types.cpu(),
                       keys=_dense_history(cache.keys, search.block_table, search.lengths),
                       values=_dense_history(cache.values, search.block_table, search.lengths),
                       depth=search.depth)
        assert search.step() is not None
        search.check()
    finally:
        for n in names:
            setattr(K, n, originals[n])
    assert search.beams * search.slots >= 4096
    assert all(calls[n] > 0 for n in names), calls
    return search, oracle, rules, parents


def test_advance_matches_oracle_at_rollout_shape(rollout):
    search, oracle, rules, parents = rollout
    a_parent, a_xfer, a_src, a_dst = (t.cpu() for t in search.last_actions)
    n = a_parent.numel()
    s_new = search.slots
    states = parents["states"][a_parent]
    live, types = parents["live"][a_parent], parents["types"][a_parent]
    pad = s_new - states.shape[1]
    states = torch.nn.functional.pad(states, (0, 0, 0, pad))
    live = torch.nn.functional.pad(live, (0, pad), value=False)
    types = torch.nn.functional.pad(types, (0, pad), value=-1)
    sources = torch.tensor([rules.xfer_to_source[x] for x in a_xfer.tolist()])
    dst_types = torch.full_like(a_dst, -1)
    for i, x in enumerate(a_xfer.tolist()):
        d = rules.destination_gate_types[x]
        dst_types[i, : len(d)] = torch.tensor(d, dtype=torch.long)
    dst_types[a_dst < 0] = -1
    past_k = parents["keys"][:, a_parent]
    past_v = parents["values"][:, a_parent]
    with torch.no_grad():
        exp_states, exp_live, exp_types, _, _, _ = oracle.advance(
            states, live, types, past_k, past_v, parents["depth"], xfer_ids=a_xfer,
            source_ids=sources, source_slots=a_src, destination_slots=a_dst,
            destination_types=dst_types)
    got = search.states.float().cpu()
    assert got.shape == exp_states.shape == (n, s_new, oracle.width)
    assert torch.equal(search.live.cpu(), exp_live)
    assert torch.equal(search.types.cpu(), exp_types)
    _assert_close_rows(got[exp_live], exp_states[exp_live], "advance states")


def test_readout_logits_candidates_match_oracle_at_rollout_shape(rollout):
    from graph_rewrite_system_b200 import synthetic
    from graph_rewrite_system_b200.threshold_inference import select_candidates_device
    from oracle.candidates import threshold_candidates

    search, oracle, rules, _ = rollout
    model, cache, topo = search.model, search.cache, search.topo
    with torch.no_grad():
        readout, _, _ = model.readout_incremental(
            search.states, search.live, search.types, readout_key_cache=cache.readout_keys,
            readout_value_cache=cache.readout_values, block_table=search.block_table,
            lengths=search.lengths, ports=topo.ports())
        logits, eligible = model.match_logits(readout, search.live, search.types)
        k = 80
        cand = select_candidates_device(model, search.types, search.live, topo.ports(),
                                        topo.distance, logits, eligible,
                                        synthetic.SELECT_ALL_THRESHOLDS, k)
        torch.cuda.synchronize()
        states = search.states.float().cpu()
        live, types = search.live.cpu(), search.types.cpu()
        hk = _dense_history(cache.readout_keys, search.block_table, search.lengths)
        hv = _dense_history(cache.readout_values, search.block_table, search.lengths)
        lengths = search.lengths.long().cpu()
        edges = _edges(topo)
        exp = oracle.fuse_action_history(states, live, hk, hv, lengths)
        exp = oracle.fuse_readout_graph(exp, live, *edges)
        exp_logits, exp_eligible = oracle.match_logits(exp, live, types)
        distance = topo.distance.long().cpu()
        exp_cand = threshold_candidates(oracle, types, live, distance, edges, exp_logits,
                                        exp_eligible, synthetic.SELECT_ALL_THRESHOLDS,
                                        max_candidates_per_state=k)
    got = readout.float().cpu()
    _assert_close_rows(got[live], exp[live], "readout")
    assert torch.equal(eligible.cpu(), exp_eligible)
    got_logits = logits.cpu()
    e = exp_eligible
    assert _rel(got_logits[e], exp_logits[e]) < TOL
    err = (got_logits[e] - exp_logits[e]).abs()
    assert float(err.max()) < TOL * max(1.0, float(exp_logits[e].abs().max()))

    # candidates: clear of the k-th oracle score by more than the logit error
    margin = max(4 * float(err.max()), 1e-3)
    ns = oracle.num_sources
    b = types.shape[0]
    flat = exp_logits.flatten(1).masked_fill(~e.flatten(1), -torch.inf)
    kth = torch.sort(flat, 1, descending=True).values[:, min(k, flat.shape[1]) - 1]
    keep = cand["sources"].cpu() >= 0
    got_rows = {}
    for bi, so, an, bind, pr in zip(cand["batch_ids"].cpu()[keep].tolist(),
                                    cand["sources"].cpu()[keep].tolist(),
                                    cand["anchors"].cpu()[keep].tolist(),
                                    cand["bindings"].cpu()[keep].tolist(),
                                    cand["probabilities"].cpu()[keep].tolist()):
        got_rows[(bi, an * ns + so)] = (bind, pr)
    exp_rows = {}
    for bi, so, an, bind, pr in zip(exp_cand["batch_ids"].tolist(), exp_cand["sources"].tolist(),
                                    exp_cand["anchors"].tolist(), exp_cand["bindings"].tolist(),
                                    exp_cand["probabilities"].tolist()):
        exp_rows[(bi, an * ns + so)] = (bind, pr)
    clear = 0
    for (bi, pos), (bind, pr) in exp_rows.items():
        if float(flat[bi, pos]) > float(kth[bi]) + margin:
            assert (bi, pos) in got_rows, (bi, pos)
            assert got_rows[(bi, pos)][0] == bind, (bi, pos)
            assert abs(got_rows[(bi, pos)][1] - pr) < TOL
            clear += 1
    for (bi, pos) in got_rows:
        assert float(flat[bi, pos]) >= float(kth[bi]) - margin, (bi, pos)
    # with random weights many scores sit near the 80th: a quarter clear of it
    assert clear >= len(exp_rows) // 4 > 0, (clear, len(exp_rows))
    assert len(got_rows) <= b * k

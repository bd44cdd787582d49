"""The allocation-free proposal ranking entry point, called through the C ABI.

grs_proposals_rank_static exists for callers that cannot allocate device
memory when they rank proposals (a runtime that has reserved all device
memory for its own pool, a foreign-language binding with no access to the
framework's allocator, a loop where a cudaMalloc would stall the device).
Its scratch is a fixed 8 MiB array inside the library.  This test checks it
against the workspace-taking grs_proposals_rank on two calls in a row (the
second call reuses the array the first one left behind) and that inputs too
large for the array are refused.  The file is named to run last.
"""
from __future__ import annotations

import numpy as np
import pytest
import torch

pytestmark = pytest.mark.gpu


def _case(seed, parents, per, device):
    from graph_rewrite_system_b200.synthetic import synthetic_rules

    rules = synthetic_rules()
    rng = np.random.default_rng(seed)
    batch = np.repeat(np.arange(parents), per)
    sources = rng.integers(0, rules.num_sources, batch.size)
    probs = (1 / (1 + np.exp(-rng.integers(-30, 30, batch.size) / 7.0))).astype(np.float32)
    gates = rng.integers(255, 262, parents)
    t = lambda a: torch.from_numpy(np.asarray(a)).to(device)
    return rules, t(batch), t(sources), t(probs), t(gates)


def _call_static(index, batch, sources, probs, gates, cap, global_cap):
    from graph_rewrite_system_b200 import _lib

    dev = batch.device
    i64 = dict(device=dev, dtype=torch.int64)
    rows, xfers, nexts = (torch.full((global_cap,), -7, **i64) for _ in range(3))
    count = torch.full((1,), -7, **i64)
    metrics = torch.full((2,), -7, **i64)
    status = torch.zeros(1, device=dev, dtype=torch.int32)
    bound = sources.numel() * index.max_xfers_per_source
    code = _lib.lib().grs_proposals_rank_static(
        batch.data_ptr(), sources.data_ptr(), probs.data_ptr(), sources.numel(),
        gates.data_ptr(), gates.numel(), index.xfer_offsets.data_ptr(),
        index.xfer_counts.data_ptr(), index.xfer_ids.data_ptr(), index.gate_deltas.data_ptr(),
        index.all_xfer_counts.data_ptr(), index.xfer_counts.numel(), bound, cap, global_cap,
        rows.data_ptr(), xfers.data_ptr(), nexts.data_ptr(), count.data_ptr(),
        metrics.data_ptr(), status.data_ptr(), torch.cuda.current_stream(dev).cuda_stream)
    return code, rows, xfers, nexts, count, metrics, status


def test_static_scratch_matches_workspace_entry_point(cuda_device):
    from graph_rewrite_system_b200.gpu_proposals import GpuRuleIndex, rank_proposals_device

    for seed, parents in ((21, 200), (22, 150)):   # two calls in a row
        rules, batch, sources, probs, gates = _case(seed, parents, 80, cuda_device)
        index = GpuRuleIndex.build(rules.source_to_xfers(), rules.gate_deltas(),
                                   rules.num_sources, 1, cuda_device)
        expected = rank_proposals_device(batch, sources, probs, gates, index,
                                         per_parent_cap=16, global_cap=3000)
        code, rows, xfers, nexts, count, metrics, status = _call_static(
            index, batch, sources, probs, gates, 16, 3000)
        torch.cuda.synchronize()
        assert code == 0
        assert int(status.item()) == 0 and int(expected.status.item()) == 0
        n = int(expected.count.item())
        assert int(count.item()) == n > 0
        assert torch.equal(rows[:n], expected.rows[:n])
        assert torch.equal(xfers[:n], expected.xfer_ids[:n])
        assert torch.equal(nexts[:n], expected.next_gate[:n])
        assert torch.equal(metrics, expected.metrics)


def test_static_scratch_rejects_oversized_inputs(cuda_device):
    from graph_rewrite_system_b200.gpu_proposals import GpuRuleIndex

    rules, batch, sources, probs, gates = _case(23, 1000, 200, cuda_device)
    index = GpuRuleIndex.build(rules.source_to_xfers(), rules.gate_deltas(),
                               rules.num_sources, 1, cuda_device)
    code, *_ = _call_static(index, batch, sources, probs, gates, 16, 100)
    assert code == -9  # GRS_ERR_TOO_LARGE: nothing launched

"""Proposal expansion and bounded ranking with the reference's API.

Mirrors ``gpu_proposals.py``: ``GpuRuleIndex.build(source_to_xfers,
gate_deltas, num_sources, max_gate_increase, device)`` (``:20-50``) and
``build_gpu_proposals(candidates, beam, rule_index, *, per_parent_cap,
global_cap, profile_stages=False) -> (list[Proposal], metrics, timing)``
(``:69-192``).  Expansion, the per-parent cap and the global rank run in
``csrc/proposals.cu``; ``rank_proposals_device`` returns the selected rows as
device tensors for the device-resident search loop, and
``build_gpu_proposals`` performs the one compact device-to-host copy and the
``Proposal`` packing of the reference.
"""
from __future__ import annotations

from dataclasses import dataclass
import time

import torch

from . import _lib
from .types import BeamState, CandidateTensors, Proposal



@dataclass(frozen=True)
class GpuRuleIndex:
    xfer_offsets: torch.Tensor
    xfer_counts: torch.Tensor
    xfer_ids: torch.Tensor
    gate_deltas: torch.Tensor
    all_xfer_counts: torch.Tensor

    @classmethod
    def build(cls, source_to_xfers: dict[int, list[int]], gate_deltas: list[int],
              num_sources: int, max_gate_increase: int, device) -> "GpuRuleIndex":
        allowed, offsets, counts, all_counts = [], [], [], []
        for source in range(num_sources):
            xs = source_to_xfers.get(source, [])
            selected = [x for x in xs if gate_deltas[x] <= max_gate_increase]
            offsets.append(len(allowed))
            allowed.extend(selected)
            counts.append(len(selected))
            all_counts.append(len(xs))
        i32 = dict(device=device, dtype=torch.int32)
        return cls(
            xfer_offsets=torch.tensor(offsets, **i32),
            xfer_counts=torch.tensor(counts, **i32),
            xfer_ids=torch.tensor(allowed or [0], **i32),
            gate_deltas=torch.tensor(gate_deltas, **i32),
            all_xfer_counts=torch.tensor(all_counts, **i32),
        )

    @property
    def max_xfers_per_source(self) -> int:
        if not hasattr(self, "_max_per_source"):
            object.__setattr__(self, "_max_per_source",
                               int(self.xfer_counts.max().item()) if self.xfer_counts.numel() else 0)
        return self._max_per_source


_WORKSPACES: dict[tuple, torch.Tensor] = {}


def _workspace(device, candidates: int, expanded: int) -> torch.Tensor:
    need = int(_lib.lib().grs_proposals_workspace_bytes(candidates, expanded))
    key = (str(device),)
    buf = _WORKSPACES.get(key)
    if buf is None or buf.numel() < need:
        buf = torch.empty(max(need, 1), device=device, dtype=torch.uint8)
        _WORKSPACES[key] = buf
    return buf


@dataclass
class RankedProposals:
    """Device-resident result of the expansion/rank (``count`` valid rows)."""

    rows: torch.Tensor          # int64 [global_cap] candidate row, -1 padded
    xfer_ids: torch.Tensor      # int64 [global_cap]
    next_gate: torch.Tensor     # int64 [global_cap]
    count: torch.Tensor         # int64 [1] (device)
    metrics: torch.Tensor       # int64 [2] predicted, eligible (device)
    status: torch.Tensor        # int32 [1]


def rank_proposals_device(batch_ids: torch.Tensor, sources: torch.Tensor,
                          probabilities: torch.Tensor, parent_gate_counts: torch.Tensor,
                          rule_index: GpuRuleIndex, *, per_parent_cap: int,
                          global_cap: int, status: torch.Tensor | None = None) -> RankedProposals:
    _lib.require_cuda(batch_ids, sources, probabilities, parent_gate_counts)
    device = sources.device
    c = sources.numel()
    expanded_bound = c * max(1, rule_index.max_xfers_per_source)
    ws = _workspace(device, c, expanded_bound)
    i64 = dict(device=device, dtype=torch.int64)
    rows = torch.empty(max(global_cap, 0), **i64)
    xfers = torch.empty_like(rows)
    nexts = torch.empty_like(rows)
    count = torch.empty(1, **i64)
    metrics = torch.empty(2, **i64)
    if status is None:
        status = torch.zeros(1, device=device, dtype=torch.int32)
    batch_ids = batch_ids.to(torch.int64).contiguous()
    sources = sources.to(torch.int64).contiguous()
    probabilities = probabilities.to(torch.float32).contiguous()
    parent_gate_counts = parent_gate_counts.to(torch.int64).contiguous()
    _lib.check(_lib.lib().grs_proposals_rank(
        batch_ids.data_ptr(), sources.data_ptr(), probabilities.data_ptr(), c,
        parent_gate_counts.data_ptr(), parent_gate_counts.numel(),
        rule_index.xfer_offsets.data_ptr(), rule_index.xfer_counts.data_ptr(),
        rule_index.xfer_ids.data_ptr(), rule_index.gate_deltas.data_ptr(),
        rule_index.all_xfer_counts.data_ptr(), rule_index.xfer_counts.numel(),
        expanded_bound, per_parent_cap, global_cap, rows.data_ptr(), xfers.data_ptr(),
        nexts.data_ptr(), count.data_ptr(), metrics.data_ptr(), ws.data_ptr(), ws.numel(),
        status.data_ptr(), torch.cuda.current_stream(device).cuda_stream), "build_gpu_proposals")
    return RankedProposals(rows, xfers, nexts, count, metrics, status)


@torch.no_grad()
def build_gpu_proposals(candidates: CandidateTensors, beam: list[BeamState],
                        rule_index: GpuRuleIndex, *, per_parent_cap: int, global_cap: int,
                        profile_stages: bool = False):
    """Expand, cap and globally rank actions before one compact D2H copy."""
    device = candidates.sources.device
    timing: dict[str, float] = {}
    started = time.perf_counter()
    parent_gates = torch.tensor([s.gate_count for s in beam], device=device, dtype=torch.int64)
    ranked = rank_proposals_device(candidates.batch_ids, candidates.sources,
                                   candidates.probabilities, parent_gates, rule_index,
                                   per_parent_cap=per_parent_cap, global_cap=global_cap)
    if profile_stages:
        torch.cuda.synchronize(device)
        timing["gpu_proposal_rank_seconds"] = time.perf_counter() - started
    started = time.perf_counter()
    code = int(ranked.status.item())
    if code:
        _lib.check(code, "build_gpu_proposals")
    count = int(ranked.count.item())
    predicted, eligible = ranked.metrics.tolist()
    rows = ranked.rows[:count]
    metadata = torch.stack((candidates.batch_ids[rows].long(), ranked.xfer_ids[:count],
                            candidates.anchors[rows].long(), ranked.next_gate[:count]), 1).cpu()
    bindings = candidates.bindings[rows].cpu()
    probabilities = candidates.probabilities[rows].float().cpu()
    proposals = []
    for row, binding, probability in zip(metadata.tolist(), bindings.tolist(),
                                         probabilities.tolist()):
        parent, xfer_id, anchor, next_gate = row
        proposals.append(Proposal(parent=parent, xfer_id=xfer_id, anchor_slot=anchor,
                                  binding=tuple(s for s in binding if s >= 0),
                                  probability=probability, next_gate_count=next_gate))
    if profile_stages:
        timing["proposal_device_to_host_and_pack_seconds"] = time.perf_counter() - started
    return proposals, {"predicted_actions": int(predicted), "eligible_actions": int(eligible)}, timing


# Largest per-parent cap (and per-parent expansion) of the grouped ranking:
# one parent's expanded actions sit in shared memory (include/grs_b200.h).
GROUPED_MAX_EXPANSION = 4096


def rank_proposals_grouped(sources: torch.Tensor, probabilities: torch.Tensor, k: int,
                           parent_gate_counts: torch.Tensor, rule_index: GpuRuleIndex, *,
                           per_parent_cap: int, global_cap: int,
                           status: torch.Tensor | None = None) -> RankedProposals:
    """Same result as ``rank_proposals_device`` for candidates laid out
    [parents, k] (parent b owns rows b*k..b*k+k-1, absent rows have source
    -1), with the per-parent cap taken per parent in shared memory."""
    _lib.require_cuda(sources, probabilities, parent_gate_counts)
    device = sources.device
    parents = parent_gate_counts.numel()
    if sources.numel() != parents * k:
        raise ValueError("grouped candidates must be [parents * k]")
    need = int(_lib.lib().grs_proposals_grouped_workspace_bytes(parents, per_parent_cap))
    key = (str(device), "grouped")
    ws = _WORKSPACES.get(key)
    if ws is None or ws.numel() < need:
        ws = torch.empty(max(need, 1), device=device, dtype=torch.uint8)
        _WORKSPACES[key] = ws
    i64 = dict(device=device, dtype=torch.int64)
    rows = torch.empty(max(global_cap, 0), **i64)
    xfers = torch.empty_like(rows)
    nexts = torch.empty_like(rows)
    count = torch.empty(1, **i64)
    metrics = torch.empty(2, **i64)
    if status is None:
        status = torch.zeros(1, device=device, dtype=torch.int32)
    _lib.check(_lib.lib().grs_proposals_rank_grouped(
        sources.to(torch.int64).contiguous().data_ptr(),
        probabilities.to(torch.float32).contiguous().data_ptr(), parents, k,
        parent_gate_counts.to(torch.int64).contiguous().data_ptr(),
        rule_index.xfer_offsets.data_ptr(), rule_index.xfer_counts.data_ptr(),
        rule_index.xfer_ids.data_ptr(), rule_index.gate_deltas.data_ptr(),
        rule_index.all_xfer_counts.data_ptr(), rule_index.xfer_counts.numel(), per_parent_cap,
        global_cap, rows.data_ptr(), xfers.data_ptr(), nexts.data_ptr(), count.data_ptr(),
        metrics.data_ptr(), ws.data_ptr(), ws.numel(), status.data_ptr(),
        torch.cuda.current_stream(device).cuda_stream), "rank_proposals_grouped")
    return RankedProposals(rows, xfers, nexts, count, metrics, status)


def rank_proposals_exploration(primary: dict, exploration: dict,
                               parent_gate_counts: torch.Tensor, rule_index: GpuRuleIndex, *,
                               per_parent_cap: int, exploration_per_parent: int,
                               global_cap: int, status: torch.Tensor | None = None):
    """Proposals from a primary and an exploration model's candidates with a
    per-parent exploration quota (build_legacy_proposals,
    paged_rollout_benchmark.py:101-210), on the device.  `primary` and
    `exploration` are candidate dicts (batch_ids, sources, anchors,
    probabilities; source -1 marks an absent row).  Returns
    (RankedProposals whose rows index the concatenated candidate table
    [primary rows | exploration rows], metrics int64 [5]: primary predicted,
    primary eligible, exploration predicted, exploration eligible, selected
    exploration proposals)."""
    device = primary["sources"].device
    cat = lambda k, dt: torch.cat((primary[k], exploration[k])).to(dt).contiguous()
    batch_ids, sources = cat("batch_ids", torch.int64), cat("sources", torch.int64)
    anchors, probs = cat("anchors", torch.int64), cat("probabilities", torch.float32)
    _lib.require_cuda(batch_ids, parent_gate_counts)
    c, cp = sources.numel(), primary["sources"].numel()
    parents = parent_gate_counts.numel()
    expanded_bound = c * max(1, rule_index.max_xfers_per_source)
    need = int(_lib.lib().grs_proposals_exploration_workspace_bytes(c, cp, expanded_bound,
                                                                    parents))
    key = (str(device), "exploration")
    ws = _WORKSPACES.get(key)
    if ws is None or ws.numel() < need:
        ws = torch.empty(max(need, 1), device=device, dtype=torch.uint8)
        _WORKSPACES[key] = ws
    i64 = dict(device=device, dtype=torch.int64)
    rows = torch.empty(max(global_cap, 0), **i64)
    xfers = torch.empty_like(rows)
    nexts = torch.empty_like(rows)
    count = torch.empty(1, **i64)
    metrics = torch.empty(5, **i64)
    if status is None:
        status = torch.zeros(1, device=device, dtype=torch.int32)
    _lib.check(_lib.lib().grs_proposals_rank_exploration(
        batch_ids.data_ptr(), sources.data_ptr(), anchors.data_ptr(), probs.data_ptr(), c, cp,
        parent_gate_counts.to(torch.int64).contiguous().data_ptr(), parents,
        rule_index.xfer_offsets.data_ptr(), rule_index.xfer_counts.data_ptr(),
        rule_index.xfer_ids.data_ptr(), rule_index.gate_deltas.data_ptr(),
        rule_index.all_xfer_counts.data_ptr(), rule_index.xfer_counts.numel(), expanded_bound,
        per_parent_cap, exploration_per_parent, global_cap, rows.data_ptr(), xfers.data_ptr(),
        nexts.data_ptr(), count.data_ptr(), metrics.data_ptr(), ws.data_ptr(), ws.numel(),
        status.data_ptr(), _lib.current_stream()), "rank_proposals_exploration")
    ranked = RankedProposals(rows, xfers, nexts, count, metrics[:2], status)
    return ranked, metrics

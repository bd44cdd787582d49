"""Candidate selection with the reference's API (threshold_inference.py:208-297).

``threshold_candidate_tensors(model, batch, logits, eligible, config, *,
max_candidates_per_state, batch_offset, timing)`` returns ``CandidateTensors``
of the structurally valid candidates in (beam, rank) order.  Selection and
decoding run in ``csrc/candidates.cu``; ``select_candidates_device`` keeps the
padded [beams * k] layout (invalid rows carry source -1) for the device loop.
"""
from __future__ import annotations

import time

import torch

from . import kernels as K
from .types import CandidateTensors


@torch.no_grad()
def select_candidates_device(model, gate_types, live, ports, distance, logits, eligible, config,
                             k: int):
    """Padded candidates: dict of [B*k] batch_ids/sources/anchors/probabilities
    and [B*k, max_pattern] bindings; rows without a valid candidate have
    source -1."""
    b, s, ns = logits.shape
    dev = logits.device
    k = min(k, s * ns)
    n = b * k
    i64 = dict(device=dev, dtype=torch.int64)
    batch_ids, sources, anchors = (torch.empty(n, **i64) for _ in range(3))
    probs = torch.empty(n, device=dev, dtype=torch.float32)
    K.select_candidates(logits.contiguous(), eligible.contiguous(),
                        distance.to(torch.int32).contiguous(), k, config["groups"], batch_ids,
                        sources, anchors, probs)
    bindings = torch.empty(n, model.max_pattern, **i64)
    valid = torch.empty(n, device=dev, dtype=torch.bool)
    K.structural_decode(gate_types.to(torch.int64).contiguous(), live.contiguous(), ports,
                        model.rule_tables(), batch_ids, sources, anchors, bindings, valid,
                        clear_invalid=True)
    return {"batch_ids": batch_ids, "sources": sources, "anchors": anchors,
            "bindings": bindings, "probabilities": probs, "valid": valid}


@torch.no_grad()
def threshold_candidate_tensors(model, batch: dict, logits: torch.Tensor,
                                eligible: torch.Tensor, config: dict, *,
                                max_candidates_per_state: int = 2048, batch_offset: int = 0,
                                timing: dict[str, float] | None = None) -> CandidateTensors:
    """GPU candidate selection, structural decode and validity filter."""
    started = time.perf_counter()
    types = batch["current_types"]
    b, s = types.shape
    ports = model._ports(batch, b, s, logits.device)
    padded = select_candidates_device(model, types, types.ge(0), ports,
                                      batch["current_rewrite_distance"], logits, eligible, config,
                                      max_candidates_per_state)
    keep = padded["valid"]
    out = CandidateTensors(
        batch_ids=padded["batch_ids"][keep] + batch_offset, sources=padded["sources"][keep],
        anchors=padded["anchors"][keep], bindings=padded["bindings"][keep],
        probabilities=padded["probabilities"][keep])
    if timing is not None:
        torch.cuda.synchronize(logits.device)
        timing["candidate_selection_and_decode_seconds"] = (
            timing.get("candidate_selection_and_decode_seconds", 0.0)
            + time.perf_counter() - started)
    return out

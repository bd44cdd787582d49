"""Value types shared with the reference's hot path.

``BeamState`` and ``Proposal`` follow ``beam_search_benchmark.py:35-61``;
``CandidateTensors`` follows ``threshold_inference.py:11-34``.  The device
search loop keeps beams as tensors; these types exist for the drop-in API.
"""
from __future__ import annotations

from dataclasses import dataclass
from typing import Any

import torch


@dataclass
class BeamState:
    graph: Any
    snapshot: dict | None
    guid_to_slot: dict[int, int]
    next_slot: int
    last_touched: Any
    rewrite_distance: Any
    previous_preferred: set[int]
    local_streak: int
    gate_count: int
    depth: int
    history: tuple
    topology_index: Any = None
    exact_graph_checkpoint: Any = None
    exact_slot_checkpoint: dict[int, int] | None = None
    exact_checkpoint_depth: int = 0


@dataclass(frozen=True)
class Proposal:
    parent: int
    xfer_id: int
    anchor_slot: int
    binding: tuple[int, ...] | None
    probability: float
    next_gate_count: int


@dataclass(frozen=True)
class CandidateTensors:
    batch_ids: torch.Tensor
    sources: torch.Tensor
    anchors: torch.Tensor
    bindings: torch.Tensor
    probabilities: torch.Tensor

    @classmethod
    def cat(cls, chunks: list["CandidateTensors"]) -> "CandidateTensors":
        if not chunks:
            raise ValueError("cannot concatenate an empty candidate list")
        return cls(**{
            name: torch.cat([getattr(chunk, name) for chunk in chunks])
            for name in ("batch_ids", "sources", "anchors", "bindings", "probabilities")
        })

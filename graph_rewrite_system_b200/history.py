"""Beam histories of the device search in the reference's JSONL format.

The reference can dump every search level as one JSON line so an external
exact-refresh / audit step (Quartz replay, not part of this path) can run
off-box: ``serialized_history_state`` and ``append_beam_level``
(paged_rollout_benchmark.py:213-239), written after a metadata line
(:821-835).  The beam stays on the GPU here, so ``BeamHistoryRecorder``
copies each level's children - parent index, xfer id, source and
destination slots, gate count - to the host once per level (one pinned
copy) and rebuilds every beam's action history by following parent links.
The lines are byte-identical to the reference's for the same beam: the same
keys, ``sort_keys=True`` and json's default separators.
"""
from __future__ import annotations

import json
from pathlib import Path
from typing import Iterable, Sequence

import numpy as np

Action = tuple[int, tuple[int, ...], tuple[int, ...]]   # (xfer_id, source slots, destination slots)


def serialized_history_state(gate_count: int, history: Iterable[Action]) -> dict:
    """One beam state as paged_rollout_benchmark.py:213-224 serialises it."""
    return {
        "gate_count": int(gate_count),
        "history": [
            {"xfer_id": int(xfer), "source_slots": [int(s) for s in source],
             "destination_slots": [int(d) for d in destination]}
            for xfer, source, destination in history
        ],
    }


def beam_level_line(depth: int, states: Sequence[tuple[int, Sequence[Action]]]) -> str:
    """The JSONL line of one level (paged_rollout_benchmark.py:227-239);
    `states` are (gate_count, history) pairs in beam order."""
    return json.dumps({"type": "beam_level", "depth": int(depth),
                       "states": [serialized_history_state(g, h) for g, h in states]},
                      sort_keys=True) + "\n"


def metadata_line(initial_snapshot: dict, qasm: str | None = None,
                  initial_qasm: str | None = None) -> str:
    """The first line of a dump (paged_rollout_benchmark.py:821-833); the
    synthetic circuits have no QASM source, so those fields may be null."""
    return json.dumps({"type": "metadata", "qasm": qasm, "initial_qasm": initial_qasm,
                       "initial_snapshot": initial_snapshot}, sort_keys=True) + "\n"


class BeamHistoryRecorder:
    """Host record of a ``DeviceBeamSearch``'s actions, one level at a time.

    Call ``record()`` after every ``search.step()`` that returned a row (and
    ``reset()`` after ``search.reset()``); ``states()`` gives the current
    beam's (gate_count, history) pairs, ``append_beam_level(path)`` writes
    them as the reference's JSONL line."""

    def __init__(self, search):
        if getattr(search, "world", 1) != 1:
            raise NotImplementedError("history export follows parent links within one GPU's "
                                      "beam: record the single-GPU search")
        self.search = search
        self.reset()

    def reset(self) -> None:
        self.levels: list[tuple[np.ndarray, np.ndarray, list, list]] = []
        self.gate_counts = np.asarray(self.search.topo.gate.tolist(), dtype=np.int64)
        self.device_to_host_bytes = 0

    @staticmethod
    def _unpad(rows: np.ndarray) -> list[tuple[int, ...]]:
        return [tuple(int(v) for v in row if v >= 0) for row in rows]

    def record(self) -> None:
        """Copy the last level's children to the host (one synchronisation)."""
        host = self.search.level_actions_host()
        self.device_to_host_bytes += host["nbytes"]
        self.levels.append((host["parent"].numpy().copy(), host["xfer"].numpy().copy(),
                            self._unpad(host["source_slots"].numpy()),
                            self._unpad(host["destination_slots"].numpy())))
        self.gate_counts = host["gate_count"].numpy().copy()

    @property
    def depth(self) -> int:
        return len(self.levels)

    def histories(self) -> list[tuple[Action, ...]]:
        """The action history of every beam of the last recorded level."""
        hist: list[tuple[Action, ...]] = [()]
        for parent, xfer, source, destination in self.levels:
            hist = [hist[p] + ((int(x), s, d),)
                    for p, x, s, d in zip(parent.tolist(), xfer.tolist(), source, destination)]
        return hist

    def states(self) -> list[tuple[int, tuple[Action, ...]]]:
        return list(zip(self.gate_counts.tolist(), self.histories()))

    def append_beam_level(self, path: str | Path, depth: int | None = None) -> None:
        """Append the current beam as one line of the reference's dump."""
        with Path(path).open("a") as stream:
            stream.write(beam_level_line(self.depth if depth is None else depth, self.states()))

"""Device-resident lazy topology of the beam (lazy_rollout_benchmark.py:47-485).

``TopologyState`` holds, for up to ``beams`` rows of ``slots`` slots, the port
arrays, gate types, touch steps, previous-preferred flags, rewrite distances
and the per-beam scalars (next slot, local streak, gate count, fingerprint).
``xfer_table`` packs every xfer's source/destination wire structure for the
planning and materialisation kernels of ``csrc/topology.cu``.
"""
from __future__ import annotations

from dataclasses import dataclass

import numpy as np
import torch

from . import _lib
from .synthetic import RuleMetadata, parse_pattern


TAB_MAXP, TAB_MAXW, TAB_MAXE = 4, 4, 8


def _wires(ops):
    wires: dict[int, list[tuple[int, int]]] = {}
    for index, op in enumerate(ops):
        for port, qubit in enumerate(op.qubits):
            wires.setdefault(qubit, []).append((index, port))
    return wires


def xfer_table(rules: RuleMetadata, device) -> torch.Tensor:
    """int32 [xfers, width]: source/destination lengths, destination types,
    per-wire boundary ops/ports and the destination's internal edges."""
    width = int(_lib.lib().grs_topology_table_width())
    table = np.full((rules.num_xfers, width), -1, np.int32)
    for x in range(rules.num_xfers):
        src = parse_pattern(rules.xfer_sources[x])
        dst = parse_pattern(rules.xfer_destinations[x])
        if len(src) > TAB_MAXP or len(dst) > TAB_MAXP:
            raise ValueError("patterns longer than 4 operations are not supported")
        row = table[x]
        row[0], row[1] = len(src), len(dst)
        for i, op in enumerate(dst):
            row[2 + i] = op.gate_type
        sw, dw = _wires(src), _wires(dst)
        qubits = sorted(set(sw) | set(dw))
        if len(qubits) > TAB_MAXW:
            raise ValueError("patterns on more than 4 qubits are not supported")
        row[6] = len(qubits)
        internal = []
        for w, q in enumerate(qubits):
            base = 7 + 8 * w
            if q in sw:
                (fi, fp), (li, lp) = sw[q][0], sw[q][-1]
                row[base:base + 4] = (fi, fp, li, lp)
            if q in dw:
                (fi, fp), (li, lp) = dw[q][0], dw[q][-1]
                row[base + 4:base + 8] = (fi, fp, li, lp)
                internal += [(a, b, pa, pb) for (a, pa), (b, pb) in zip(dw[q], dw[q][1:])]
        if len(internal) > TAB_MAXE:
            raise ValueError("too many internal destination edges")
        nint = 7 + 8 * TAB_MAXW
        row[nint] = len(internal)
        for e, edge in enumerate(internal):
            row[nint + 1 + 4 * e: nint + 5 + 4 * e] = edge
    return torch.from_numpy(table).to(device)


@dataclass
class TopologyState:
    """Views of one beam generation: [B, S] / [B, S, 4] rows and [B] scalars."""

    types: torch.Tensor          # int64 [B, S], -1 = dead
    out_node: torch.Tensor       # int32 [B, S, 4], -1 = unconnected
    out_port: torch.Tensor
    in_node: torch.Tensor
    in_port: torch.Tensor
    touched: torch.Tensor        # int32 [B, S], -1 = never
    preferred: torch.Tensor      # uint8 [B, S]
    distance: torch.Tensor       # int32 [B, S]
    next_slot: torch.Tensor      # int32 [B]
    streak: torch.Tensor         # int32 [B]
    gate: torch.Tensor           # int64 [B]
    fingerprint: torch.Tensor    # 64-bit fingerprints stored as int64 [B]

    @property
    def slots(self) -> int:
        return self.types.shape[1]

    def ports(self):
        return (self.in_node, self.in_port, self.out_node, self.out_port)


class TopologyBuffers:
    """Flat storage for `beams` rows of up to `slots` slots; ``state(rows,
    slots)`` views it with any row stride up to the capacity."""

    def __init__(self, beams: int, slots: int, device):
        self.beams, self.capacity = beams, slots
        n = beams * slots
        i32 = dict(device=device, dtype=torch.int32)
        self._types = torch.empty(n, device=device, dtype=torch.int64)
        self._ports = [torch.empty(n * 4, **i32) for _ in range(4)]
        self._touched = torch.empty(n, **i32)
        self._preferred = torch.empty(n, device=device, dtype=torch.uint8)
        self._distance = torch.empty(n, **i32)
        self.next_slot = torch.empty(beams, **i32)
        self.streak = torch.empty(beams, **i32)
        self.gate = torch.empty(beams, device=device, dtype=torch.int64)
        self.fingerprint = torch.empty(beams, device=device, dtype=torch.int64)

    def state(self, rows: int, slots: int) -> TopologyState:
        if rows > self.beams or slots > self.capacity:
            raise ValueError("topology buffers too small")
        n = rows * slots
        v = lambda t: t[:n].view(rows, slots)
        p = lambda t: t[: n * 4].view(rows, slots, 4)
        return TopologyState(v(self._types), *(p(t) for t in self._ports), v(self._touched),
                             v(self._preferred), v(self._distance), self.next_slot[:rows],
                             self.streak[:rows], self.gate[:rows], self.fingerprint[:rows])


def initial_topology(buffers: TopologyBuffers, nodes: list[tuple[int, int]], edges,
                     slots: int) -> TopologyState:
    """Row 0 = the s0 circuit (indexed_topology, lazy_rollout_benchmark.py:62-89)."""
    device = buffers.gate.device
    st = buffers.state(1, slots)
    types = np.full((1, slots), -1, np.int64)
    for slot, gate in nodes:
        types[0, slot] = gate
    ports = np.full((4, 1, slots, 4), -1, np.int32)   # out_node, out_port, in_node, in_port
    for s, d, sp, dp in edges:
        ports[0, 0, s, sp], ports[1, 0, s, sp] = d, dp
        ports[2, 0, d, dp], ports[3, 0, d, dp] = s, sp
    st.types.copy_(torch.from_numpy(types))
    for t, a in zip((st.out_node, st.out_port, st.in_node, st.in_port), ports):
        t.copy_(torch.from_numpy(a))
    st.touched.fill_(-1)
    st.preferred.zero_()
    st.distance.fill_(5)
    st.next_slot.fill_(max(s for s, _ in nodes) + 1 if nodes else 0)
    st.streak.zero_()
    st.gate.fill_(len(nodes))
    _lib.check(_lib.lib().grs_topology_fingerprint(
        st.types.data_ptr(), st.out_node.data_ptr(), st.out_port.data_ptr(), st.in_node.data_ptr(),
        st.in_port.data_ptr(), 1, slots, st.fingerprint.data_ptr(),
        torch.cuda.current_stream(device).cuda_stream), "topology_fingerprint")
    return st

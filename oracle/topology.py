"""Oracle of the lazy topology update and the accept/dedup loop (pure Python).

Restates ``lazy_rollout_benchmark.py``: ``indexed_topology`` (``:62-89``),
``plan_indexed_rewrite`` (``:105-211``), ``materialize_indexed_rewrite``
(``:214-270``), ``distance_slots_from_index`` / ``dense_distances_from_index``
(``:306-333``), ``dense_last_touched`` (``:336-352``) and ``lazy_child_indexed``
(``:392-485``), plus the accept loop of ``paged_rollout_benchmark.py:1013-1046``
and the stable record sort of ``:1045``.

Fingerprints: the reference XORs Python ``hash(("node"|"edge", ...))``
components, which are salted per process, so only the accept/duplicate
*decisions* are comparable.  This oracle and the CUDA kernels XOR the same
deterministic 64-bit components (splitmix64 of a packed node or edge key).
"""
from __future__ import annotations

from dataclasses import dataclass, field

import numpy as np

MASK64 = (1 << 64) - 1


def mix64(z: int) -> int:
    """splitmix64 finaliser (Steele, Lea & Flood 2014)."""
    z = (z + 0x9E3779B97F4A7C15) & MASK64
    z = ((z ^ (z >> 30)) * 0xBF58476D1CE4E5B9) & MASK64
    z = ((z ^ (z >> 27)) * 0x94D049BB133111EB) & MASK64
    return z ^ (z >> 31)


def node_component(slot: int, gate: int) -> int:
    return mix64((1 << 62) | (slot << 16) | (gate & 0xFFFF))


def edge_component(src: int, dst: int, sp: int, dp: int) -> int:
    return mix64((2 << 62) | (src << 36) | (dst << 12) | ((sp & 63) << 6) | (dp & 63))


@dataclass
class Topology:
    nodes: dict[int, int]
    out_edge: dict[tuple[int, int], tuple[int, int]]
    in_edge: dict[tuple[int, int], tuple[int, int]]
    fingerprint: int

    @property
    def edges(self) -> set[tuple[int, int, int, int]]:
        return {(s, d, sp, dp) for (s, sp), (d, dp) in self.out_edge.items()}

    def neighbors(self, slot: int):
        for port in range(4):
            if (slot, port) in self.out_edge:
                yield self.out_edge[(slot, port)][0]
            if (slot, port) in self.in_edge:
                yield self.in_edge[(slot, port)][0]


def indexed_topology(nodes: dict[int, int], edges) -> Topology:
    """lazy_rollout_benchmark.py:62-89 (order-independent XOR fingerprint)."""
    out_edge, in_edge = {}, {}
    fp = 0
    for slot, gate in nodes.items():
        fp ^= node_component(slot, gate)
    for s, d, sp, dp in edges:
        out_edge[(s, sp)] = (d, dp)
        in_edge[(d, dp)] = (s, sp)
        fp ^= edge_component(s, d, sp, dp)
    return Topology(dict(nodes), out_edge, in_edge, fp)


def pattern_wires(ops) -> dict[int, list[tuple[int, int]]]:
    wires: dict[int, list[tuple[int, int]]] = {}
    for index, op in enumerate(ops):
        for port, qubit in enumerate(op.qubits):
            wires.setdefault(qubit, []).append((index, port))
    return wires


def plan_rewrite(parent: Topology, source, destination, source_slots, destination_slots):
    """lazy_rollout_benchmark.py:105-211; raises ValueError like the reference."""
    if len(source) != len(source_slots):
        raise ValueError("source pattern/binding length mismatch")
    if len(destination) != len(destination_slots):
        raise ValueError("destination pattern/binding length mismatch")
    removed = set(source_slots)
    if not removed.issubset(parent.nodes):
        raise ValueError("source binding contains a non-live node")
    if any(slot in parent.nodes for slot in destination_slots):
        raise ValueError("destination binding reuses a live slot")
    sw, dw = pattern_wires(source), pattern_wires(destination)
    boundaries = {}
    for qubit, wire in sw.items():
        (fi, fpt), (li, lpt) = wire[0], wire[-1]
        pred = parent.in_edge.get((source_slots[fi], fpt))
        succ = parent.out_edge.get((source_slots[li], lpt))
        if pred is not None and pred[0] in removed:
            pred = None
        if succ is not None and succ[0] in removed:
            succ = None
        boundaries[qubit] = (pred, succ)
    removed_edges = set()
    for slot in removed:
        for port in range(4):
            o = parent.out_edge.get((slot, port))
            if o is not None:
                removed_edges.add((slot, o[0], port, o[1]))
            i = parent.in_edge.get((slot, port))
            if i is not None:
                removed_edges.add((i[0], slot, i[1], port))
    requested = set()
    for qubit in set(sw) | set(dw):
        wire = dw.get(qubit, [])
        pred, succ = boundaries.get(qubit, (None, None))
        if wire:
            for (li, lp), (ri, rp) in zip(wire, wire[1:]):
                requested.add((destination_slots[li], destination_slots[ri], lp, rp))
            (fi, fpt), (la, lpt) = wire[0], wire[-1]
            if pred is not None:
                requested.add((pred[0], destination_slots[fi], pred[1], fpt))
            if succ is not None:
                requested.add((destination_slots[la], succ[0], lpt, succ[1]))
        elif pred is not None and succ is not None:
            requested.add((pred[0], succ[0], pred[1], succ[1]))
    parent_edges = parent.edges
    added = {e for e in requested if e in removed_edges or e not in parent_edges}
    fp = parent.fingerprint
    for slot in source_slots:
        fp ^= node_component(slot, parent.nodes[slot])
    for slot, op in zip(destination_slots, destination):
        fp ^= node_component(slot, op.gate_type)
    for e in removed_edges:
        fp ^= edge_component(*e)
    for e in added:
        fp ^= edge_component(*e)
    return fp, removed_edges, added


def materialize(parent: Topology, destination, source_slots, destination_slots, fp, removed_edges,
                added_edges) -> Topology:
    """lazy_rollout_benchmark.py:214-270."""
    nodes = dict(parent.nodes)
    for slot in source_slots:
        del nodes[slot]
    for slot, op in zip(destination_slots, destination):
        nodes[slot] = op.gate_type
    out_edge, in_edge = dict(parent.out_edge), dict(parent.in_edge)
    for s, d, sp, dp in removed_edges:
        if out_edge.get((s, sp)) == (d, dp):
            del out_edge[(s, sp)]
        if in_edge.get((d, dp)) == (s, sp):
            del in_edge[(d, dp)]
    for s, d, sp, dp in added_edges:
        out_edge[(s, sp)] = (d, dp)
        in_edge[(d, dp)] = (s, sp)
    return Topology(nodes, out_edge, in_edge, fp)


def dense_distances(topology: Topology, core: set[int], slots: int) -> np.ndarray:
    """BFS from the live core; min(d, 4) when reachable, else 5 (:306-333);
    dead slots read 5 (the collation fill, tensorized_batch.py:40)."""
    dist = np.full(slots, -1, np.int64)
    queue = [s for s in sorted(core) if s in topology.nodes]
    for s in queue:
        dist[s] = 0
    cursor = 0
    while cursor < len(queue):
        slot = queue[cursor]
        cursor += 1
        for nb in topology.neighbors(slot):
            if dist[nb] < 0:
                dist[nb] = dist[slot] + 1
                queue.append(nb)
    out = np.full(slots, 5, np.int64)
    for slot in topology.nodes:
        out[slot] = min(dist[slot], 4) if dist[slot] >= 0 else 5
    return out


@dataclass
class BeamNode:
    """The per-beam host state the lazy topology keeps (BeamState fields)."""

    topology: Topology
    next_slot: int
    last_touched: np.ndarray           # dense, -1 = never
    rewrite_distance: np.ndarray       # dense, 5 = far / dead
    previous_preferred: set[int]
    local_streak: int
    gate_count: int
    depth: int
    history: tuple = field(default_factory=tuple)


def initial_beam(nodes: dict[int, int], edges, slots: int) -> BeamNode:
    topo = indexed_topology(nodes, edges)
    next_slot = max(nodes) + 1 if nodes else 0
    return BeamNode(topo, next_slot, np.full(slots, -1, np.int64), np.full(slots, 5, np.int64),
                    set(), 0, len(nodes), 0)


def lazy_child(parent: BeamNode, binding, anchor, xfer_id, next_gate, source, destination,
               seen: set, slots: int):
    """lazy_rollout_benchmark.py:392-485 -> (child | None, fingerprint | None, duplicate)."""
    dest_slots = tuple(range(parent.next_slot, parent.next_slot + len(destination)))
    try:
        fp, removed_edges, added_edges = plan_rewrite(parent.topology, source, destination,
                                                      tuple(binding), dest_slots)
    except ValueError:
        return None, None, False
    if fp in seen:
        return None, fp, True
    child_topo = materialize(parent.topology, destination, binding, dest_slots, fp,
                             removed_edges, added_edges)
    removed = set(binding)
    changed = removed_edges.symmetric_difference(added_edges)
    live = set(child_topo.nodes)
    core = set(dest_slots)
    for s, d, _, _ in changed:
        if s in live:
            core.add(s)
        if d in live:
            core.add(d)
    touched = parent.last_touched.copy()
    for slot in removed:
        touched[slot] = -1
    for slot in core:
        touched[slot] = parent.depth
    preds = set()
    for slot in binding:
        for port in range(4):
            inc = parent.topology.in_edge.get((slot, port))
            if inc is not None:
                preds.add(inc[0])
    preferred = (set(dest_slots) | preds) & live
    streak = parent.local_streak + 1 if anchor in parent.previous_preferred else 0
    if len(child_topo.nodes) != next_gate:
        raise RuntimeError(f"gate delta mismatch: expected {next_gate}, got {len(child_topo.nodes)}")
    child = BeamNode(child_topo, parent.next_slot + len(destination), touched,
                     dense_distances(child_topo, core, slots), preferred, streak, next_gate,
                     parent.depth + 1, parent.history + ((xfer_id, tuple(binding), dest_slots),))
    return child, fp, False


def accept(beam, proposals, sources, destinations, seen: set, beam_size: int, slots: int):
    """The accept loop (paged_rollout_benchmark.py:1013-1046) and the stable
    record sort by (gate_count, len(history)).  proposals: list of tuples
    (parent, xfer, anchor, binding, next_gate).  Returns (records, metrics)
    where records = [(child, proposal_index)]."""
    records = []
    attempted = invalid = duplicates = 0
    for index, (parent, xfer, anchor, binding, next_gate) in enumerate(proposals):
        if len(records) >= beam_size:
            break
        attempted += 1
        child, fp, dup = lazy_child(beam[parent], binding, anchor, xfer, next_gate,
                                    sources[xfer], destinations[xfer], seen, slots)
        if dup:
            duplicates += 1
            continue
        if child is None:
            invalid += 1
            continue
        seen.add(fp)
        records.append((child, index))
    records.sort(key=lambda r: (r[0].gate_count, len(r[0].history)))
    return records[:beam_size], {"attempted": attempted, "invalid": invalid,
                                 "duplicates": duplicates}

"""Seeded synthetic workloads for the beam-search decode path.

The reference searches the Quartz ``hwb6`` circuit with the Nam ECC rule set
and a trained checkpoint; none of those ship with it.  This module builds
seeded stand-ins with the same shapes and value distributions:

* a rule set written as Quartz-style pattern strings over
  {h, x, cx, t, tdg, s, sdg, rz} (gate ids follow ``dataset.py:13-47``);
* random circuits drawn uniformly from that gate mix on random wires, as the
  lightweight port graph the reference keeps per beam
  (``beam_search_benchmark.py:81-97``: nodes are gates, an edge joins
  consecutive gates on one wire, ports are qubit positions in the gate);
* model configurations for the CPU equivalence case and the full rollout.

Everything here is plain Python/NumPy with fixed seeds so the same workload
is rebuilt bit-for-bit on any host.
"""
from __future__ import annotations

from dataclasses import dataclass, field
from functools import lru_cache

import numpy as np

# Gate vocabulary of the reference (dataset.py:13-47).  Only the names used by
# the synthetic rule set and circuits are needed, but the ids must agree.
GATE_NAME_TO_ID = {
    "h": 0, "x": 1, "y": 2, "rx": 3, "ry": 4, "rz": 5, "cx": 6, "ccx": 7,
    "add": 8, "neg": 9, "z": 10, "s": 11, "sdg": 12, "t": 13, "tdg": 14,
    "ch": 15, "swap": 16, "p": 17, "pdg": 18, "u1": 19, "u2": 20, "u3": 21,
    "ccz": 22, "cz": 23, "rx1": 24, "rx3": 25, "input_qubit": 26,
    "input_param": 27, "ry1": 28, "ry3": 29, "rxx1": 30, "rxx3": 31, "sx": 32,
}
NUM_GATE_TYPES = 33
MAX_PORTS = 4

CIRCUIT_GATES = ("h", "x", "cx", "t", "tdg", "s", "sdg", "rz")


@dataclass(frozen=True)
class PatternOperation:
    """One gate of a rule pattern: its type id and the pattern qubits it uses."""

    gate_type: int
    qubits: tuple[int, ...]


@lru_cache(maxsize=None)
def parse_pattern(pattern: str) -> tuple[PatternOperation, ...]:
    """Parse ``"cx 0 1; t 0"`` into operations (incremental_graph.py:15-31)."""
    operations = []
    for instruction in pattern.split(";"):
        fields = instruction.strip().split()
        if not fields:
            continue
        if fields[0] not in GATE_NAME_TO_ID:
            raise ValueError(f"unknown gate {fields[0]}")
        operations.append(
            PatternOperation(GATE_NAME_TO_ID[fields[0]], tuple(map(int, fields[1:])))
        )
    return tuple(operations)


def pattern_gate_types(pattern: str, *, allow_empty: bool = False) -> tuple[int, ...]:
    types = tuple(op.gate_type for op in parse_pattern(pattern))
    if not types and not allow_empty:
        raise ValueError("empty pattern")
    return types


@dataclass(frozen=True)
class RuleMetadata:
    """Same fields and meaning as the reference's ``RuleMetadata`` (dataset.py:65-89)."""

    source_patterns: tuple[str, ...]
    source_gate_types: tuple[tuple[int, ...], ...]
    destination_gate_types: tuple[tuple[int, ...], ...]
    xfer_to_source: tuple[int, ...]
    xfer_sources: tuple[str, ...]
    xfer_destinations: tuple[str, ...]
    num_gate_types: int = NUM_GATE_TYPES

    @classmethod
    def from_payload(cls, payload: dict) -> "RuleMetadata":
        return cls(
            source_patterns=tuple(payload["source_patterns"]),
            source_gate_types=tuple(
                pattern_gate_types(p) for p in payload["source_patterns"]
            ),
            destination_gate_types=tuple(
                pattern_gate_types(p, allow_empty=True)
                for p in payload["xfer_destinations"]
            ),
            xfer_to_source=tuple(map(int, payload["xfer_to_source"])),
            xfer_sources=tuple(payload["xfer_sources"]),
            xfer_destinations=tuple(payload["xfer_destinations"]),
        )

    @property
    def num_sources(self) -> int:
        return len(self.source_patterns)

    @property
    def num_xfers(self) -> int:
        return len(self.xfer_to_source)

    def source_to_xfers(self) -> dict[int, list[int]]:
        table: dict[int, list[int]] = {}
        for xfer, source in enumerate(self.xfer_to_source):
            table.setdefault(source, []).append(xfer)
        return table

    def gate_deltas(self) -> list[int]:
        return [
            len(self.destination_gate_types[x])
            - len(self.source_gate_types[self.xfer_to_source[x]])
            for x in range(self.num_xfers)
        ]


# Builder-defined rewrite rules: (source pattern, [destination patterns]).
# Cancellations, merges, commutations and expansions over the circuit gate
# mix; one expansion has delta +2 so the max-gate-increase filter is exercised.
_RULES: tuple[tuple[str, tuple[str, ...]], ...] = (
    ("h 0; h 0", ("",)),
    ("x 0; x 0", ("",)),
    ("cx 0 1; cx 0 1", ("",)),
    ("t 0; tdg 0", ("",)),
    ("tdg 0; t 0", ("",)),
    ("s 0; sdg 0", ("",)),
    ("sdg 0; s 0", ("",)),
    ("t 0; t 0", ("s 0",)),
    ("tdg 0; tdg 0", ("sdg 0",)),
    ("rz 0; rz 0", ("rz 0",)),
    ("cx 0 1; x 0; cx 0 1", ("x 0; x 1",)),
    ("rz 0; t 0", ("t 0; rz 0",)),
    ("t 0; rz 0", ("rz 0; t 0",)),
    ("t 0; s 0", ("s 0; t 0",)),
    ("s 0; t 0", ("t 0; s 0",)),
    ("cx 0 1; t 0", ("t 0; cx 0 1",)),
    ("t 0; cx 0 1", ("cx 0 1; t 0",)),
    ("cx 0 1; x 1", ("x 1; cx 0 1",)),
    ("x 0; cx 1 0", ("cx 1 0; x 0",)),
    ("cx 0 1; rz 0", ("rz 0; cx 0 1",)),
    ("rz 0; cx 0 1", ("cx 0 1; rz 0",)),
    ("cx 0 1; s 0", ("s 0; cx 0 1",)),
    ("s 0; cx 0 1", ("cx 0 1; s 0",)),
    ("h 0; x 0; h 0", ("x 0; h 0; h 0", "h 0; h 0; x 0")),
    ("t 0", ("s 0; tdg 0", "tdg 0; s 0")),
    ("s 0", ("t 0; t 0",)),
    ("sdg 0", ("tdg 0; tdg 0",)),
    ("x 0", ("x 0; h 0; h 0",)),
    ("cx 0 1; cx 1 0; cx 0 1", ("cx 1 0; cx 0 1; cx 1 0",)),
    ("tdg 0; sdg 0", ("sdg 0; tdg 0",)),
    ("sdg 0; tdg 0", ("tdg 0; sdg 0",)),
)


def synthetic_rules() -> RuleMetadata:
    """The builder-defined rule set used by every synthetic workload."""
    source_patterns = []
    xfer_to_source = []
    xfer_sources = []
    xfer_destinations = []
    for source_id, (source, destinations) in enumerate(_RULES):
        source_patterns.append(source)
        for destination in destinations:
            xfer_to_source.append(source_id)
            xfer_sources.append(source)
            xfer_destinations.append(destination)
    return RuleMetadata.from_payload(
        {
            "source_patterns": source_patterns,
            "xfer_to_source": xfer_to_source,
            "xfer_sources": xfer_sources,
            "xfer_destinations": xfer_destinations,
        }
    )


def small_rules() -> RuleMetadata:
    """A 6-source subset over an 8-type vocabulary (the CPU equivalence case)."""
    keep = [0, 2, 7, 15, 24, 10]
    source_patterns, xfer_to_source, xfer_sources, xfer_destinations = [], [], [], []
    for new_id, index in enumerate(keep):
        source, destinations = _RULES[index]
        source_patterns.append(source)
        for destination in destinations:
            xfer_to_source.append(new_id)
            xfer_sources.append(source)
            xfer_destinations.append(destination)
    return RuleMetadata.from_payload(
        {
            "source_patterns": source_patterns,
            "xfer_to_source": xfer_to_source,
            "xfer_sources": xfer_sources,
            "xfer_destinations": xfer_destinations,
        }
    )


@dataclass
class Circuit:
    """A circuit as the lightweight port graph: ``nodes`` [(slot, gate_type)],
    ``edges`` [(src_slot, dst_slot, src_port, dst_port)], and the per-gate
    ``qubits`` (host attribute only; Rz angles likewise)."""

    nodes: list[tuple[int, int]]
    edges: list[tuple[int, int, int, int]]
    qubits: list[tuple[int, ...]] = field(default_factory=list)
    angles: list[int] = field(default_factory=list)

    def snapshot(self) -> dict:
        """Reference snapshot format (beam_search_benchmark.py:81-97)."""
        return {
            "nodes": sorted((slot, gate, -1) for slot, gate in self.nodes),
            "edges": sorted(self.edges),
        }


def random_circuit(num_qubits: int, num_gates: int, seed: int,
                   gate_names: tuple[str, ...] = CIRCUIT_GATES) -> Circuit:
    """Gates uniform from ``gate_names`` on uniform random wires (seeded)."""
    rng = np.random.default_rng(seed)
    last_on_wire: dict[int, tuple[int, int]] = {}
    nodes, edges, qubit_rows, angles = [], [], [], []
    for slot in range(num_gates):
        name = gate_names[int(rng.integers(len(gate_names)))]
        if name == "cx":
            control, target = rng.choice(num_qubits, size=2, replace=False)
            qubits = (int(control), int(target))
        else:
            qubits = (int(rng.integers(num_qubits)),)
        angle = int(rng.integers(8)) if name == "rz" else 0
        nodes.append((slot, GATE_NAME_TO_ID[name]))
        qubit_rows.append(qubits)
        angles.append(angle)
        for port, qubit in enumerate(qubits):
            if qubit in last_on_wire:
                prev_slot, prev_port = last_on_wire[qubit]
                edges.append((prev_slot, slot, prev_port, port))
            last_on_wire[qubit] = (slot, port)
    return Circuit(nodes, edges, qubit_rows, angles)


def random_dag(num_nodes: int, num_gate_types: int, seed: int) -> Circuit:
    """Random DAG with <=2 in/out ports per node (the CPU equivalence s0)."""
    names = ["h", "x", "cx", "t", "tdg", "s", "sdg", "rz"][:num_gate_types]
    return random_circuit(4, num_nodes, seed, tuple(names))


@dataclass(frozen=True)
class ModelConfig:
    """Architecture hyper-parameters (model_factory.py:7-41 argument names)."""

    width: int
    retrieval_width: int
    graph_layers: int
    action_layers: int
    action_heads: int
    max_sequence_length: int
    readout_graph_layers: int
    ordered_binding_roles: bool = False
    readout_graph_input: str = "cached"
    readout_locality_features: bool = False
    identity_readout_prefix: int = 0


# CPU equivalence: d_model 128, 4 heads x 32, 2 causal layers, fp32.
CPU_EQUIVALENCE_MODEL = ModelConfig(
    width=128, retrieval_width=64, graph_layers=1, action_layers=2,
    action_heads=4, max_sequence_length=64, readout_graph_layers=2,
)

# Full rollout: d_model 256, 8 heads, 4 causal + 4 message-passing layers.
ROLLOUT_MODEL = ModelConfig(
    width=256, retrieval_width=128, graph_layers=2, action_layers=4,
    action_heads=8, max_sequence_length=256, readout_graph_layers=4,
)


@dataclass(frozen=True)
class RolloutConfig:
    """Search settings of the full rollout step (paged_rollout_benchmark.py:560-695)."""

    beam_size: int = 1000
    depth: int = 64
    microbatch: int = 512
    page_size: int = 16
    max_candidates_per_state: int = 2048
    per_parent_cap: int = 16
    proposal_factor: int = 16
    max_gate_increase: int = 1
    num_qubits: int = 6
    num_gates: int = 259
    seed: int = 0

    @property
    def global_cap(self) -> int:
        return self.beam_size * self.proposal_factor

    @property
    def cache_pages(self) -> int:
        # paged_rollout_benchmark.py:840-842
        return self.beam_size * (-(-self.depth // self.page_size) + 3)


# Threshold configuration with near == far, unit scale, zero bias and a raw
# threshold below the -1e4 ineligible fill: every eligible (slot, source)
# pair passes and the per-state top-k cap does the bounding.
SELECT_ALL_THRESHOLDS = {
    "groups": {
        name: {"scale": 1.0, "bias": 0.0, "raw_threshold": -1.0e9,
               "probability_threshold": 0.0}
        for name in ("near", "far")
    }
}


def deterministic_parameters(shapes: dict[str, tuple[int, ...]], seed: int,
                             std: float = 0.05) -> dict[str, np.ndarray]:
    """Seeded float32 parameters by name (sorted order), independent of any
    framework's initialisation order.  LayerNorm weights are centred on 1."""
    rng = np.random.default_rng(seed)
    out = {}
    for name in sorted(shapes):
        values = rng.standard_normal(shapes[name]).astype(np.float32) * std
        if name.endswith("norm.weight") or name.endswith("_norm.weight"):
            values = values + 1.0
        out[name] = values
    return out


def parameter_shapes(cfg: ModelConfig, rules: RuleMetadata) -> dict[str, tuple[int, ...]]:
    """Names and shapes of the reference model's trainable parameters
    (paged_model.py:97-195, model.py:143-206) for a configuration."""
    w, r = cfg.width, cfg.retrieval_width
    ns, nx = rules.num_sources, rules.num_xfers
    max_pattern = max(map(len, rules.source_gate_types))
    shapes = {
        "gate_embedding.weight": (rules.num_gate_types, w),
        "source_embedding.weight": (ns, w),
        "xfer_embedding.weight": (nx, w),
        "pattern_position.weight": (max_pattern, w),
        "initial_marker": (w,),
        "pattern_composer.0.weight": (2 * w, w), "pattern_composer.0.bias": (2 * w,),
        "pattern_composer.2.weight": (w, 2 * w), "pattern_composer.2.bias": (w,),
        "current_graph_marker": (w,),
        "action_context.0.weight": (2 * w, 3 * w), "action_context.0.bias": (2 * w,),
        "action_context.3.weight": (w, 2 * w), "action_context.3.bias": (w,),
        "node_query.weight": (w, w), "binding_key.weight": (w, w),
        "binding_value.weight": (w, w),
        "action_delta.0.weight": (2 * w, 3 * w), "action_delta.0.bias": (2 * w,),
        "action_delta.3.weight": (w, 2 * w), "action_delta.3.bias": (w,),
        "action_norm.weight": (w,), "action_norm.bias": (w,),
        "destination_state.0.weight": (2 * w, 3 * w), "destination_state.0.bias": (2 * w,),
        "destination_state.2.weight": (w, 2 * w), "destination_state.2.bias": (w,),
        "retrieval_node.weight": (r, w), "retrieval_source.weight": (r, w),
        "source_bias": (ns,),
        "pointer_node.weight": (r, w),
        "pointer_query.0.weight": (2 * w, 3 * w), "pointer_query.0.bias": (2 * w,),
        "pointer_query.2.weight": (r, 2 * w), "pointer_query.2.bias": (r,),
        "action_position.weight": (cfg.max_sequence_length, w),
        "action_output_norm.weight": (w,), "action_output_norm.bias": (w,),
        "node_action_query.weight": (w, w), "node_action_key.weight": (w, w),
        "node_action_value.weight": (w, w), "node_action_output.weight": (w, w),
        "node_action_norm.weight": (w,), "node_action_norm.bias": (w,),
    }
    for prefix, count in (("graph_layers", cfg.graph_layers),
                          ("readout_graph_layers", cfg.readout_graph_layers)):
        for i in range(count):
            p = f"{prefix}.{i}."
            shapes.update({
                p + "forward_message.weight": (w, w), p + "backward_message.weight": (w, w),
                p + "relation.weight": (32, w),
                p + "update.0.weight": (2 * w, 2 * w), p + "update.0.bias": (2 * w,),
                p + "update.2.weight": (w, 2 * w), p + "update.2.bias": (w,),
                p + "norm.weight": (w,), p + "norm.bias": (w,),
            })
    if cfg.readout_graph_layers:
        shapes["readout_graph_output.weight"] = (w, w)
    for i in range(cfg.action_layers):
        p = f"causal_action_layers.{i}."
        shapes.update({
            p + "input_norm.weight": (w,), p + "input_norm.bias": (w,),
            p + "qkv.weight": (3 * w, w), p + "output.weight": (w, w),
            p + "ffn_norm.weight": (w,), p + "ffn_norm.bias": (w,),
            p + "ffn.0.weight": (4 * w, w), p + "ffn.0.bias": (4 * w,),
            p + "ffn.3.weight": (w, 4 * w), p + "ffn.3.bias": (w,),
        })
    return shapes

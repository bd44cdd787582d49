"""Paged action model with the reference's module structure and decode API.

``PagedActionBindingModel`` has the reference's submodules and parameter
names (paged_model.py:97-195, model.py:12-206), so a reference ``state_dict``
loads unchanged.  Its decode-path methods run on the kernels of
``csrc/model_ops.cu``, ``csrc/paged_attention.cu``, ``csrc/candidates.cu``
and, for every bf16 projection, the tcgen05 GEMM of ``csrc/gemm_tc.cu`` with
the following bias / GELU / residual / LayerNorm / match-logit work fused
into its epilogue (the fp32 CPU-equivalence configuration uses fp32 GEMMs and
the separate row kernels):

* ``initialize_incremental`` (paged_model.py:438-442)
* ``advance_incremental`` with paged K/V (paged_model.py:444-613)
* ``project_action_readout_kv`` (paged_model.py:338-347)
* ``readout_incremental`` with paged readout K/V (paged_model.py:615-655)
* ``match_logits`` (model.py:375-389), ``structural_decode`` (model.py:391-478)

Activations are stored in ``compute_dtype`` (bf16 for the rollout, fp32 for
the CPU-equivalence configuration); every kernel accumulates in fp32.
Supported options are the rollout's: ``readout_graph_input='cached'``, no
ordered binding roles, no locality features; others raise
``NotImplementedError``.
"""
from __future__ import annotations

import math

import torch
from torch import nn
import torch.nn.functional as F

from . import _lib
from . import kernels as K
from .paged_attention import _status_word, paged_attention
from .synthetic import RuleMetadata, parse_pattern


class InitialGraphLayer(nn.Module):
    """Parameters of the reference's message-passing layer (model.py:12-24)."""

    def __init__(self, width: int, num_relations: int = 16):
        super().__init__()
        self.forward_message = nn.Linear(width, width, bias=False)
        self.backward_message = nn.Linear(width, width, bias=False)
        self.relation = nn.Embedding(2 * num_relations, width)
        self.update = nn.Sequential(nn.Linear(2 * width, 2 * width), nn.GELU(),
                                    nn.Linear(2 * width, width))
        self.norm = nn.LayerNorm(width)
        self.num_relations = num_relations


class CausalActionLayer(nn.Module):
    """Parameters of the reference's causal decoder block (paged_model.py:14-35)."""

    def __init__(self, width: int, heads: int, dropout: float):
        super().__init__()
        if width % heads:
            raise ValueError("width must be divisible by heads")
        self.width, self.heads, self.head_width = width, heads, width // heads
        self.input_norm = nn.LayerNorm(width)
        self.qkv = nn.Linear(width, 3 * width, bias=False)
        self.output = nn.Linear(width, width, bias=False)
        self.attention_dropout = nn.Dropout(dropout)
        self.ffn_norm = nn.LayerNorm(width)
        self.ffn = nn.Sequential(nn.Linear(width, 4 * width), nn.GELU(), nn.Dropout(dropout),
                                 nn.Linear(4 * width, width))
        self.residual_dropout = nn.Dropout(dropout)


def _rule_buffers(rules: RuleMetadata):
    """Source-pattern tables of the structural decoder (model.py:75-141)."""
    ns = len(rules.source_gate_types)
    max_pattern = max(map(len, rules.source_gate_types))
    source_types = torch.full((ns, max_pattern), -1, dtype=torch.long)
    source_lengths = torch.zeros(ns, dtype=torch.long)
    for s, types in enumerate(rules.source_gate_types):
        source_types[s, : len(types)] = torch.tensor(types)
        source_lengths[s] = len(types)
    rows, max_edges = [], 0
    for pattern in rules.source_patterns:
        wires: dict[int, list[tuple[int, int]]] = {}
        for op_index, op in enumerate(parse_pattern(pattern)):
            for port, qubit in enumerate(op.qubits):
                wires.setdefault(qubit, []).append((op_index, port))
        edges = [(a, b, pa, pb) for wire in wires.values()
                 for (a, pa), (b, pb) in zip(wire, wire[1:])]
        rows.append(edges)
        max_edges = max(max_edges, len(edges))
    child = torch.full((ns, max_pattern), -1, dtype=torch.long)
    parent, parent_port, child_port = (torch.full_like(child, -1) for _ in range(3))
    direction = torch.zeros_like(child)
    pattern_edges = torch.full((ns, max(max_edges, 1), 4), -1, dtype=torch.long)
    for s, edges in enumerate(rows):
        if edges:
            pattern_edges[s, : len(edges)] = torch.tensor(edges)
        mapped = {0}
        for step in range(int(source_lengths[s]) - 1):
            for a, b, pa, pb in edges:
                if a in mapped and b not in mapped:
                    child[s, step], parent[s, step] = b, a
                    parent_port[s, step], child_port[s, step], direction[s, step] = pa, pb, 1
                    mapped.add(b)
                    break
                if b in mapped and a not in mapped:
                    child[s, step], parent[s, step] = a, b
                    parent_port[s, step], child_port[s, step], direction[s, step] = pb, pa, -1
                    mapped.add(a)
                    break
    return dict(source_types=source_types, source_lengths=source_lengths, binding_child=child,
                binding_parent=parent, binding_parent_port=parent_port,
                binding_child_port=child_port, binding_direction=direction,
                pattern_edges=pattern_edges)


class PagedActionBindingModel(nn.Module):
    def __init__(self, rules: RuleMetadata, *, num_xfers: int, width: int = 192,
                 retrieval_width: int = 128, graph_layers: int = 3, action_layers: int = 4,
                 action_heads: int = 6, max_sequence_length: int = 256,
                 ordered_binding_roles: bool = False, readout_graph_layers: int = 0,
                 readout_graph_input: str = "cached", readout_locality_features: bool = False,
                 identity_readout_prefix: int = 0, readout_attention_backend: str = "paged",
                 dropout: float = 0.05, compute_dtype: torch.dtype = torch.bfloat16):
        super().__init__()
        if ordered_binding_roles or readout_locality_features or readout_graph_input != "cached":
            raise NotImplementedError(
                "the B200 decode path implements readout_graph_input='cached' without "
                "ordered binding roles or locality features")
        if readout_attention_backend != "paged":
            raise ValueError("the B200 decode path reads readout K/V pages in place: "
                             "readout_attention_backend must be 'paged'")
        if not 0 <= identity_readout_prefix <= readout_graph_layers:
            raise ValueError("identity_readout_prefix exceeds readout graph depth")
        self.width, self.retrieval_width = width, retrieval_width
        self.num_sources = len(rules.source_gate_types)
        self.max_pattern = max(map(len, rules.source_gate_types))
        for name, value in _rule_buffers(rules).items():
            self.register_buffer(name, value)
        self.gate_embedding = nn.Embedding(rules.num_gate_types, width)
        self.source_embedding = nn.Embedding(self.num_sources, width)
        self.xfer_embedding = nn.Embedding(num_xfers, width)
        self.pattern_position = nn.Embedding(self.max_pattern, width)
        self.initial_marker = nn.Parameter(torch.zeros(width))
        self.pattern_composer = nn.Sequential(nn.Linear(width, 2 * width), nn.GELU(),
                                              nn.Linear(2 * width, width))
        self.graph_layers = nn.ModuleList(InitialGraphLayer(width) for _ in range(graph_layers))
        self.current_graph_marker = nn.Parameter(torch.zeros(width))
        self.action_context = nn.Sequential(nn.Linear(3 * width, 2 * width), nn.GELU(),
                                            nn.Dropout(dropout), nn.Linear(2 * width, width))
        self.node_query = nn.Linear(width, width, bias=False)
        self.binding_key = nn.Linear(width, width, bias=False)
        self.binding_value = nn.Linear(width, width, bias=False)
        self.action_delta = nn.Sequential(nn.Linear(3 * width, 2 * width), nn.GELU(),
                                          nn.Dropout(dropout), nn.Linear(2 * width, width))
        self.action_norm = nn.LayerNorm(width)
        self.destination_state = nn.Sequential(nn.Linear(3 * width, 2 * width), nn.GELU(),
                                               nn.Linear(2 * width, width))
        self.retrieval_node = nn.Linear(width, retrieval_width, bias=False)
        self.retrieval_source = nn.Linear(width, retrieval_width, bias=False)
        self.source_bias = nn.Parameter(torch.zeros(self.num_sources))
        self.pointer_node = nn.Linear(width, retrieval_width, bias=False)
        self.pointer_query = nn.Sequential(nn.Linear(3 * width, 2 * width), nn.GELU(),
                                           nn.Linear(2 * width, retrieval_width))
        self.action_layers_count = action_layers
        self.action_heads = action_heads
        self.max_sequence_length = max_sequence_length
        self.ordered_binding_roles = False
        self.readout_graph_layers_count = readout_graph_layers
        self.readout_locality_features = False
        self.identity_readout_prefix = identity_readout_prefix
        self.readout_attention_backend = "paged"
        self.readout_graph_input = "cached"
        self.action_position = nn.Embedding(max_sequence_length, width)
        self.causal_action_layers = nn.ModuleList(
            CausalActionLayer(width, action_heads, dropout) for _ in range(action_layers))
        self.action_output_norm = nn.LayerNorm(width)
        self.node_action_query = nn.Linear(width, width, bias=False)
        self.node_action_key = nn.Linear(width, width, bias=False)
        self.node_action_value = nn.Linear(width, width, bias=False)
        self.node_action_output = nn.Linear(width, width, bias=False)
        self.node_action_norm = nn.LayerNorm(width)
        nn.init.zeros_(self.node_action_output.weight)
        if readout_graph_layers:
            self.readout_graph_layers = nn.ModuleList(
                InitialGraphLayer(width) for _ in range(readout_graph_layers))
            if identity_readout_prefix:
                for layer in self.readout_graph_layers[identity_readout_prefix:]:
                    nn.init.zeros_(layer.update[-1].weight)
                    nn.init.zeros_(layer.update[-1].bias)
            self.readout_graph_output = nn.Linear(width, width, bias=False)
            nn.init.zeros_(self.readout_graph_output.weight)
        self.compute_dtype = compute_dtype
        self._prepared_key = None
        self._w: dict[str, torch.Tensor] = {}

    # ---- weight preparation ---------------------------------------------------
    def _apply(self, fn, *args, **kwargs):
        # .to()/.cuda()/.float() may swap parameter storage: list them afresh
        self._param_list = None
        return super()._apply(fn, *args, **kwargs)

    def _version_key(self):
        """Storage pointer and in-place version of every parameter: changes
        whenever a parameter is replaced or written (load_state_dict, an
        optimizer step), so the prepared weights are rebuilt."""
        params = getattr(self, "_param_list", None)
        if params is None:
            params = self._param_list = list(self.parameters())
        return tuple((p.data_ptr(), p._version) for p in params) + (self.compute_dtype,)

    @torch.no_grad()
    def prepare(self) -> dict[str, torch.Tensor]:
        """Kernel-ready weights: transposed compute-dtype GEMM operands,
        fp32 vectors and the precomputed per-type / per-position tables.
        Rebuilt whenever a parameter changes."""
        key = self._version_key()
        if self._prepared_key == key:
            return self._w
        dt, w, W = self.compute_dtype, {}, self.width
        t = lambda m: m.detach().t().contiguous().to(dt)
        f = lambda v: v.detach().float().contiguous()
        c = lambda v: v.detach().to(dt).contiguous()   # GEMM-epilogue biases (autocast rounds them)
        for name in ("gate_embedding", "xfer_embedding", "action_position"):
            w[name] = f(getattr(self, name).weight)
        w["initial_marker"] = f(self.initial_marker)
        reps = self._source_representations_fp32()
        w["source_reps"] = reps.contiguous()
        w["source_vectors_t"] = t(F.linear(reps, self.retrieval_source.weight.float()))
        w["source_bias"] = f(self.source_bias)
        w["first_types"] = self.source_types[:, 0].contiguous()
        for prefix, layers in (("graph", self.graph_layers),
                               ("readout_graph", getattr(self, "readout_graph_layers", []))):
            for i, layer in enumerate(layers):
                p = f"{prefix}{i}."
                w[p + "fb_t"] = t(torch.cat((layer.forward_message.weight,
                                             layer.backward_message.weight), 0))
                w[p + "rel"] = f(layer.relation.weight)
                w[p + "u0_t"], w[p + "u0_b"] = t(layer.update[0].weight), f(layer.update[0].bias)
                w[p + "u2_t"], w[p + "u2_b"] = t(layer.update[2].weight), c(layer.update[2].bias)
                w[p + "norm_w"], w[p + "norm_b"] = f(layer.norm.weight), f(layer.norm.bias)
        if self.readout_graph_layers_count:
            w["readout_graph_output_t"] = t(self.readout_graph_output.weight)
        ac0 = self.action_context[0]
        w["ac0_t"], w["ac0_b"] = t(ac0.weight), f(ac0.bias)
        w["ac3_t"], w["ac3_b"] = t(self.action_context[3].weight), c(self.action_context[3].bias)
        d0 = self.action_delta[0].weight
        w["qxa_t"] = t(torch.cat((self.node_query.weight, d0[:, :W]), 0))
        w["bk_t"] = t(self.binding_key.weight)
        w["bv_t"] = t(self.binding_value.weight)
        w["d0b_t"] = t(d0[:, W:2 * W])
        w["d0c_t"], w["d0_b"] = t(d0[:, 2 * W:]), c(self.action_delta[0].bias)
        w["d3_t"], w["d3_b"] = t(self.action_delta[3].weight), c(self.action_delta[3].bias)
        w["action_norm_w"], w["action_norm_b"] = f(self.action_norm.weight), f(self.action_norm.bias)
        ds0 = self.destination_state[0].weight.float()
        w["ds0a_t"], w["ds0_b"] = t(ds0[:, :W]), c(self.destination_state[0].bias)
        w["ds_type_table"] = (self.gate_embedding.weight.float() @ ds0[:, W:2 * W].t()).contiguous()
        w["ds_pos_table"] = (self.pattern_position.weight.float() @ ds0[:, 2 * W:].t()).contiguous()
        w["ds2_t"], w["ds2_b"] = t(self.destination_state[2].weight), c(self.destination_state[2].bias)
        for i, layer in enumerate(self.causal_action_layers):
            p = f"causal{i}."
            w[p + "in_w"], w[p + "in_b"] = f(layer.input_norm.weight), f(layer.input_norm.bias)
            w[p + "qkv_t"], w[p + "out_t"] = t(layer.qkv.weight), t(layer.output.weight)
            w[p + "ffn_norm_w"], w[p + "ffn_norm_b"] = f(layer.ffn_norm.weight), f(layer.ffn_norm.bias)
            w[p + "f0_t"], w[p + "f0_b"] = t(layer.ffn[0].weight), f(layer.ffn[0].bias)
            w[p + "f3_t"], w[p + "f3_b"] = t(layer.ffn[3].weight), c(layer.ffn[3].bias)
        w["out_norm_w"] = f(self.action_output_norm.weight)
        w["out_norm_b"] = f(self.action_output_norm.bias)
        w["naq_t"], w["nak_t"] = t(self.node_action_query.weight), t(self.node_action_key.weight)
        w["nav_t"], w["nao_t"] = t(self.node_action_value.weight), t(self.node_action_output.weight)
        w["na_norm_w"], w["na_norm_b"] = f(self.node_action_norm.weight), f(self.node_action_norm.bias)
        w["retrieval_node_t"] = t(self.retrieval_node.weight)
        if dt == torch.bfloat16:
            self._prepare_tensor_core(w)
        self._w, self._prepared_key = w, key
        return w

    @torch.no_grad()
    def _prepare_tensor_core(self, w: dict) -> None:
        """K-major bf16 operands ([out, in], the Linear layout) of the tcgen05
        GEMMs and their fp32 epilogue biases rounded to bf16 first, as bf16
        autocast rounds a Linear's bias."""
        W = self.width
        k = lambda m: m.detach().to(torch.bfloat16).contiguous()
        b = lambda v: v.detach().to(torch.bfloat16).float().contiguous()
        dev = self.gate_embedding.weight.device
        w["zero_bias"] = torch.zeros(W, device=dev, dtype=torch.float32)
        for prefix, layers in (("graph", self.graph_layers),
                               ("readout_graph", getattr(self, "readout_graph_layers", []))):
            for i, layer in enumerate(layers):
                p = f"{prefix}{i}."
                w[p + "fb_k"] = k(torch.cat((layer.forward_message.weight,
                                             layer.backward_message.weight), 0))
                w[p + "u0_k"], w[p + "u0_bf"] = k(layer.update[0].weight), b(layer.update[0].bias)
                w[p + "u2_k"], w[p + "u2_bf"] = k(layer.update[2].weight), b(layer.update[2].bias)
        if self.readout_graph_layers_count:
            w["readout_graph_output_k"] = k(self.readout_graph_output.weight)
        w["ac0_k"], w["ac0_bf"] = k(self.action_context[0].weight), b(self.action_context[0].bias)
        w["ac3_k"], w["ac3_bf"] = k(self.action_context[3].weight), b(self.action_context[3].bias)
        d0 = self.action_delta[0].weight
        w["qxa_k"] = k(torch.cat((self.node_query.weight, d0[:, :W]), 0))
        w["bk_k"], w["bv_k"] = k(self.binding_key.weight), k(self.binding_value.weight)
        w["d0b_k"], w["d0c_k"] = k(d0[:, W:2 * W]), k(d0[:, 2 * W:])
        w["d0_bf"] = b(self.action_delta[0].bias)
        w["d3_k"], w["d3_bf"] = k(self.action_delta[3].weight), b(self.action_delta[3].bias)
        ds0 = self.destination_state[0].weight
        w["ds0a_k"], w["ds0_bf"] = k(ds0[:, :W]), b(self.destination_state[0].bias)
        w["ds2_k"], w["ds2_bf"] = k(self.destination_state[2].weight), b(self.destination_state[2].bias)
        for i, layer in enumerate(self.causal_action_layers):
            p = f"causal{i}."
            w[p + "qkv_k"], w[p + "out_k"] = k(layer.qkv.weight), k(layer.output.weight)
            w[p + "f0_k"], w[p + "f0_bf"] = k(layer.ffn[0].weight), b(layer.ffn[0].bias)
            w[p + "f3_k"], w[p + "f3_bf"] = k(layer.ffn[3].weight), b(layer.ffn[3].bias)
        w["naq_k"], w["nak_k"] = k(self.node_action_query.weight), k(self.node_action_key.weight)
        w["nav_k"], w["nao_k"] = k(self.node_action_value.weight), k(self.node_action_output.weight)
        if self.num_sources <= 32:
            w["match_k"] = self._match_weight(w["source_vectors_t"].t().float())

    def _match_weight(self, source_vectors: torch.Tensor) -> torch.Tensor:
        """[32, W] bf16: the source vectors times the retrieval_node weight,
        so node projection and source product (model.py:375-389) are one
        GEMM; rows past the source count are zero."""
        prod = source_vectors.float() @ self.retrieval_node.weight.detach().float()
        out = torch.zeros(32, self.width, device=prod.device, dtype=torch.float32)
        out[: prod.shape[0]] = prod
        return out.to(torch.bfloat16).contiguous()

    def _tc(self) -> bool:
        """bf16: every projection runs on the tcgen05 GEMM."""
        return self.compute_dtype == torch.bfloat16

    def _status(self, device) -> torch.Tensor:
        status = getattr(self, "kernel_status", None)
        return _status_word(device) if status is None else status

    @torch.no_grad()
    def _source_representations_fp32(self) -> torch.Tensor:
        positions = self.pattern_position.weight[: self.max_pattern].float()
        tokens = self.gate_embedding.weight.float()[self.source_types.clamp_min(0)] + positions.unsqueeze(0)
        mask = self.source_types.ge(0).unsqueeze(-1)
        composed = (tokens * mask).sum(1) / mask.sum(1).clamp_min(1)
        pc = self.pattern_composer
        hidden = F.gelu(F.linear(composed, pc[0].weight.float(), pc[0].bias.float()))
        return self.source_embedding.weight.float() + F.linear(hidden, pc[2].weight.float(),
                                                               pc[2].bias.float())

    def source_representations(self) -> torch.Tensor:
        """model.py:208-214 (fp32, computed once per weight version)."""
        return self.prepare()["source_reps"]

    # ---- message passing ----------------------------------------------------
    def _graph_layers(self, prefix: str, count: int, x_buf: torch.Tensor, live: torch.Tensor,
                      ports, slots: int, keep_input: bool = False) -> torch.Tensor:
        """Run `count` InitialGraphLayer blocks (model.py:26-53).  x_buf is
        [M, 2W] with the layer input in its first W columns; returns the
        [M, 2W] buffer whose first W columns hold the output.  With
        keep_input the first W columns of x_buf are left untouched.

        bf16: the message projection (a tcgen05 GEMM), the aggregation kernel,
        then the update MLP with its GELU, the residual, the LayerNorm and the
        dead-row mask in one fused tcgen05 launch (width 256; other widths run
        the two GEMMs with fused epilogues)."""
        w, W = self.prepare(), self.width
        m = x_buf.shape[0]
        tc = self._tc()
        status = self._status(x_buf.device) if tc else None
        spare = [torch.empty_like(x_buf)]
        if keep_input and count > 1:
            spare.append(torch.empty_like(x_buf))
        fb = torch.empty(m, 2 * W, device=x_buf.device, dtype=x_buf.dtype)
        hidden = None if tc and W == 256 else torch.empty(m, 2 * W, device=x_buf.device,
                                                          dtype=x_buf.dtype)
        upd = None if tc else torch.empty(m, W, device=x_buf.device, dtype=x_buf.dtype)
        live_flat = live.reshape(-1)
        for i in range(count):
            p = f"{prefix}{i}."
            x = x_buf[:, :W]
            target = spare.pop(0)
            if tc:
                K.gemm(x, w[p + "fb_k"], out=fb, status=status)
                K.graph_aggregate(fb, w[p + "rel"], ports, slots, x_buf[:, W:])
                if W == 256:   # update MLP + residual + LayerNorm, GELU kept on chip
                    K.graph_mlp(x_buf, w[p + "u0_k"], w[p + "u0_bf"], w[p + "u2_k"],
                                w[p + "u2_bf"], x, w[p + "norm_w"], w[p + "norm_b"],
                                zero_row=live_flat, out=target[:, :W], status=status)
                else:
                    K.gemm(x_buf, w[p + "u0_k"], w[p + "u0_bf"], gelu=True, out=hidden,
                           status=status)
                    K.gemm_layernorm(hidden, w[p + "u2_k"], w[p + "u2_bf"], x, w[p + "norm_w"],
                                     w[p + "norm_b"], zero_row=live_flat, out=target[:, :W],
                                     status=status)
            else:
                K.linear(x, w[p + "fb_t"], out=fb)
                K.graph_aggregate(fb, w[p + "rel"], ports, slots, x_buf[:, W:])
                K.linear(x_buf, w[p + "u0_t"], out=hidden)
                K.bias_gelu(hidden, w[p + "u0_b"])
                K.linear(hidden, w[p + "u2_t"], w[p + "u2_b"], out=upd)
                K.add_layernorm(x, upd, gamma=w[p + "norm_w"], beta=w[p + "norm_b"],
                                ln_out=target[:, :W], zero_row=live_flat)
            if not (keep_input and i == 0):
                spare.append(x_buf)
            x_buf = target
        return x_buf

    def _ports(self, batch: dict, b: int, s: int, device):
        return K.edges_to_ports(batch["current_edge_batch"] if "current_edge_batch" in batch
                                else batch["edge_batch"],
                                batch["current_edge_src"] if "current_edge_src" in batch
                                else batch["edge_src"],
                                batch["current_edge_dst"] if "current_edge_dst" in batch
                                else batch["edge_dst"],
                                batch["current_edge_relation"] if "current_edge_relation" in batch
                                else batch["edge_relation"], b, s, device)

    @torch.no_grad()
    def initialize_incremental(self, batch: dict):
        """Encode s0 once (paged_model.py:243-260, 438-442)."""
        w, W = self.prepare(), self.width
        types = batch["initial_types"].to(self.gate_embedding.weight.device, torch.int64).contiguous()
        b, s = types.shape
        dev = types.device
        x_buf = torch.empty(b * s, 2 * W, device=dev, dtype=self.compute_dtype)
        live = torch.empty(b, s, device=dev, dtype=torch.bool)
        K.embed_initial(types, w["gate_embedding"], w["initial_marker"], x_buf[:, :W], live)
        if self.graph_layers:
            ports = K.edges_to_ports(batch["edge_batch"], batch["edge_src"], batch["edge_dst"],
                                     batch["edge_relation"], b, s, dev)
            x_buf = self._graph_layers("graph", len(self.graph_layers), x_buf, live, ports, s)
        states = x_buf[:, :W].contiguous().view(b, s, W)
        return states, live, types.clone()

    # ---- readout --------------------------------------------------------------
    @torch.no_grad()
    def readout_incremental(self, states, live, gate_types, action_states=None, action_mask=None,
                            batch: dict | None = None, *, readout_key_cache=None,
                            readout_value_cache=None, block_table=None, lengths=None, ports=None):
        """Paged node readout then the readout graph (paged_model.py:615-655).

        ``ports`` (in_node, in_port, out_node, out_port int32 [B, S, 4]) may be
        given instead of the batch's edge lists."""
        paged = (readout_key_cache, readout_value_cache, block_table, lengths)
        if any(v is None for v in paged):
            raise ValueError("the B200 readout reads the paged readout K/V cache: supply "
                             "readout_key_cache, readout_value_cache, block_table and lengths")
        w, W = self.prepare(), self.width
        b, s, _ = states.shape
        h = self.action_heads
        states = states.to(self.compute_dtype).contiguous()
        flat = states.view(b * s, W)
        live_flat = live.reshape(-1)
        tc = self._tc()
        status = self._status(states.device) if tc else None
        live_u8 = live_flat.view(torch.uint8) if live_flat.dtype == torch.bool else live_flat
        q = K.gemm(flat, w["naq_k"], status=status) if tc else K.linear(flat, w["naq_t"])
        query = q.view(b, s, h, W // h).transpose(1, 2)
        ctx = paged_attention(query, readout_key_cache, readout_value_cache, block_table, lengths)
        ctx2d = ctx.transpose(1, 2).reshape(b * s, W)
        x_buf = torch.empty(b * s, 2 * W, device=states.device, dtype=states.dtype)
        lengths32 = lengths.to(torch.int32).contiguous()
        if tc:   # output projection + residual + LayerNorm + masks in one GEMM
            K.gemm_layernorm(ctx2d, w["nao_k"], w["zero_bias"], flat, w["na_norm_w"],
                             w["na_norm_b"], zero_row=live_u8, where_len=lengths32,
                             rows_per_beam=s, out=x_buf[:, :W], status=status)
        else:
            u = K.linear(ctx2d, w["nao_t"])
            K.add_layernorm(flat, u, gamma=w["na_norm_w"], beta=w["na_norm_b"],
                            ln_out=x_buf[:, :W], zero_row=live_flat, where_len=lengths32,
                            rows_per_beam=s)
        if not self.readout_graph_layers_count:
            return x_buf[:, :W].contiguous().view(b, s, W), live, gate_types
        if ports is None:
            if batch is None:
                raise ValueError("readout graph layers require an action-derived graph")
            ports = self._ports(batch, b, s, states.device)
        g = self._graph_layers("readout_graph", self.readout_graph_layers_count, x_buf, live,
                               ports, s, keep_input=True)
        out = torch.empty(b * s, W, device=states.device, dtype=states.dtype)
        if tc:   # (states + readout_graph_output(g)) * live in one GEMM
            K.gemm(g[:, :W], w["readout_graph_output_k"], residual=x_buf[:, :W],
                   zero_row=live_u8, out=out, status=status)
        else:
            proj = K.linear(g[:, :W], w["readout_graph_output_t"])
            K.add_layernorm(x_buf[:, :W], proj, sum_out=out, zero_row=live_flat,
                            zero_before=True)
        return out.view(b, s, W), live, gate_types

    @torch.no_grad()
    def project_action_readout_kv(self, action_states):
        """Readout K/V of a new contextual action (paged_model.py:338-347)."""
        w = self.prepare()
        b = action_states.shape[0]
        shape = (b, self.action_heads, self.width // self.action_heads)
        a = action_states.to(self.compute_dtype).contiguous()
        if self._tc():
            status = self._status(a.device)
            return (K.gemm(a, w["nak_k"], status=status).view(shape),
                    K.gemm(a, w["nav_k"], status=status).view(shape))
        return K.linear(a, w["nak_t"]).view(shape), K.linear(a, w["nav_t"]).view(shape)

    # ---- one action -------------------------------------------------------------
    @torch.no_grad()
    def advance_incremental(self, states, live, gate_types, past_keys=None, past_values=None,
                            past_action_states=None, past_mask=None, *, xfer_ids, source_ids,
                            source_slots, destination_slots, destination_types,
                            paged_key_cache=None, paged_value_cache=None, block_table=None,
                            past_lengths=None, return_mask: bool = True):
        """Append exactly one action per beam and return its per-layer K/V.

        Returns (next_states, next_live, next_gate_types, new_keys [L,B,H,D],
        new_values, action_token [B,W], next_mask) as paged_model.py:605-613."""
        paged = (paged_key_cache, paged_value_cache, block_table, past_lengths)
        if any(v is None for v in paged):
            raise ValueError("the B200 decode path attends to physical cache pages: supply "
                             "paged_key_cache, paged_value_cache, block_table and past_lengths")
        w, W = self.prepare(), self.width
        dev, dt = states.device, self.compute_dtype
        b = states.shape[0]
        h = self.action_heads
        hd = W // h
        i64 = lambda t: t.to(device=dev, dtype=torch.int64).contiguous()
        xfer_ids, source_ids = i64(xfer_ids), i64(source_ids)
        source_slots, destination_slots = i64(source_slots), i64(destination_slots)
        destination_types = i64(destination_types)
        past_lengths = past_lengths.to(device=dev, dtype=torch.int32).contiguous()
        states = states.to(dt)
        referenced = torch.cat((source_slots, destination_slots), 1)
        if referenced.numel():
            top = int(referenced.max().item())
            if top >= states.shape[1]:
                extra = top + 1 - states.shape[1]
                states = F.pad(states, (0, 0, 0, extra))
                live = F.pad(live, (0, extra), value=False)
                gate_types = F.pad(gate_types, (0, extra), value=-1)
        states = states.contiguous()
        live = live.contiguous()
        gate_types = gate_types.to(torch.int64).contiguous()
        if int(past_lengths.max().item() if past_lengths.numel() else 0) >= self.max_sequence_length:
            raise ValueError("incremental prefix exceeds max_sequence_length")
        next_states, next_live, next_types, new_keys, new_values, action = self.advance_device(
            states, live, gate_types, xfer_ids, source_ids, source_slots, destination_slots,
            destination_types, paged_key_cache, paged_value_cache, block_table, past_lengths)
        next_mask = None
        if return_mask:
            max_past = int(past_lengths.max().item()) if b else 0
            history = torch.arange(max_past, device=dev).unsqueeze(0) < past_lengths.unsqueeze(1)
            next_mask = torch.cat((history, xfer_ids.ge(0).unsqueeze(1)), 1)
        return next_states, next_live, next_types, new_keys, new_values, action, next_mask

    @torch.no_grad()
    def advance_device(self, states, live, gate_types, xfer_ids, source_ids, source_slots,
                       destination_slots, destination_types, paged_key_cache, paged_value_cache,
                       block_table, past_lengths, return_readout_kv: bool = False,
                       graphed: bool = False):
        """One-token step without host synchronisation: states [B, S, W] already
        hold every referenced slot; ids int64, past_lengths int32 on the device.
        Returns (next_states, next_live, next_types, new_keys [L,B,H,D],
        new_values, action_token) (+ the action's readout key and value with
        return_readout_kv).  With `graphed` the per-beam token path replays a
        CUDA graph and the returned keys, values, action and readout K/V are
        overwritten by the next graphed step of the same shape."""
        w, W = self.prepare(), self.width
        dev, dt = states.device, self.compute_dtype
        b = states.shape[0]
        h = self.action_heads
        hd = W // h
        s = states.shape[1]
        pattern = source_slots.shape[1]
        bound = torch.empty(b, pattern, W, device=dev, dtype=dt)
        ctx_in = torch.empty(b, 3 * W, device=dev, dtype=dt)
        source_mask = torch.empty(b, pattern, device=dev, dtype=torch.bool)
        active = torch.empty(b, device=dev, dtype=torch.bool)
        K.action_inputs(states, xfer_ids, source_ids, source_slots, w["xfer_embedding"],
                        w["source_reps"], bound, ctx_in, source_mask, active)
        step = self._token_step if graphed else self._token_step_eager
        raw, new_keys, new_values, action, rk, rv = step(
            ctx_in, active, past_lengths.to(torch.int32).contiguous(),
            block_table.to(torch.int32).contiguous(), paged_key_cache, paged_value_cache)
        next_states, next_live, next_types = self._update_and_apply(
            states, live, gate_types, bound, source_mask, raw, active, source_slots,
            destination_slots, destination_types)
        if return_readout_kv:
            return next_states, next_live, next_types, new_keys, new_values, action, rk, rv
        return next_states, next_live, next_types, new_keys, new_values, action

    # ---- the per-beam token path of one step (CUDA graph per shape) ------------
    USE_GRAPHS = True
    # captured token-step graphs kept (least recently used dropped): a 64-level
    # search meets at most ~64 (beams, block-table width) shapes
    GRAPH_CACHE_LIMIT = 64

    def _token_step_eager(self, ctx_in, active, past_lengths, block_table, key_cache,
                          value_cache):
        """Action context MLP, position token, the causal layers over the paged
        cache, output norm and the readout K/V of the new action: everything
        of a step that works on one row per beam (paged_model.py:444-613,
        338-347).  Returns (raw, new_keys, new_values, action, readout key,
        readout value)."""
        w, W = self.prepare(), self.width
        dev, dt = ctx_in.device, self.compute_dtype
        b = ctx_in.shape[0]
        h = self.action_heads
        hd = W // h
        tc = self._tc()
        status = self._status(dev) if tc else None
        if tc:
            hidden = K.gemm(ctx_in, w["ac0_k"], w["ac0_bf"], gelu=True, status=status)
            raw = K.gemm(hidden, w["ac3_k"], w["ac3_bf"], status=status)
        else:
            hidden = K.bias_gelu(K.linear(ctx_in, w["ac0_t"]), w["ac0_b"])
            raw = K.linear(hidden, w["ac3_t"], w["ac3_b"])
        token = torch.empty_like(raw)
        K.position_token(raw, w["action_position"], past_lengths, active, token)
        valid = active
        # every layer's [q | k | v] rows in one buffer: the new keys and values
        # of all layers leave it in two copies after the loop
        qkv_all = torch.empty(self.action_layers_count, b, 3 * W, device=dev, dtype=dt)
        ln = torch.empty_like(token)
        token2 = torch.empty_like(token)
        for layer in range(self.action_layers_count):
            p = f"causal{layer}."
            K.add_layernorm(token, gamma=w[p + "in_w"], beta=w[p + "in_b"], ln_out=ln)
            if tc:
                qkv = K.gemm(ln, w[p + "qkv_k"], out=qkv_all[layer], status=status).view(b, 3, h, hd)
            else:
                qkv = K.linear(ln, w[p + "qkv_t"], out=qkv_all[layer]).view(b, 3, h, hd)
            q, k, v = qkv.unbind(1)
            ctx = paged_attention(q.unsqueeze(2), key_cache[layer], value_cache[layer],
                                  block_table, past_lengths, current_key=k, current_value=v,
                                  current_valid=valid, status=status)
            if tc:
                o = K.gemm(ctx.reshape(b, W), w[p + "out_k"], status=status)
            else:
                o = K.linear(ctx.reshape(b, W), w[p + "out_t"])
            K.add_layernorm(token, o, gamma=w[p + "ffn_norm_w"], beta=w[p + "ffn_norm_b"],
                            sum_out=token2, ln_out=ln)
            token = torch.empty_like(token2)
            if tc:   # FFN; the second GEMM adds the residual and zeroes inactive beams
                f0 = K.gemm(ln, w[p + "f0_k"], w[p + "f0_bf"], gelu=True, status=status)
                K.gemm(f0, w[p + "f3_k"], w[p + "f3_bf"], residual=token2, zero_row=active,
                       out=token, status=status)
            else:
                f0 = K.bias_gelu(K.linear(ln, w[p + "f0_t"]), w[p + "f0_b"])
                f3 = K.linear(f0, w[p + "f3_t"], w[p + "f3_b"])
                K.add_layernorm(token2, f3, sum_out=token, zero_beam=active, zero_before=True)
        kv = qkv_all.view(self.action_layers_count, b, 3, h, hd)
        new_keys, new_values = kv[:, :, 1].contiguous(), kv[:, :, 2].contiguous()
        action = torch.empty_like(token)
        K.add_layernorm(token, gamma=w["out_norm_w"], beta=w["out_norm_b"], ln_out=action,
                        zero_beam=active)
        rk, rv = self.project_action_readout_kv(action)
        return raw, new_keys, new_values, action, rk, rv

    def _token_step(self, ctx_in, active, past_lengths, block_table, key_cache, value_cache):
        """_token_step_eager replayed from a CUDA graph captured once per
        (beams, block-table width, weights, cache) key: ~60 launches of one-row-
        per-beam work cost one replay and four input copies of host time.  The
        outputs live in the graph's pool until the next replay of that key, so
        they must be consumed before the next step (the search does)."""
        if not self.USE_GRAPHS or ctx_in.shape[0] == 0:
            return self._token_step_eager(ctx_in, active, past_lengths, block_table, key_cache,
                                          value_cache)
        version = self._version_key()
        graphs = getattr(self, "_graphs", None)
        if graphs is None or graphs[0] != version:
            if graphs is not None and graphs[1]:
                torch.cuda.synchronize(ctx_in.device)   # no replay of a dropped graph pending
            graphs = self._graphs = (version, {})
        # the captured attention bakes in the arena's address and its page
        # count (the page-id bound): a new cache allocated at a freed cache's
        # address with another capacity must not replay the old graph
        key = (ctx_in.shape[0], block_table.shape[1], block_table.dtype, ctx_in.dtype,
               key_cache.data_ptr(), tuple(key_cache.shape), key_cache.dtype,
               value_cache.data_ptr(), tuple(value_cache.shape), value_cache.dtype,
               ctx_in.device)
        entry = graphs[1].pop(key, None)
        inputs = (ctx_in, active, past_lengths, block_table)
        if entry is None:
            if len(graphs[1]) >= self.GRAPH_CACHE_LIMIT:
                torch.cuda.synchronize(ctx_in.device)
                graphs[1].pop(next(iter(graphs[1])))    # least recently used
            entry = self._capture_token_step(inputs, key_cache, value_cache)
        graphs[1][key] = entry                          # most recently used last
        static, graph, outs, launches = entry
        for dst, src in zip(static, inputs):
            dst.copy_(src)
        graph.replay()
        _lib.lib().grs_count_launches(launches)
        return outs

    def _capture_token_step(self, inputs, key_cache, value_cache):
        static = [t.clone() for t in inputs]
        current = torch.cuda.current_stream(inputs[0].device)
        side = torch.cuda.Stream(inputs[0].device)
        side.wait_stream(current)
        with torch.cuda.stream(side), _lib.pinned_stream():   # warm-up: libraries initialise
            self._token_step_eager(*static, key_cache, value_cache)
        current.wait_stream(side)
        graph = torch.cuda.CUDAGraph()
        before = int(_lib.lib().grs_launch_count())
        with torch.cuda.graph(graph, capture_error_mode="thread_local"), _lib.pinned_stream():
            outs = self._token_step_eager(*static, key_cache, value_cache)
        launches = int(_lib.lib().grs_launch_count()) - before
        return static, graph, outs, launches

    def _update_and_apply(self, states, live, gate_types, bound, source_mask, raw, active,
                          source_slots, destination_slots, destination_types):
        """_update_live_nodes then slot kill/create (paged_model.py:560-604)."""
        w, W = self.prepare(), self.width
        b, s, _ = states.shape
        dev, dt = states.device, states.dtype
        m = b * s
        pattern = bound.shape[1]
        flat = states.view(m, W)
        tc = self._tc()
        status = self._status(dev) if tc else None
        bound2d = bound.view(b * pattern, W)
        if tc:
            qxa = K.gemm(flat, w["qxa_k"], status=status)                         # [M, 3W]
            keys = K.gemm(bound2d, w["bk_k"], status=status)                      # [B*P, W]
            vw = K.gemm(K.gemm(bound2d, w["bv_k"], status=status), w["d0b_k"],
                        status=status)                                            # [B*P, 2W]
            cvec = K.gemm(raw, w["d0c_k"], w["d0_bf"], status=status)             # [B, 2W]
        else:
            qxa = K.linear(flat, w["qxa_t"])
            keys = K.linear(bound2d, w["bk_t"])
            vw = K.linear(K.linear(bound2d, w["bv_t"]), w["d0b_t"])
            cvec = K.linear(raw, w["d0c_t"], w["d0_b"])
        hidden = torch.empty(m, 2 * W, device=dev, dtype=dt)
        affinity = torch.empty(m, device=dev, dtype=torch.float32)
        K.update_live_hidden(qxa, keys, vw, cvec, source_mask, s, W, hidden, affinity)
        next_states = torch.empty_like(states)
        if tc:   # action_delta output + affinity scale + residual + LayerNorm + masks
            K.gemm_layernorm(hidden, w["d3_k"], w["d3_bf"], flat, w["action_norm_w"],
                             w["action_norm_b"], row_scale=affinity, where_row=live.reshape(-1),
                             where_beam=active, rows_per_beam=s, out=next_states.view(m, W),
                             status=status)
        else:
            delta = K.linear(hidden, w["d3_t"], w["d3_b"])
            K.add_layernorm(flat, delta, scale=affinity, gamma=w["action_norm_w"],
                            beta=w["action_norm_b"], ln_out=next_states.view(m, W),
                            where_row=live.reshape(-1), where_beam=active, rows_per_beam=s)
        next_live = live.clone()
        next_types = gate_types.clone()
        dpattern = destination_slots.shape[1]
        r = K.gemm(raw, w["ds0a_k"], w["ds0_bf"], status=status) if tc else \
            K.linear(raw, w["ds0a_t"], w["ds0_b"])
        dh = torch.empty(b * dpattern, 2 * W, device=dev, dtype=dt)
        K.destination_hidden(r, w["ds_type_table"], w["ds_pos_table"], destination_slots,
                             destination_types, active, dh)
        created = K.gemm(dh, w["ds2_k"], w["ds2_bf"], status=status) if tc else \
            K.linear(dh, w["ds2_t"], w["ds2_b"])
        K.apply_slots(next_states, next_live, next_types, source_slots, source_mask,
                      destination_slots, destination_types, active, created)
        return next_states, next_live, next_types

    # ---- match logits -------------------------------------------------------------
    @torch.no_grad()
    def match_logits(self, states, live, gate_types, source_vectors=None):
        """fp32 logits [B, S, sources] masked to -1e4 off the eligible set and
        the eligible mask (model.py:375-389)."""
        w = self.prepare()
        b, s, W = states.shape
        flat = states.to(self.compute_dtype).contiguous().view(b * s, W)
        logits = torch.empty(b, s, self.num_sources, device=states.device, dtype=torch.float32)
        eligible = torch.empty(b, s, self.num_sources, device=states.device, dtype=torch.bool)
        scale = 1.0 / math.sqrt(self.retrieval_width)
        if self._tc():
            if self.num_sources > 32:
                raise ValueError("the tensor-core match logits take at most 32 source patterns")
            weight = w["match_k"] if source_vectors is None else \
                self._match_weight(source_vectors.to(flat.device))
            K.match_logits_gemm(flat, weight, w["source_bias"], w["first_types"],
                                live.contiguous(), gate_types.to(torch.int64).contiguous(), scale,
                                logits, eligible, status=self._status(flat.device))
            return logits, eligible
        node = K.linear(flat, w["retrieval_node_t"])
        sv_t = w["source_vectors_t"] if source_vectors is None else \
            source_vectors.t().contiguous().to(self.compute_dtype)
        acc = K.linear(node, sv_t)
        K.match_logits(acc, w["source_bias"], w["first_types"], live.contiguous(),
                       gate_types.to(torch.int64).contiguous(), scale, logits, eligible)
        return logits, eligible

    # ---- structural decode ------------------------------------------------------
    def rule_tables(self) -> dict[str, torch.Tensor]:
        return {name: getattr(self, name).contiguous() for name in (
            "source_types", "source_lengths", "binding_child", "binding_parent",
            "binding_parent_port", "binding_child_port", "binding_direction", "pattern_edges")}

    @torch.no_grad()
    def structural_decode(self, batch, gate_types, live, batch_ids, source_ids, anchor_slots,
                          ports=None):
        """Port-following decoder for complete ordered bindings (model.py:391-478).
        Returns (bindings int64 [n, max_pattern], valid bool [n])."""
        b, s = gate_types.shape
        dev = gate_types.device
        if ports is None:
            ports = self._ports(batch, b, s, dev)
        n = batch_ids.numel()
        bindings = torch.empty(n, self.max_pattern, device=dev, dtype=torch.int64)
        valid = torch.empty(n, device=dev, dtype=torch.bool)
        sources = source_ids.to(torch.int64).clone()
        K.structural_decode(gate_types.to(torch.int64).contiguous(), live.contiguous(), ports,
                            self.rule_tables(), batch_ids.to(torch.int64).contiguous(), sources,
                            anchor_slots.to(torch.int64).contiguous(), bindings, valid)
        return bindings, valid

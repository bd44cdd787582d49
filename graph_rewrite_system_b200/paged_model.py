"""Paged action model with the reference's module structure and decode API.

``PagedActionBindingModel`` has the reference's submodules and parameter
names (paged_model.py:97-195, model.py:12-206), so a reference ``state_dict``
loads unchanged.  Its decode-path methods run on the kernels of
``csrc/model_ops.cu``, ``csrc/paged_attention.cu`` and ``csrc/candidates.cu``
with plain cuBLAS GEMMs in between:

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
                if dt == torch.bfloat16:   # K-major operands of the tensor-core GEMMs
                    w[p + "u0_k"] = c(layer.update[0].weight)
                    w[p + "u2_k"] = c(layer.update[2].weight)
                    w[p + "u2_bf"] = c(layer.update[2].bias).float()
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
        self._w, self._prepared_key = w, key
        return w

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
        keep_input the first W columns of x_buf are left untouched."""
        w, W = self.prepare(), self.width
        m = x_buf.shape[0]
        spare = [torch.empty_like(x_buf)]
        if keep_input and count > 1:
            spare.append(torch.empty_like(x_buf))
        fb = torch.empty(m, 2 * W, device=x_buf.device, dtype=x_buf.dtype)
        hidden = torch.empty(m, 2 * W, device=x_buf.device, dtype=x_buf.dtype)
        upd = torch.empty(m, W, device=x_buf.device, dtype=x_buf.dtype)
        live_flat = live.reshape(-1)
        for i in range(count):
            p = f"{prefix}{i}."
            x = x_buf[:, :W]
            K.linear(x, w[p + "fb_t"], out=fb)
            K.graph_aggregate(fb, w[p + "rel"], ports, slots, x_buf[:, W:])
            if not self._fused_update(x_buf, w.get(p + "u0_k"), w[p + "u0_b"], hidden):
                K.linear(x_buf, w[p + "u0_t"], out=hidden)
                K.bias_gelu(hidden, w[p + "u0_b"])
            target = spare.pop(0)
            if not self._fused_update_norm(hidden, w.get(p + "u2_k"), w.get(p + "u2_bf"), x,
                                           w[p + "norm_w"], w[p + "norm_b"], live_flat,
                                           target[:, :W]):
                K.linear(hidden, w[p + "u2_t"], w[p + "u2_b"], out=upd)
                K.add_layernorm(x, upd, gamma=w[p + "norm_w"], beta=w[p + "norm_b"],
                                ln_out=target[:, :W], zero_row=live_flat)
            if not (keep_input and i == 0):
                spare.append(x_buf)
            x_buf = target
        return x_buf

    # rows from which the tensor-core GEMM with the fused GELU epilogue is used
    FUSED_MIN_ROWS = 4096

    def _fused_update(self, x: torch.Tensor, weight_k, bias, out: torch.Tensor) -> bool:
        """hidden = GELU(x @ u0^T + b) in one tensor-core pass (bf16, large
        batches); False when the caller must run the GEMM and bias+GELU
        separately (fp32 configuration, small batch, or a shape the kernel
        does not take)."""
        if weight_k is None or x.shape[0] < self.FUSED_MIN_ROWS:
            return False
        status = getattr(self, "kernel_status", None)
        if status is None:
            status = _status_word(x.device)
        code = K.gemm_bias_gelu(x, weight_k, bias, True, out, status)
        if code == -4:                       # GRS_ERR_SHAPE: nothing launched
            return False
        _lib.check(code, "tensor-core GEMM")
        return True

    def _fused_update_norm(self, hidden, weight_k, bias, residual, gamma, beta, zero_row,
                           out) -> bool:
        """out = LayerNorm(residual + hidden @ u2^T + b) (dead rows zeroed)
        in one tensor-core pass; False when the caller must run the GEMM and
        the add+LayerNorm separately."""
        if weight_k is None or hidden.shape[0] < self.FUSED_MIN_ROWS:
            return False
        status = getattr(self, "kernel_status", None)
        if status is None:
            status = _status_word(hidden.device)
        code = K.gemm_residual_layernorm(hidden, weight_k, bias, residual, gamma, beta, zero_row,
                                         out, status)
        if code == -4:                       # GRS_ERR_SHAPE: nothing launched
            return False
        _lib.check(code, "tensor-core GEMM + LayerNorm")
        return True

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
        q = K.linear(flat, w["naq_t"])
        query = q.view(b, s, h, W // h).transpose(1, 2)
        ctx = paged_attention(query, readout_key_cache, readout_value_cache, block_table, lengths)
        ctx2d = ctx.transpose(1, 2).reshape(b * s, W)
        u = K.linear(ctx2d, w["nao_t"])
        x_buf = torch.empty(b * s, 2 * W, device=states.device, dtype=states.dtype)
        lengths32 = lengths.to(torch.int32).contiguous()
        K.add_layernorm(flat, u, gamma=w["na_norm_w"], beta=w["na_norm_b"], ln_out=x_buf[:, :W],
                        zero_row=live_flat, where_len=lengths32, rows_per_beam=s)
        if not self.readout_graph_layers_count:
            return x_buf[:, :W].contiguous().view(b, s, W), live, gate_types
        if ports is None:
            if batch is None:
                raise ValueError("readout graph layers require an action-derived graph")
            ports = self._ports(batch, b, s, states.device)
        g = self._graph_layers("readout_graph", self.readout_graph_layers_count, x_buf, live,
                               ports, s, keep_input=True)
        proj = K.linear(g[:, :W], w["readout_graph_output_t"])
        out = torch.empty(b * s, W, device=states.device, dtype=states.dtype)
        K.add_layernorm(x_buf[:, :W], proj, sum_out=out, zero_row=live_flat, zero_before=True)
        return out.view(b, s, W), live, gate_types

    @torch.no_grad()
    def project_action_readout_kv(self, action_states):
        """Readout K/V of a new contextual action (paged_model.py:338-347)."""
        w = self.prepare()
        b = action_states.shape[0]
        shape = (b, self.action_heads, self.width // self.action_heads)
        a = action_states.to(self.compute_dtype).contiguous()
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
    GRAPH_CACHE_LIMIT = 16   # captured token-step graphs kept (least recently used dropped)

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
        hidden = K.bias_gelu(K.linear(ctx_in, w["ac0_t"]), w["ac0_b"])
        raw = K.linear(hidden, w["ac3_t"], w["ac3_b"])
        token = torch.empty_like(raw)
        K.position_token(raw, w["action_position"], past_lengths, active, token)
        valid = active
        new_keys = torch.empty(self.action_layers_count, b, h, hd, device=dev, dtype=dt)
        new_values = torch.empty_like(new_keys)
        ln = torch.empty_like(token)
        token2 = torch.empty_like(token)
        for layer in range(self.action_layers_count):
            p = f"causal{layer}."
            K.add_layernorm(token, gamma=w[p + "in_w"], beta=w[p + "in_b"], ln_out=ln)
            qkv = K.linear(ln, w[p + "qkv_t"]).view(b, 3, h, hd)
            q, k, v = qkv.unbind(1)
            ctx = paged_attention(q.unsqueeze(2), key_cache[layer], value_cache[layer],
                                  block_table, past_lengths, current_key=k, current_value=v,
                                  current_valid=valid)
            o = K.linear(ctx.reshape(b, W), w[p + "out_t"])
            K.add_layernorm(token, o, gamma=w[p + "ffn_norm_w"], beta=w[p + "ffn_norm_b"],
                            sum_out=token2, ln_out=ln)
            f0 = K.bias_gelu(K.linear(ln, w[p + "f0_t"]), w[p + "f0_b"])
            f3 = K.linear(f0, w[p + "f3_t"], w[p + "f3_b"])
            token = torch.empty_like(token2)
            K.add_layernorm(token2, f3, sum_out=token, zero_beam=active, zero_before=True)
            new_keys[layer].copy_(k)
            new_values[layer].copy_(v)
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
        key = (ctx_in.shape[0], block_table.shape[1], ctx_in.dtype, key_cache.data_ptr(),
               value_cache.data_ptr(), ctx_in.device)
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
        qxa = K.linear(flat, w["qxa_t"])                                   # [M, 3W]
        keys = K.linear(bound.view(b * pattern, W), w["bk_t"])             # [B*P, W]
        vw = K.linear(K.linear(bound.view(b * pattern, W), w["bv_t"]), w["d0b_t"])  # [B*P, 2W]
        cvec = K.linear(raw, w["d0c_t"], w["d0_b"])                         # [B, 2W]
        hidden = torch.empty(m, 2 * W, device=dev, dtype=dt)
        affinity = torch.empty(m, device=dev, dtype=torch.float32)
        K.update_live_hidden(qxa, keys, vw, cvec, source_mask, s, W, hidden, affinity)
        delta = K.linear(hidden, w["d3_t"], w["d3_b"])
        next_states = torch.empty_like(states)
        K.add_layernorm(flat, delta, scale=affinity, gamma=w["action_norm_w"],
                        beta=w["action_norm_b"], ln_out=next_states.view(m, W),
                        where_row=live.reshape(-1), where_beam=active, rows_per_beam=s)
        next_live = live.clone()
        next_types = gate_types.clone()
        dpattern = destination_slots.shape[1]
        r = K.linear(raw, w["ds0a_t"], w["ds0_b"])
        dh = torch.empty(b * dpattern, 2 * W, device=dev, dtype=dt)
        K.destination_hidden(r, w["ds_type_table"], w["ds_pos_table"], destination_slots,
                             destination_types, active, dh)
        created = K.linear(dh, w["ds2_t"], w["ds2_b"])
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
        node = K.linear(flat, w["retrieval_node_t"])
        sv_t = w["source_vectors_t"] if source_vectors is None else \
            source_vectors.t().contiguous().to(self.compute_dtype)
        acc = K.linear(node, sv_t)
        logits = torch.empty(b, s, self.num_sources, device=states.device, dtype=torch.float32)
        eligible = torch.empty(b, s, self.num_sources, device=states.device, dtype=torch.bool)
        K.match_logits(acc, w["source_bias"], w["first_types"], live.contiguous(),
                       gate_types.to(torch.int64).contiguous(), 1.0 / math.sqrt(self.retrieval_width),
                       logits, eligible)
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

"""Oracle of the paged action model (CPU, fp32, functional).

Restates ``PagedActionBindingModel`` (paged_model.py:97-777) and the parts of
``S0ActionBindingModel`` it inherits (model.py:12-478) over a parameter
dictionary keyed by the reference's ``state_dict`` names, so the same seeded
weights drive the reference, this oracle and the CUDA path.  Supported
options: ``readout_graph_input="cached"``, no ordered binding roles, no
locality features (the rollout configuration).

Each function cites the reference lines it follows.
"""
from __future__ import annotations

import math

import torch
import torch.nn.functional as F

from graph_rewrite_system_b200.synthetic import (ModelConfig, RuleMetadata, parameter_shapes,  # noqa: F401
                                                  parse_pattern)


def rule_buffers(rules: RuleMetadata) -> dict[str, torch.Tensor]:
    """Structural-decoder tables built from the source patterns (model.py:75-141)."""
    ns = rules.num_sources
    max_pattern = max(map(len, rules.source_gate_types))
    source_types = torch.full((ns, max_pattern), -1, dtype=torch.long)
    source_lengths = torch.zeros(ns, dtype=torch.long)
    for s, types in enumerate(rules.source_gate_types):
        source_types[s, : len(types)] = torch.tensor(types)
        source_lengths[s] = len(types)
    edge_rows, max_edges = [], 0
    for pattern in rules.source_patterns:
        wires: dict[int, list[tuple[int, int]]] = {}
        for op_index, op in enumerate(parse_pattern(pattern)):
            for port, qubit in enumerate(op.qubits):
                wires.setdefault(qubit, []).append((op_index, port))
        edges = [(a, b, pa, pb) for wire in wires.values()
                 for (a, pa), (b, pb) in zip(wire, wire[1:])]
        edge_rows.append(edges)
        max_edges = max(max_edges, len(edges))
    child = torch.full((ns, max_pattern), -1, dtype=torch.long)
    parent = torch.full_like(child, -1)
    parent_port = torch.full_like(child, -1)
    child_port = torch.full_like(child, -1)
    direction = torch.zeros_like(child)
    pattern_edges = torch.full((ns, max_edges, 4), -1, dtype=torch.long)
    for s, edges in enumerate(edge_rows):
        if edges:
            pattern_edges[s, : len(edges)] = torch.tensor(edges)
        mapped = {0}
        for step in range(int(source_lengths[s]) - 1):
            for a, b, pa, pb in edges:
                if a in mapped and b not in mapped:
                    child[s, step], parent[s, step] = b, a
                    parent_port[s, step], child_port[s, step] = pa, pb
                    direction[s, step] = 1
                    mapped.add(b)
                    break
                if b in mapped and a not in mapped:
                    child[s, step], parent[s, step] = a, b
                    parent_port[s, step], child_port[s, step] = pb, pa
                    direction[s, step] = -1
                    mapped.add(a)
                    break
    return dict(source_types=source_types, source_lengths=source_lengths,
                binding_child=child, binding_parent=parent, binding_parent_port=parent_port,
                binding_child_port=child_port, binding_direction=direction,
                pattern_edges=pattern_edges)


def _linear(x, p, name, bias=True):
    return F.linear(x, p[name + ".weight"], p.get(name + ".bias") if bias else None)


def _layer_norm(x, p, name):
    return F.layer_norm(x, (x.shape[-1],), p[name + ".weight"], p[name + ".bias"], 1e-5)


def _mlp(x, p, name, second_index):
    h = F.gelu(_linear(x, p, f"{name}.0"))
    return _linear(h, p, f"{name}.{second_index}")


class OracleModel:
    def __init__(self, params: dict[str, torch.Tensor], rules: RuleMetadata, cfg: ModelConfig):
        self.p = {k: v.float() for k, v in params.items()}
        self.rules, self.cfg = rules, cfg
        self.width = cfg.width
        self.heads = cfg.action_heads
        self.num_sources = rules.num_sources
        self.buf = rule_buffers(rules)
        self.max_pattern = self.buf["source_types"].shape[1]

    # ---- s0 and message passing ------------------------------------------
    def graph_layer(self, prefix, states, live, eb, es, ed, er):
        """InitialGraphLayer.forward (model.py:26-53)."""
        p = self.p
        b, s, w = states.shape
        flat = states.reshape(b * s, w)
        agg = torch.zeros_like(flat)
        deg = torch.zeros(b * s, 1)
        if eb.numel():
            si, di = eb * s + es, eb * s + ed
            fwd = F.linear(flat[si], p[prefix + "forward_message.weight"]) + \
                p[prefix + "relation.weight"][er]
            bwd = F.linear(flat[di], p[prefix + "backward_message.weight"]) + \
                p[prefix + "relation.weight"][er + 16]
            agg.index_add_(0, di, fwd)
            agg.index_add_(0, si, bwd)
            ones = torch.ones(si.numel(), 1)
            deg.index_add_(0, di, ones)
            deg.index_add_(0, si, ones)
        agg = (agg / deg.clamp_min(1.0)).view_as(states)
        h = torch.cat((states, agg), -1)
        upd = F.linear(F.gelu(F.linear(h, p[prefix + "update.0.weight"], p[prefix + "update.0.bias"])),
                       p[prefix + "update.2.weight"], p[prefix + "update.2.bias"])
        out = F.layer_norm(states + upd, (w,), p[prefix + "norm.weight"], p[prefix + "norm.bias"], 1e-5)
        return out * live.unsqueeze(-1)

    def initial_state(self, initial_types, eb, es, ed, er):
        """_initial_state (paged_model.py:243-260)."""
        live = initial_types.ge(0)
        states = self.p["gate_embedding.weight"][initial_types.clamp_min(0)] + self.p["initial_marker"]
        states = states * live.unsqueeze(-1)
        for i in range(self.cfg.graph_layers):
            states = self.graph_layer(f"graph_layers.{i}.", states, live, eb, es, ed, er)
        return states, live, initial_types.clone()

    def source_representations(self):
        """model.py:208-214."""
        p = self.p
        st = self.buf["source_types"]
        tokens = p["gate_embedding.weight"][st.clamp_min(0)] + \
            p["pattern_position.weight"][: self.max_pattern].unsqueeze(0)
        mask = st.ge(0).unsqueeze(-1)
        composed = (tokens * mask).sum(1) / mask.sum(1).clamp_min(1)
        return p["source_embedding.weight"] + _mlp(composed, p, "pattern_composer", 2)

    # ---- one action ---------------------------------------------------------
    def update_live_nodes(self, states, live, bound, source_mask, context, active):
        """paged_model.py:213-241."""
        p = self.p
        q = F.linear(states, p["node_query.weight"])
        k = F.linear(bound, p["binding_key.weight"])
        logits = torch.einsum("bsd,bkd->bsk", q, k) / math.sqrt(self.width)
        logits = logits.masked_fill(~source_mask.unsqueeze(1), -1e4)
        attn = logits.softmax(-1)
        local = torch.einsum("bsk,bkd->bsd", attn, F.linear(bound, p["binding_value.weight"]))
        affinity = logits.max(-1).values.sigmoid().unsqueeze(-1)
        expanded = context.unsqueeze(1).expand(-1, states.shape[1], -1)
        delta = _mlp(torch.cat((states, local, expanded), -1), p, "action_delta", 3)
        mask = live & active.unsqueeze(-1)
        updated = _layer_norm(states + affinity * delta, p, "action_norm")
        return torch.where(mask.unsqueeze(-1), updated, states)

    def action_context(self, states, xfer_ids, source_ids, source_slots, active):
        """Bound-slot pooling and action_context (paged_model.py:502-523)."""
        p = self.p
        source_mask = source_slots.ge(0) & active.unsqueeze(-1)
        bound = torch.gather(states, 1, source_slots.clamp_min(0).unsqueeze(-1)
                             .expand(-1, -1, self.width))
        pool = (bound * source_mask.unsqueeze(-1)).sum(1) / \
            source_mask.sum(1, keepdim=True).clamp_min(1)
        reps = self.source_representations()
        raw = _mlp(torch.cat((p["xfer_embedding.weight"][xfer_ids.clamp_min(0)],
                              reps[source_ids.clamp_min(0)], pool), -1), p, "action_context", 3)
        return raw, bound, source_mask

    def causal_step(self, layer, token, past_k, past_v, key_mask):
        """CausalActionLayer.forward_step (paged_model.py:37-64), dense past."""
        p, pre = self.p, f"causal_action_layers.{layer}."
        b, w = token.shape
        h, d = self.heads, w // self.heads
        qkv = F.linear(_layer_norm(token, p, pre + "input_norm"), p[pre + "qkv.weight"])
        q, k, v = qkv.view(b, 3, h, d).unbind(1)
        k, v = k.unsqueeze(2), v.unsqueeze(2)
        if past_k is not None:
            k = torch.cat((past_k, k), 2)
            v = torch.cat((past_v, v), 2)
        scores = torch.einsum("bhd,bhtd->bht", q, k) / math.sqrt(d)
        scores = scores.masked_fill(~key_mask.unsqueeze(1), -1e4)
        attn = F.softmax(scores.float(), -1)
        ctx = torch.einsum("bht,bhtd->bhd", attn, v).reshape(b, w)
        token = token + F.linear(ctx, p[pre + "output.weight"])
        token = token + _mlp(_layer_norm(token, p, pre + "ffn_norm"), p, pre + "ffn", 3)
        return token, k, v

    def apply_slots(self, states, live, types, source_slots, source_mask, destination_slots,
                    destination_types, active, raw):
        """Kill source slots, create destination slots (paged_model.py:569-604)."""
        p = self.p
        states, live, types = states.clone(), live.clone(), types.clone()
        rows = torch.arange(states.shape[0])
        for pos in range(source_slots.shape[1]):
            valid = source_mask[:, pos]
            if valid.any():
                r, s = rows[valid], source_slots[valid, pos]
                live[r, s] = False
                types[r, s] = -1
                states[r, s] = 0
        dmask = destination_slots.ge(0) & active.unsqueeze(-1)
        for pos in range(destination_slots.shape[1]):
            valid = dmask[:, pos]
            if not valid.any():
                continue
            r, s = rows[valid], destination_slots[valid, pos]
            t = destination_types[valid, pos]
            created = _mlp(torch.cat((raw[valid], p["gate_embedding.weight"][t],
                                      p["pattern_position.weight"][pos].expand(r.numel(), -1)), -1),
                           p, "destination_state", 2)
            states[r, s] = created
            live[r, s] = True
            types[r, s] = t
        return states, live, types

    def advance(self, states, live, types, past_k, past_v, past_len, *, xfer_ids, source_ids,
                source_slots, destination_slots, destination_types):
        """One action with a dense past (advance_incremental's non-paged branch,
        paged_model.py:444-613).  past_k/v: [L,B,H,T,D] or None; past_len: int
        (every row of the batch has that many past actions)."""
        p = self.p
        b = states.shape[0]
        active = xfer_ids.ge(0)
        ref = torch.cat((source_slots, destination_slots), 1)
        if ref.numel() and int(ref.max()) >= states.shape[1]:
            extra = int(ref.max()) + 1 - states.shape[1]
            states = F.pad(states, (0, 0, 0, extra))
            live = F.pad(live, (0, extra), value=False)
            types = F.pad(types, (0, extra), value=-1)
        raw, bound, source_mask = self.action_context(states, xfer_ids, source_ids, source_slots,
                                                      active)
        token = (raw + p["action_position.weight"][past_len]) * active.unsqueeze(-1)
        past_mask = torch.ones(b, past_len, dtype=torch.bool)
        key_mask = torch.cat((past_mask, active.unsqueeze(1)), 1)
        new_k, new_v = [], []
        for layer in range(self.cfg.action_layers):
            pk = None if past_k is None else past_k[layer]
            pv = None if past_v is None else past_v[layer]
            token, k, v = self.causal_step(layer, token, pk, pv, key_mask)
            token = token * active.unsqueeze(-1)
            new_k.append(k[:, :, -1])
            new_v.append(v[:, :, -1])
        token = _layer_norm(token, p, "action_output_norm") * active.unsqueeze(-1)
        states = self.update_live_nodes(states, live, bound, source_mask, raw, active)
        states, live, types = self.apply_slots(states, live, types, source_slots, source_mask,
                                               destination_slots, destination_types, active, raw)
        return states, live, types, torch.stack(new_k), torch.stack(new_v), token

    def project_readout_kv(self, action):
        """paged_model.py:338-347."""
        b = action.shape[0]
        shape = (b, self.heads, self.width // self.heads)
        return (F.linear(action, self.p["node_action_key.weight"]).view(shape),
                F.linear(action, self.p["node_action_value.weight"]).view(shape))

    # ---- readout ------------------------------------------------------------
    def fuse_action_history(self, states, live, history_k, history_v, lengths):
        """Node readout over projected action K/V (paged_model.py:349-379).
        history_k/v: [B, H, T, D] projected readout keys/values, lengths [B]."""
        p = self.p
        b, s, w = states.shape
        h, d = self.heads, w // self.heads
        q = F.linear(states, p["node_action_query.weight"]).view(b, s, h, d).transpose(1, 2)
        t = history_k.shape[2]
        mask = torch.arange(t).unsqueeze(0) < lengths.unsqueeze(1)
        if t:
            scores = torch.einsum("bhnd,bhtd->bhnt", q, history_k) / math.sqrt(d)
            scores = scores.masked_fill(~mask[:, None, None, :], float("-inf"))
            has = mask.any(1)
            scores = torch.where(has[:, None, None, None], scores, torch.zeros_like(scores))
            ctx = torch.einsum("bhnt,bhtd->bhnd", scores.softmax(-1), history_v)
            ctx = ctx * has[:, None, None, None]
        else:
            ctx = torch.zeros_like(q)
        ctx = ctx.transpose(1, 2).reshape(b, s, w)
        updated = _layer_norm(states + F.linear(ctx, p["node_action_output.weight"]), p,
                              "node_action_norm")
        states = torch.where(lengths[:, None, None].gt(0), updated, states)
        return states * live.unsqueeze(-1)

    def fuse_readout_graph(self, states, live, eb, es, ed, er):
        """paged_model.py:381-436 with readout_graph_input='cached'."""
        if not self.cfg.readout_graph_layers:
            return states
        g = states
        for i in range(self.cfg.readout_graph_layers):
            g = self.graph_layer(f"readout_graph_layers.{i}.", g, live, eb, es, ed, er)
        return (states + F.linear(g, self.p["readout_graph_output.weight"])) * live.unsqueeze(-1)

    def match_logits(self, states, live, types):
        """model.py:375-389."""
        p = self.p
        node = F.linear(states, p["retrieval_node.weight"])
        source = F.linear(self.source_representations(), p["retrieval_source.weight"])
        logits = torch.einsum("bsd,vd->bsv", node, source) / math.sqrt(self.cfg.retrieval_width)
        logits = logits + p["source_bias"]
        first = self.buf["source_types"][:, 0]
        eligible = live.unsqueeze(-1) & types.unsqueeze(-1).eq(first)
        return logits.masked_fill(~eligible, -1e4), eligible

    def structural_decode(self, types, live, edges, batch_ids, source_ids, anchors):
        """model.py:391-478.  edges = (batch, src, dst, relation)."""
        eb, es, ed, er = edges
        b, s = types.shape
        out_node = torch.full((b, s, 4), -1, dtype=torch.long)
        out_port = torch.full_like(out_node, -1)
        in_node = torch.full_like(out_node, -1)
        in_port = torch.full_like(out_node, -1)
        sp, dp = er // 4, er % 4
        out_node[eb, es, sp] = ed
        out_port[eb, es, sp] = dp
        in_node[eb, ed, dp] = es
        in_port[eb, ed, dp] = sp
        bf = self.buf
        n = batch_ids.numel()
        bindings = torch.full((n, self.max_pattern), -1, dtype=torch.long)
        bindings[:, 0] = anchors
        valid = live[batch_ids, anchors] & types[batch_ids, anchors].eq(bf["source_types"][source_ids, 0])
        rows = torch.arange(n)
        for step in range(self.max_pattern - 1):
            act = bf["source_lengths"][source_ids].gt(step + 1)
            cpos = bf["binding_child"][source_ids, step]
            ppos = bf["binding_parent"][source_ids, step]
            valid &= ~act | (ppos.ge(0) & cpos.ge(0))
            pslots = bindings[rows, ppos.clamp_min(0)].clamp_min(0)
            pports = bf["binding_parent_port"][source_ids, step].clamp_min(0)
            cports = bf["binding_child_port"][source_ids, step]
            fwd = bf["binding_direction"][source_ids, step].gt(0)
            cand = torch.where(fwd, out_node[batch_ids, pslots, pports], in_node[batch_ids, pslots, pports])
            cport = torch.where(fwd, out_port[batch_ids, pslots, pports], in_port[batch_ids, pslots, pports])
            ok = cand.ge(0) & cport.eq(cports)
            safe = cand.clamp_min(0)
            ok &= live[batch_ids, safe]
            ok &= types[batch_ids, safe].eq(bf["source_types"][source_ids, cpos.clamp_min(0)])
            ok &= ~bindings.eq(cand.unsqueeze(1)).any(1)
            valid &= ~act | ok
            ar = act.nonzero(as_tuple=False).squeeze(1)
            if ar.numel():
                bindings[ar, cpos[ar]] = cand[ar]
        pe = bf["pattern_edges"]
        for e in range(pe.shape[1]):
            edge = pe[source_ids, e]
            act = edge[:, 0].ge(0)
            ss = bindings[rows, edge[:, 0].clamp_min(0)].clamp_min(0)
            ds = bindings[rows, edge[:, 1].clamp_min(0)]
            ok = out_node[batch_ids, ss, edge[:, 2].clamp_min(0)].eq(ds)
            ok &= out_port[batch_ids, ss, edge[:, 2].clamp_min(0)].eq(edge[:, 3])
            valid &= ~act | ok
        return bindings, valid

    # ---- full prefix ----------------------------------------------------------
    def encode(self, batch: dict):
        """Full-prefix forward (paged_model.py:657-777): s0 message passing, every
        action through the causal layers with a dense past, slot kill/create,
        then the readout over the whole projected history and the readout graph."""
        states, live, types = self.initial_state(
            batch["initial_types"], batch["edge_batch"], batch["edge_src"], batch["edge_dst"],
            batch["edge_relation"])
        xfers = batch["action_xfers"]
        b, t = xfers.shape
        past_k = past_v = None
        tokens = []
        for a in range(t):
            states, live, types, nk, nv, token = self.advance(
                states, live, types, past_k, past_v, a, xfer_ids=xfers[:, a],
                source_ids=batch["action_sources"][:, a], source_slots=batch["binding_slots"][:, a],
                destination_slots=batch["destination_slots"][:, a],
                destination_types=batch["destination_types"][:, a])
            nk, nv = nk.unsqueeze(3), nv.unsqueeze(3)   # [L,B,H,1,D]
            past_k = nk if past_k is None else torch.cat((past_k, nk), 3)
            past_v = nv if past_v is None else torch.cat((past_v, nv), 3)
            tokens.append(token)
        if tokens:
            history = torch.stack(tokens, 1)
            rk, rv = self.project_readout_kv(history.reshape(b * t, -1))
            rk = rk.view(b, t, self.heads, -1).transpose(1, 2)
            rv = rv.view(b, t, self.heads, -1).transpose(1, 2)
            lengths = xfers.ge(0).sum(1)
            states = self.fuse_action_history(states, live, rk, rv, lengths)
        else:
            states = states * live.unsqueeze(-1)
        states = self.fuse_readout_graph(states, live, batch["current_edge_batch"],
                                         batch["current_edge_src"], batch["current_edge_dst"],
                                         batch["current_edge_relation"])
        return states, live, types

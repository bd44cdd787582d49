"""Oracle beam search on the CPU (fp32), the reference's loop restated.

Follows paged_rollout_benchmark.py:898-1207 with the decode-path settings of
the synthetic rollout (paged readout, tensorized state batches, GPU-style
proposals, indexed lazy topology, raw dedup, no refresh): per level,
readout + match logits (oracle.model), candidate selection and structural
decode (oracle.candidates), expansion / cap / rank (oracle.proposals), the
lazy-child accept loop (oracle.topology), then the one-token advance of the
accepted children with a dense per-beam history (equivalent to the paged
cache, whose bit-exactness is tested separately).
"""
from __future__ import annotations

import math

import numpy as np
import torch

from graph_rewrite_system_b200.synthetic import parse_pattern
from oracle import candidates as C
from oracle import proposals as PR
from oracle import topology as T


class _ModelBeam:
    """One model's per-beam state: slot states and the dense action history
    (causal K/V per layer, readout K/V) of every beam."""

    def __init__(self, model, states, live, types):
        self.model = model
        self.states, self.live, self.types = states, live, types
        self.past_k = self.past_v = None          # [L, B, H, T, D]
        self.hist_k = self.hist_v = None          # readout K/V [B, H, T, D]

    def logits(self, edges, depth):
        m, b = self.model, self.states.shape[0]
        lengths = torch.full((b,), depth, dtype=torch.long)
        if self.hist_k is not None:
            readout = m.fuse_action_history(self.states, self.live, self.hist_k, self.hist_v,
                                            lengths)
        else:
            readout = self.states * self.live.unsqueeze(-1)
        readout = m.fuse_readout_graph(readout, self.live, *edges)
        return m.match_logits(readout, self.live, self.types)

    def advance(self, parents, xfers, sources, src_slots, dst_slots, dst_types, new_s, depth):
        s = self.states.shape[1]
        states = self.states[parents]
        live, types = self.live[parents], self.types[parents]
        if new_s > s:
            states = torch.nn.functional.pad(states, (0, 0, 0, new_s - s))
            live = torch.nn.functional.pad(live, (0, new_s - s), value=False)
            types = torch.nn.functional.pad(types, (0, new_s - s), value=-1)
        pk = None if self.past_k is None else self.past_k[:, parents]
        pv = None if self.past_v is None else self.past_v[:, parents]
        states, live, types, nk, nv, token = self.model.advance(
            states, live, types, pk, pv, depth, xfer_ids=xfers, source_ids=sources,
            source_slots=src_slots, destination_slots=dst_slots, destination_types=dst_types)
        rk, rv = self.model.project_readout_kv(token)
        nk, nv = nk.unsqueeze(3), nv.unsqueeze(3)
        self.past_k = nk if pk is None else torch.cat((pk, nk), 3)
        self.past_v = nv if pv is None else torch.cat((pv, nv), 3)
        hk = None if self.hist_k is None else self.hist_k[parents]
        hv = None if self.hist_v is None else self.hist_v[parents]
        self.hist_k = rk.unsqueeze(2) if hk is None else torch.cat((hk, rk.unsqueeze(2)), 2)
        self.hist_v = rv.unsqueeze(2) if hv is None else torch.cat((hv, rv.unsqueeze(2)), 2)
        self.states, self.live, self.types = states, live, types


class OracleBeamSearch:
    def __init__(self, model, rules, circuit, config, thresholds, *, exploration_model=None,
                 exploration_thresholds=None, exploration_per_parent=0,
                 exploration_until_depth=0):
        """With `exploration_model`, a second model proposes alongside under a
        per-parent quota (build_legacy_proposals, paged_rollout_benchmark.py
        :101-210), advances with every child (:1071-1091) and leaves the
        search from level `exploration_until_depth` on (0: never, :900-911)."""
        self.model, self.rules, self.circuit, self.cfg = model, rules, circuit, config
        self.thresholds = thresholds
        self.exploration_model = exploration_model
        self.exploration_thresholds = exploration_thresholds or thresholds
        self.exploration_per_parent = exploration_per_parent
        self.exploration_until_depth = exploration_until_depth
        self.src = [parse_pattern(p) for p in rules.xfer_sources]
        self.dst = [parse_pattern(p) for p in rules.xfer_destinations]
        self.index = PR.build_rule_index(rules.source_to_xfers(), rules.gate_deltas(),
                                         rules.num_sources, config.max_gate_increase)
        self.slot_cap = max(s for s, _ in circuit.nodes) + 1 + config.depth * 4 + 8

    def reset(self):
        nodes = dict(self.circuit.nodes)
        s0 = max(nodes) + 1
        types = torch.full((1, s0), -1, dtype=torch.long)
        for s, g in nodes.items():
            types[0, s] = g
        e = torch.tensor(self.circuit.edges, dtype=torch.long).reshape(-1, 4)
        args = (types, torch.zeros(e.shape[0], dtype=torch.long), e[:, 0], e[:, 1],
                e[:, 2] * 4 + e[:, 3])
        self.primary = _ModelBeam(self.model, *self.model.initial_state(*args))
        self.exploration = None
        if self.exploration_model is not None:
            self.exploration = _ModelBeam(self.exploration_model,
                                          *self.exploration_model.initial_state(*args))
        self.beam = [T.initial_beam(nodes, [tuple(x) for x in self.circuit.edges], self.slot_cap)]
        self.seen = {self.beam[0].topology.fingerprint}
        self.rows = []

    # the primary model's state under the names the tests read
    @property
    def states(self):
        return self.primary.states

    def _edges(self):
        eb, es, ed, er = [], [], [], []
        for b, node in enumerate(self.beam):
            for s, d, sp, dp in sorted(node.topology.edges):
                eb.append(b); es.append(s); ed.append(d); er.append(sp * 4 + dp)
        t = lambda x: torch.tensor(x, dtype=torch.long)
        return t(eb), t(es), t(ed), t(er)

    def _candidates(self, side, thresholds, edges, distance, depth):
        logits, eligible = side.logits(edges, depth)
        return C.threshold_candidates(side.model, side.types, side.live, distance, edges, logits,
                                      eligible, thresholds,
                                      max_candidates_per_state=self.cfg.max_candidates_per_state)

    def step(self):
        cfg = self.cfg
        b = len(self.beam)
        depth = self.beam[0].depth
        if (self.exploration is not None and self.exploration_until_depth
                and depth >= self.exploration_until_depth):
            self.exploration = None
        s = self.primary.states.shape[1]
        edges = self._edges()
        distance = torch.stack([torch.from_numpy(n.rewrite_distance[:s]) for n in self.beam])
        cand = self._candidates(self.primary, self.thresholds, edges, distance, depth)
        cap = max(cfg.per_parent_cap, math.ceil(cfg.beam_size / max(1, b)) * 2)
        gates = np.array([n.gate_count for n in self.beam], np.int64)
        np_ = lambda d: {k: v.numpy() for k, v in d.items()}
        x_metrics = {}
        if self.exploration is not None:
            cand_x = self._candidates(self.exploration, self.exploration_thresholds, edges,
                                      distance, depth)
            sel, metrics = PR.rank_proposals_exploration(
                np_(cand), np_(cand_x), gates, self.index, per_parent_cap=cap,
                exploration_per_parent=self.exploration_per_parent, global_cap=cfg.global_cap)
            bindings = sel["binding"]
            x_metrics = {k: metrics[k] for k in ("exploration_predicted_actions",
                                                 "exploration_eligible_actions",
                                                 "selected_exploration_proposals")}
        else:
            sel, metrics = PR.rank_proposals(cand["batch_ids"].numpy(), cand["sources"].numpy(),
                                             cand["anchors"].numpy(), cand["bindings"].numpy(),
                                             cand["probabilities"].numpy(), gates, self.index,
                                             per_parent_cap=cap, global_cap=cfg.global_cap)
            bindings = [tuple(int(x) for x in row if x >= 0) for row in sel["binding"]]
        proposals = []
        for i in range(len(sel["parent"])):
            proposals.append((int(sel["parent"][i]), int(sel["xfer"][i]), int(sel["anchor"][i]),
                              tuple(bindings[i]), int(sel["next_gate"][i])))
        records, acc = T.accept(self.beam, proposals, self.src, self.dst, self.seen,
                                cfg.beam_size, self.slot_cap)
        row = {"step": depth + 1, "input_states": b, "accepted_actions": len(records),
               "attempted_actions": acc["attempted"],
               "invalid_structural_actions": acc["invalid"],
               "duplicate_speculative_successors": acc["duplicates"],
               "proposals_after_caps": len(proposals),
               "predicted_actions": metrics["predicted_actions"],
               "eligible_actions_before_parent_cap": metrics["eligible_actions"],
               "children": [(proposals[j][0], proposals[j][1], proposals[j][3]) for _, j in records],
               **x_metrics}
        self.rows.append(row)
        if not records:
            return None
        # advance the accepted children
        parents = torch.tensor([proposals[j][0] for _, j in records], dtype=torch.long)
        xfers = torch.tensor([proposals[j][1] for _, j in records], dtype=torch.long)
        sources = torch.tensor([self.rules.xfer_to_source[x] for x in xfers.tolist()],
                               dtype=torch.long)
        maxp = max(len(x) for x in self.rules.source_gate_types)
        maxd = max(max(len(x) for x in self.rules.destination_gate_types), 1)
        src_slots = torch.full((len(records), maxp), -1, dtype=torch.long)
        dst_slots = torch.full((len(records), maxd), -1, dtype=torch.long)
        dst_types = torch.full_like(dst_slots, -1)
        for i, (child, j) in enumerate(records):
            binding = proposals[j][3]
            src_slots[i, : len(binding)] = torch.tensor(binding)
            dest = child.history[-1][2]
            if dest:
                dst_slots[i, : len(dest)] = torch.tensor(dest)
                dst_types[i, : len(dest)] = torch.tensor(self.rules.destination_gate_types[xfers[i]])
        new_s = max(max(c.next_slot for c, _ in records), s)
        for side in (self.primary, self.exploration):
            if side is not None:
                side.advance(parents, xfers, sources, src_slots, dst_slots, dst_types, new_s, depth)
        self.beam = [c for c, _ in records]
        return row

    def run(self, depth=None):
        self.reset()
        for _ in range(depth or self.cfg.depth):
            if self.step() is None:
                break
        return self.rows

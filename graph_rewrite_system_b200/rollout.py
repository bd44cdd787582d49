"""Device-resident beam search: the loop of paged_rollout_benchmark.py:898-1207
without Quartz (no exact refresh or audit), every stage on the GPU.

One search level (``step``):

1. paged node readout + readout graph over the device port graph
   (paged_model_matches, :243-386; replaces the host collation of
   tensorized_batch.py);
2. match logits, near/far threshold, per-state top-k and structural decode
   into a padded candidate table (threshold_candidate_tensors);
3. expansion, per-parent cap and global rank (build_gpu_proposals);
4. rewrite planning with XOR fingerprints, first-occurrence dedup against
   the global seen set, accept the first beam_size, stable sort by gate count
   (the lazy_child accept loop, :1013-1046);
5. child topology materialisation with the BFS rewrite distance;
6. one-token model advance of the children, readout K/V projection, paged
   cache append (fork/COW) and release of the parents (advance_selected,
   :390-556).

The host synchronises once per level, after the accept, to read a small
summary (accepted count, metrics, the next slot extent) that sizes the next
launches.
"""
from __future__ import annotations

from dataclasses import dataclass
import math
import time

import torch

from . import _lib
from . import kernels as K
from .gpu_proposals import (GROUPED_MAX_EXPANSION, GpuRuleIndex, RankedProposals,
                            rank_proposals_device, rank_proposals_exploration,
                            rank_proposals_grouped)
from .paged_cache import PagedKVCache
from .paged_model import PagedActionBindingModel
from .synthetic import (Circuit, RolloutConfig, RuleMetadata, SELECT_ALL_THRESHOLDS)
from .threshold_inference import select_candidates_device
from .topology import TopologyBuffers, initial_topology, xfer_table


def _round_up(v: int, m: int) -> int:
    return (v + m - 1) // m * m


def _pow2_at_least(v: int) -> int:
    return 1 << max(1, int(v - 1).bit_length())


@dataclass
class StepRow:
    """Per-level record with the reference's step-row field names (:1239-1276)."""

    step: int
    input_states: int
    output_states: int
    best_speculative_gate_count: int
    predicted_actions: int
    eligible_actions_before_parent_cap: int
    proposals_after_caps: int
    attempted_actions: int
    accepted_actions: int
    invalid_structural_actions: int
    duplicate_speculative_successors: int
    allocated_cache_pages: int
    logical_cache_pages: int
    page_sharing_ratio: float
    exploration_predicted_actions: int = 0
    exploration_eligible_actions: int = 0
    selected_exploration_proposals: int = 0


@dataclass
class Proposed:
    """Ranked and planned proposals of one GPU's beams at one level."""

    ranked: "RankedProposals"
    cand: dict
    valid: torch.Tensor          # uint8 [global_cap] structurally valid
    fp: torch.Tensor             # int64 [global_cap] child fingerprint
    k: int                       # candidate rows per parent
    exploration_metrics: torch.Tensor | None = None   # int64 [3] while a second model runs


class StageTimer:
    """CUDA events at stage boundaries on the current stream (the device-side
    counterpart of the reference's --profile-stages, :268-273)."""

    def __init__(self):
        self.marks: list[tuple[str, torch.cuda.Event, float]] = []
        self.totals: dict[str, float] = {}
        self.host_totals: dict[str, float] = {}     # host time spent issuing each stage

    def mark(self, name: str) -> None:
        event = torch.cuda.Event(enable_timing=True)
        event.record()
        self.marks.append((name, event, time.perf_counter()))

    def collect(self) -> None:
        """Accumulate the closed intervals (call after a synchronisation)."""
        for (name, start, h0), (_, end, h1) in zip(self.marks, self.marks[1:]):
            self.totals[name] = self.totals.get(name, 0.0) + start.elapsed_time(end)
            self.host_totals[name] = self.host_totals.get(name, 0.0) + (h1 - h0) * 1e3
        self.marks = self.marks[-1:] if self.marks else []

    def reset(self) -> None:
        self.marks, self.totals, self.host_totals = [], {}, {}


class DeviceBeamSearch:
    """Beam search over rewrite sequences with the state resident in HBM."""

    def __init__(self, model: PagedActionBindingModel, rules: RuleMetadata, circuit: Circuit,
                 config: RolloutConfig, device, thresholds: dict = SELECT_ALL_THRESHOLDS, *,
                 exploration_model: PagedActionBindingModel | None = None,
                 exploration_thresholds: dict | None = None, exploration_per_parent: int = 0,
                 exploration_until_depth: int = 0):
        """`exploration_model`: a second paged model searched alongside (the
        reference's --exploration-checkpoint, paged_rollout_benchmark.py
        :724-758): it reads the same beams from its own paged cache, its
        candidates fill up to `exploration_per_parent` of every parent's
        proposals (build_legacy_proposals, :101-210), it advances with every
        accepted child, and it is dropped from level `exploration_until_depth`
        on (0: never, :900-911)."""
        self.model, self.rules, self.circuit, self.cfg = model, rules, circuit, config
        self.device = torch.device(device)
        self.thresholds = thresholds
        if exploration_per_parent < 0 or exploration_until_depth < 0:
            raise ValueError("the exploration quota and depth must be nonnegative")
        if exploration_per_parent and exploration_model is None:
            raise ValueError("an exploration checkpoint is required for an exploration quota")
        if exploration_per_parent > config.per_parent_cap:
            raise ValueError("the exploration quota cannot exceed the per-parent cap")
        if exploration_model is not None and (
                exploration_model.width != model.width
                or exploration_model.action_layers_count != model.action_layers_count
                or exploration_model.action_heads != model.action_heads):
            raise ValueError("primary and exploration paged-cache shapes differ")
        self.exploration_model = exploration_model
        self.exploration_thresholds = exploration_thresholds or thresholds
        self.exploration_per_parent = exploration_per_parent
        self.exploration_until_depth = exploration_until_depth
        dev = self.device
        self.s0_slots = max(s for s, _ in circuit.nodes) + 1
        self.max_dst = max(len(d) for d in rules.destination_gate_types)
        self.max_src = max(len(s) for s in rules.source_gate_types)
        self.slot_cap = _round_up(self.s0_slots + config.depth * max(self.max_dst, 1), 8)
        self.topology = [TopologyBuffers(config.beam_size, self.slot_cap, dev) for _ in range(2)]
        self.table = xfer_table(rules, dev)
        self.xfer_to_source = torch.tensor(rules.xfer_to_source, device=dev, dtype=torch.int64)
        self.rule_index = GpuRuleIndex.build(rules.source_to_xfers(), rules.gate_deltas(),
                                             rules.num_sources, config.max_gate_increase, dev)
        hd = model.width // model.action_heads
        self.cache = PagedKVCache(layers=model.action_layers_count, capacity=config.cache_pages,
                                  page_size=config.page_size, heads=model.action_heads,
                                  head_width=hd, model_width=model.width, device=dev,
                                  dtype=model.compute_dtype)
        self.seen_capacity = _pow2_at_least(4 * (1 + config.depth * config.beam_size))
        self.step_capacity = _pow2_at_least(2 * config.global_cap)
        self.seen = torch.zeros(self.seen_capacity, device=dev, dtype=torch.int64)
        self.step_keys = torch.empty(self.step_capacity, device=dev, dtype=torch.int64)
        self.step_first = torch.empty(self.step_capacity, device=dev, dtype=torch.int32)
        self.status = torch.zeros(1, device=dev, dtype=torch.int32)
        # the model's tensor-core kernels report into the level's status word
        model.kernel_status = self.status
        self.exploration_cache = None
        if exploration_model is not None:
            exploration_model.kernel_status = self.status
            self.exploration_cache = PagedKVCache(
                layers=model.action_layers_count, capacity=config.cache_pages,
                page_size=config.page_size, heads=model.action_heads, head_width=hd,
                model_width=model.width, device=dev, dtype=exploration_model.compute_dtype)
        self.exploring = False
        self.summary = torch.zeros(6, device=dev, dtype=torch.int64)
        self.rows: list[StepRow] = []
        self.timer: StageTimer | None = None
        self.validate = False

    def _check_range(self, stage: str, name: str, t: torch.Tensor, low: int, high: int,
                     allow_negative_one: bool = False) -> None:
        """Validation mode: every index a later kernel dereferences is in range."""
        if not self.validate or t.numel() == 0:
            return
        torch.cuda.synchronize(self.device)
        v = t.long()
        if allow_negative_one:
            v = v[v != -1]
            if v.numel() == 0:
                return
        lo, hi = int(v.min().item()), int(v.max().item())
        if lo < low or hi >= high:
            raise RuntimeError(f"validation: {stage}: {name} in [{lo}, {hi}] outside "
                               f"[{low}, {high}) at depth {self.depth}")

    def _check_tables(self, stage: str, table: torch.Tensor, lengths: torch.Tensor) -> None:
        if not self.validate:
            return
        torch.cuda.synchronize(self.device)
        page = self.cfg.page_size
        cols = table.shape[1]
        need = (lengths.long() + page - 1) // page
        if int(need.max().item()) > cols:
            raise RuntimeError(f"validation: {stage}: lengths need {int(need.max())} blocks, "
                               f"table has {cols}")
        mask = torch.arange(cols, device=table.device).unsqueeze(0) < need.unsqueeze(1)
        used = table[mask]
        self._check_range(stage, "page id", used, 0, self.cache.capacity)

    def _mark(self, name: str) -> None:
        if self.timer is not None:
            self.timer.mark(name)

    # ---- state ---------------------------------------------------------------
    @torch.no_grad()
    def reset(self) -> None:
        """Beam = [s0] with an empty prefix (paged_rollout_benchmark.py:774-856)."""
        dev, model = self.device, self.model
        nodes, edges = self.circuit.nodes, self.circuit.edges
        s = _round_up(self.s0_slots, 8)
        types = torch.full((1, s), -1, dtype=torch.int64)
        for slot, gate in nodes:
            types[0, slot] = gate
        e = torch.tensor(edges, dtype=torch.int64).reshape(-1, 4)
        batch = {"initial_types": types.to(dev),
                 "edge_batch": torch.zeros(e.shape[0], dtype=torch.int64, device=dev),
                 "edge_src": e[:, 0].to(dev), "edge_dst": e[:, 1].to(dev),
                 "edge_relation": (e[:, 2] * 4 + e[:, 3]).to(dev)}
        self.states, self.live, self.types = model.initialize_incremental(batch)
        self.exploring = self.exploration_model is not None
        if self.exploring:
            self.x_states, self.x_live, self.x_types = \
                self.exploration_model.initialize_incremental(batch)
            self.exploration_cache.reset()
            self.x_block_table = torch.zeros(1, 1, device=dev, dtype=torch.int32)
            self.x_lengths = torch.zeros(1, device=dev, dtype=torch.int32)
        self.topo = initial_topology(self.topology[0], nodes, edges, s)
        self.cache.reset()
        self.current = 0
        self.block_table = torch.zeros(1, 1, device=dev, dtype=torch.int32)
        self.lengths = torch.zeros(1, device=dev, dtype=torch.int32)
        self.seen.zero_()
        _lib.check(_lib.lib().grs_topology_seen_insert(
            self.topo.fingerprint.data_ptr(), 1, self.seen.data_ptr(), self.seen_capacity,
            self.status.data_ptr(), K.stream()), "seen_insert")
        self.beams, self.slots, self.depth = 1, s, 0
        self.rows = []

    # ---- one level --------------------------------------------------------------
    @torch.no_grad()
    def step(self) -> StepRow | None:
        with K.pinned_stream():
            return self._step()

    def _drop_exploration(self) -> None:
        """The second model leaves the search (paged_rollout_benchmark.py:900-911)."""
        self.exploration_cache.release_device(self.x_block_table, self.x_lengths)
        self.x_states = self.x_live = self.x_types = None
        self.exploring = False

    def _step(self) -> StepRow | None:
        cfg, dev = self.cfg, self.device
        b, s, depth = self.beams, self.slots, self.depth
        if self.exploring and self.exploration_until_depth and depth >= self.exploration_until_depth:
            self._drop_exploration()
        prop = self._propose()
        # 4. accept (first occurrence of unseen valid fingerprints, in rank order)
        gcap = cfg.global_cap
        classes = torch.empty(gcap, device=dev, dtype=torch.uint8)
        child_proposal = torch.empty(cfg.beam_size, device=dev, dtype=torch.int64)
        self._mark("accept")
        _lib.check(_lib.lib().grs_topology_accept(
            gcap, prop.ranked.count.data_ptr(), prop.valid.data_ptr(), prop.fp.data_ptr(),
            prop.ranked.next_gate.data_ptr(), cfg.beam_size, self.step_keys.data_ptr(),
            self.step_first.data_ptr(), self.step_capacity, self.seen.data_ptr(),
            self.seen_capacity, classes.data_ptr(), child_proposal.data_ptr(),
            self.summary.data_ptr(), prop.ranked.rows.data_ptr(), prop.ranked.xfer_ids.data_ptr(),
            prop.cand["batch_ids"].data_ptr(), self.table.data_ptr(),
            self.topo.next_slot.data_ptr(), self.status.data_ptr(), K.stream()),
            "topology_accept")
        # one synchronisation per level
        self._mark("host_sync")
        parts = [self.summary, prop.ranked.count, prop.ranked.metrics,
                 self.cache.allocated_pages_tensor().long(), self.status.long(),
                 self.cache.status_tensor().long()]
        if prop.exploration_metrics is not None:
            parts += [prop.exploration_metrics, self.exploration_cache.status_tensor().long()]
        host = torch.cat(parts).cpu().tolist()
        (accepted, attempted, invalid, dup, extent, best, proposals, predicted, eligible_n,
         allocated, status, cache_status) = host[:12]
        x_metrics = host[12:15] if prop.exploration_metrics is not None else [0, 0, 0]
        if prop.exploration_metrics is not None and host[15]:
            self.exploration_cache.check_status()
        if status:
            self.status.zero_()
            _lib.check(int(status), "beam search step")
        if cache_status:
            self.cache.check_status()
        row = StepRow(depth + 1, b, accepted, best, predicted, eligible_n, proposals, attempted,
                      accepted, invalid, dup, allocated, 0, 0.0, *x_metrics)
        if not accepted:
            self.rows.append(row)
            return None
        s_new = max(s, _round_up(int(extent), 8))
        self._children(prop, child_proposal, self.summary, accepted, s_new)
        row.logical_cache_pages = accepted * self.block_table.shape[1]
        self._mark("end")
        self.rows.append(row)
        return row

    def _propose(self) -> "Proposed":
        """Stages 1-3 and the rewrite plan for the current beams."""
        cfg, model, dev = self.cfg, self.model, self.device
        b, s = self.beams, self.slots
        topo = self.topo
        ports = topo.ports()
        for name, t in zip(("in_node", "in_port", "out_node", "out_port"), ports):
            self._check_range("step start", name, t, 0, s if "node" in name else 4,
                              allow_negative_one=True)
        self._check_tables("step start", self.block_table, self.lengths)
        # 1-2. readout and match logits
        self._mark("readout")
        readout, _, _ = model.readout_incremental(
            self.states, self.live, self.types, readout_key_cache=self.cache.readout_keys,
            readout_value_cache=self.cache.readout_values, block_table=self.block_table,
            lengths=self.lengths, ports=ports)
        self._mark("match_logits")
        logits, eligible = model.match_logits(readout, self.live, self.types)
        self._mark("candidates")
        cand = select_candidates_device(model, self.types, self.live, ports, topo.distance, logits,
                                        eligible, self.thresholds, cfg.max_candidates_per_state)
        self._check_range("candidates", "anchor", cand["anchors"], 0, s)
        self._check_range("candidates", "source", cand["sources"], 0, self.rules.num_sources,
                          allow_negative_one=True)
        self._check_range("candidates", "binding", cand["bindings"], 0, s, allow_negative_one=True)
        cand_x = None
        if self.exploring:   # the second model's candidates on the same beams
            xm = self.exploration_model
            x_readout, _, _ = xm.readout_incremental(
                self.x_states, self.x_live, self.x_types,
                readout_key_cache=self.exploration_cache.readout_keys,
                readout_value_cache=self.exploration_cache.readout_values,
                block_table=self.x_block_table, lengths=self.x_lengths, ports=ports)
            x_logits, x_eligible = xm.match_logits(x_readout, self.x_live, self.x_types)
            cand_x = select_candidates_device(xm, self.x_types, self.x_live, ports, topo.distance,
                                              x_logits, x_eligible, self.exploration_thresholds,
                                              cfg.max_candidates_per_state)
        # 3. proposals (effective parent cap of paged_rollout_benchmark.py:963-966)
        cap = self.parent_cap()
        self._mark("proposals")
        k = cand["sources"].numel() // b
        x_metrics = None
        if cand_x is not None:
            # build_legacy_proposals with the exploration quota; the ranked
            # rows index the primary then the exploration candidate rows
            ranked, m5 = rank_proposals_exploration(
                cand, cand_x, topo.gate, self.rule_index, per_parent_cap=cap,
                exploration_per_parent=self.exploration_per_parent, global_cap=cfg.global_cap,
                status=self.status)
            x_metrics = m5[2:]
            cand = {key: torch.cat((cand[key], cand_x[key])) for key in cand}
        elif cap <= GROUPED_MAX_EXPANSION:
            ranked = rank_proposals_grouped(cand["sources"], cand["probabilities"], k, topo.gate,
                                            self.rule_index, per_parent_cap=cap,
                                            global_cap=cfg.global_cap, status=self.status)
        else:
            # few parents and a wide beam (the first levels): the general
            # expansion path takes any cap
            ranked = rank_proposals_device(cand["batch_ids"], cand["sources"],
                                           cand["probabilities"], topo.gate, self.rule_index,
                                           per_parent_cap=cap, global_cap=cfg.global_cap,
                                           status=self.status)
        self._check_range("proposals", "row", ranked.rows, 0, cand["sources"].numel(),
                          allow_negative_one=True)
        self._check_range("proposals", "xfer", ranked.xfer_ids, 0, self.rules.num_xfers,
                          allow_negative_one=True)
        # 4a. rewrite plan: validity and child fingerprint of every ranked proposal
        gcap = cfg.global_cap
        valid = torch.empty(gcap, device=dev, dtype=torch.uint8)
        fp = torch.empty(gcap, device=dev, dtype=torch.int64)
        cb = cand["bindings"]
        self._mark("plan")
        _lib.check(_lib.lib().grs_topology_plan(
            gcap, ranked.count.data_ptr(), ranked.rows.data_ptr(), ranked.xfer_ids.data_ptr(),
            ranked.next_gate.data_ptr(), cand["batch_ids"].data_ptr(), cb.data_ptr(), cb.shape[1],
            self.table.data_ptr(), topo.types.data_ptr(), topo.out_node.data_ptr(),
            topo.out_port.data_ptr(), topo.in_node.data_ptr(), topo.in_port.data_ptr(), s,
            topo.next_slot.data_ptr(), topo.fingerprint.data_ptr(), valid.data_ptr(), fp.data_ptr(),
            self.status.data_ptr(), K.stream()), "topology_plan")
        return Proposed(ranked, cand, valid, fp, k, x_metrics)

    def global_beams(self) -> int:
        """Beams of the whole search at this level (this GPU's beams here)."""
        return self.beams

    def parent_cap(self) -> int:
        """The effective per-parent proposal cap of paged_rollout_benchmark.py:963-966."""
        return max(self.cfg.per_parent_cap,
                   math.ceil(self.cfg.beam_size / max(1, self.global_beams())) * 2)

    def _children(self, prop: "Proposed", child_proposal: torch.Tensor, summary: torch.Tensor,
                  accepted: int, s_new: int) -> None:
        """Stages 5-6 for `accepted` children given as indices into the ranked
        proposals of this GPU: child topology, model advance, cache append,
        release of the parents.  Replaces the beam state."""
        cfg, model, dev = self.cfg, self.model, self.device
        b, s, depth = self.beams, self.slots, self.depth
        topo, ranked, cand, fp = self.topo, prop.ranked, prop.cand, prop.fp
        cb = cand["bindings"]
        i64 = dict(device=dev, dtype=torch.int64)
        # 5. child topology
        self._mark("materialize")
        nxt = self.topology[1 - self.current].state(accepted, s_new)
        acts = self._materialize(accepted, child_proposal, summary, ranked.rows, ranked.xfer_ids,
                                 ranked.next_gate, fp, cand["batch_ids"], cand["anchors"], cb,
                                 topo, s, nxt, s_new)
        a_parent, a_xfer, a_source, a_src, a_dst, a_dst_types = acts
        self._check_range("materialize", "parent", a_parent, 0, b)
        self._check_range("materialize", "source slot", a_src, 0, s, allow_negative_one=True)
        self._check_range("materialize", "destination slot", a_dst, 0, s_new,
                          allow_negative_one=True)
        for name, t in zip(("in_node", "in_port", "out_node", "out_port"), nxt.ports()):
            self._check_range("materialize", name, t, 0, s_new if "node" in name else 4,
                              allow_negative_one=True)
        # 6. model advance of the children, cache append, release the parents
        self._mark("advance")
        w = model.width
        states_par = torch.empty(accepted, s_new, w, device=dev, dtype=model.compute_dtype)
        K.gather_beams(self.states, a_parent, states_par)
        live_par = torch.empty(accepted, s_new, device=dev, dtype=torch.bool)
        K.gather_beams(self.live, a_parent, live_par)
        types_par = torch.empty(accepted, s_new, **i64)
        K.gather_beams(self.types, a_parent, types_par, fill_byte=0xFF)
        table_par = torch.empty(accepted, self.block_table.shape[1], device=dev, dtype=torch.int32)
        K.gather_beams(self.block_table, a_parent, table_par)
        lengths_par = torch.empty(accepted, device=dev, dtype=torch.int32)
        K.gather_beams(self.lengths, a_parent, lengths_par)
        self._check_tables("advance", table_par, lengths_par)
        states, live, types, new_k, new_v, action, rk, rv = model.advance_device(
            states_par, live_par, types_par, a_xfer, a_source, a_src, a_dst, a_dst_types,
            self.cache.keys, self.cache.values, table_par, lengths_par,
            return_readout_kv=True, graphed=True)
        self._mark("cache_append_release")
        child_cols = -(-(depth + 1) // cfg.page_size)
        child_table, child_lengths = self.cache.append_device(
            table_par, lengths_par, new_k, new_v, action, rk, rv, child_cols=child_cols)
        self._check_tables("append", child_table, child_lengths)
        self.cache.release_device(self.block_table, self.lengths)
        if self.exploring:   # the second model advances with the same children
            self._advance_exploration(a_parent, a_xfer, a_source, a_src, a_dst, a_dst_types,
                                      accepted, s_new, child_cols)
        self.states, self.live, self.types = states, live, types
        self.block_table, self.lengths = child_table, child_lengths
        self.topo, self.current = nxt, 1 - self.current
        self.last_actions = (a_parent, a_xfer, a_src, a_dst)
        self.beams, self.slots, self.depth = accepted, s_new, depth + 1

    def _advance_exploration(self, a_parent, a_xfer, a_source, a_src, a_dst, a_dst_types,
                             n: int, s_new: int, child_cols: int) -> None:
        """advance_selected for the exploration model (paged_rollout_benchmark.py:1071-1091):
        its parents' rows, one-token step, append to its cache, release its parents."""
        xm, dev, w = self.exploration_model, self.device, self.model.width
        states_par = torch.empty(n, s_new, w, device=dev, dtype=xm.compute_dtype)
        K.gather_beams(self.x_states, a_parent, states_par)
        live_par = torch.empty(n, s_new, device=dev, dtype=torch.bool)
        K.gather_beams(self.x_live, a_parent, live_par)
        types_par = torch.empty(n, s_new, device=dev, dtype=torch.int64)
        K.gather_beams(self.x_types, a_parent, types_par, fill_byte=0xFF)
        table_par = torch.empty(n, self.x_block_table.shape[1], device=dev, dtype=torch.int32)
        K.gather_beams(self.x_block_table, a_parent, table_par)
        lengths_par = torch.empty(n, device=dev, dtype=torch.int32)
        K.gather_beams(self.x_lengths, a_parent, lengths_par)
        cache = self.exploration_cache
        states, live, types, new_k, new_v, action, rk, rv = xm.advance_device(
            states_par, live_par, types_par, a_xfer, a_source, a_src, a_dst, a_dst_types,
            cache.keys, cache.values, table_par, lengths_par, return_readout_kv=True,
            graphed=True)
        child_table, child_lengths = cache.append_device(
            table_par, lengths_par, new_k, new_v, action, rk, rv, child_cols=child_cols)
        cache.release_device(self.x_block_table, self.x_lengths)
        self.x_states, self.x_live, self.x_types = states, live, types
        self.x_block_table, self.x_lengths = child_table, child_lengths

    def _materialize(self, n: int, child_proposal, summary, rows, xfers, next_gate, fp,
                     cand_batch, cand_anchor, cand_bindings, parent, slots: int, nxt,
                     s_new: int):
        """Child topology rows for `n` children (indices into a ranked list
        whose candidates point into the given parent topology) written into
        the rows of `nxt`; returns the per-child action arrays
        (parent, xfer, source, source slots, destination slots, types)."""
        i64 = dict(device=self.device, dtype=torch.int64)
        a_parent, a_xfer, a_source = (torch.empty(n, **i64) for _ in range(3))
        a_src = torch.empty(n, self.max_src, **i64)
        a_dst = torch.empty(n, max(self.max_dst, 1), **i64)
        a_dst_types = torch.empty_like(a_dst)
        if n == 0:
            return a_parent, a_xfer, a_source, a_src, a_dst, a_dst_types
        _lib.check(_lib.lib().grs_topology_materialize(
            n, child_proposal.data_ptr(), summary.data_ptr(), rows.data_ptr(),
            xfers.data_ptr(), next_gate.data_ptr(), fp.data_ptr(), cand_batch.data_ptr(),
            cand_anchor.data_ptr(), cand_bindings.data_ptr(), cand_bindings.shape[1],
            self.table.data_ptr(), self.xfer_to_source.data_ptr(), slots, s_new,
            parent.types.data_ptr(), parent.out_node.data_ptr(), parent.out_port.data_ptr(),
            parent.in_node.data_ptr(), parent.in_port.data_ptr(), parent.touched.data_ptr(),
            parent.preferred.data_ptr(), parent.next_slot.data_ptr(), parent.streak.data_ptr(),
            nxt.types.data_ptr(), nxt.out_node.data_ptr(), nxt.out_port.data_ptr(),
            nxt.in_node.data_ptr(), nxt.in_port.data_ptr(), nxt.touched.data_ptr(),
            nxt.preferred.data_ptr(), nxt.distance.data_ptr(), nxt.next_slot.data_ptr(),
            nxt.streak.data_ptr(), nxt.gate.data_ptr(), nxt.fingerprint.data_ptr(),
            a_parent.data_ptr(), a_xfer.data_ptr(), a_source.data_ptr(), a_src.data_ptr(),
            a_src.shape[1], a_dst.data_ptr(), a_dst_types.data_ptr(), a_dst.shape[1], self.depth,
            self.status.data_ptr(), K.stream()), "topology_materialize")
        return a_parent, a_xfer, a_source, a_src, a_dst, a_dst_types

    def check(self) -> None:
        code = int(self.status.item())
        if code:
            self.status.zero_()
            _lib.check(code, "beam search")
        self.cache.check_status()

    @torch.no_grad()
    def run(self, depth: int | None = None) -> list[StepRow]:
        self.reset()
        for _ in range(depth or self.cfg.depth):
            if self.step() is None:
                break
        self.check()
        return self.rows

    # ---- inspection -------------------------------------------------------------
    def last_children(self) -> list[tuple[int, int, tuple[int, ...]]]:
        """(parent, xfer, binding) of the beams produced by the last step."""
        parent, xfer, src = (t.tolist() for t in self.last_actions[:3])
        return [(p, x, tuple(v for v in b if v >= 0)) for p, x, b in zip(parent, xfer, src)]

    def level_actions_host(self) -> dict:
        """The last level's children on the host: parent (index into the
        previous level's beam), xfer id, source and destination slots (-1
        padded) and gate count, each copied through a pinned buffer with one
        synchronisation.  `nbytes` is the device-to-host volume."""
        names = ("parent", "xfer", "source_slots", "destination_slots")
        tensors = list(zip(names, self.last_actions)) + [("gate_count", self.topo.gate)]
        bufs = getattr(self, "_host_bufs", {})
        out, nbytes = {}, 0
        for name, t in tensors:
            buf = bufs.get(name)
            if buf is None or buf.numel() < t.numel():
                buf = torch.empty(max(t.numel(), 1), dtype=t.dtype, pin_memory=True)
                bufs[name] = buf
            view = buf[: t.numel()].view(t.shape)
            view.copy_(t, non_blocking=True)
            out[name] = view
            nbytes += t.numel() * t.element_size()
        self._host_bufs = bufs
        torch.cuda.current_stream(self.device).synchronize()
        out["nbytes"] = nbytes
        return out

    def beam_summary(self) -> dict:
        """Gate counts, next slots and fingerprints of the current beam (host)."""
        return {"gate_count": self.topo.gate.tolist(), "next_slot": self.topo.next_slot.tolist(),
                "fingerprint": self.topo.fingerprint.tolist(),
                "local_streak": self.topo.streak.tolist()}

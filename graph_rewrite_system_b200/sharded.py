"""Beam search sharded over the GPUs of one node, one process per GPU.

The reference search (paged_rollout_benchmark.py:898-1207) runs on one GPU.
Its beams are independent within a level except for three couplings: the
global proposal ranking and cap, the global dedup set, and the fixed global
beam width.  Each rank here holds a slice of the beams with its own paged
cache, model state and port graph, and a level runs as:

1. locally: readout, match logits, candidates, per-parent-capped ranking and
   the rewrite plan (child fingerprint and validity) of its own beams
   (``DeviceBeamSearch._propose``);
2. every rank publishes its ranked records (fixed size, ``global_cap``
   rows) with one all-gather; the records carry the reference's full ranking
   key - next gate count ascending, probability descending, parent gate count
   ascending, then the position of the proposal in the single-GPU expansion
   order (global parent, xfer, candidate row);
3. every rank merges the gathered lists identically (two stable sorts on
   packed keys) and runs the accept loop on the merged list, so the dedup
   sets stay identical and the accepted children - and their order, the
   global beam order of the next level - equal the single-GPU search on the
   same records;
4. children stay on their parent's rank up to an even share of the new
   beam; for the overflow (placed deterministically, lowest rank with room
   first) the child's proposal and its parent's row - model state,
   topology, length and the contents of its cache pages, which the receiver
   copies into pages it allocates from its own free list - move with one
   all-to-all before the children are built, so every rank materialises and
   advances exactly its share of the new beam.

No kernel reads another GPU's memory; NCCL moves all data.
"""
from __future__ import annotations

import math

import torch
import torch.distributed as dist

from . import _lib
from . import kernels as K
from .rollout import DeviceBeamSearch, StepRow, _round_up
from .topology import TopologyState

# ---- ranked records --------------------------------------------------------
# One int64 row per ranked proposal.  KEY1/KEY2 order the records; the rest
# is the payload the accept loop and the child placement need.
KEY1, KEY2, VALID, FP, CHILD_NEXT, RANK, INDEX = range(7)
NUM_FIELDS = 7
ABSENT = (1 << 63) - 1                      # KEY1 of padding rows: sorts last

# bit budgets of the packed keys
GATE_BITS, PROB_BITS = 12, 32               # next gate, ~probability bits, parent gate
PARENT_BITS, XFER_BITS, ROW_BITS = 23, 16, 11


def pack_keys(next_gate, prob, parent_gate, global_parent, xfer, candidate_in_parent):
    """KEY1 = next_gate | ~prob_bits | parent_gate and KEY2 = global_parent |
    xfer | candidate index within the parent: lexicographic order on (KEY1,
    KEY2) is the reference ranking order (probabilities are non-negative
    float32, whose bit patterns order like the values).  Field widths: gate
    counts < 4096, global parents < 2^23, xfer ids < 65536, candidates per
    parent < 2048."""
    bits = prob.to(torch.float32).contiguous().view(torch.int32).to(torch.int64)
    desc = (0xFFFFFFFF - bits) & 0xFFFFFFFF
    key1 = (next_gate << (PROB_BITS + GATE_BITS)) | (desc << GATE_BITS) | parent_gate
    key2 = (global_parent << (XFER_BITS + ROW_BITS)) | (xfer << ROW_BITS) | candidate_in_parent
    return key1, key2


def merge_records(gathered: torch.Tensor, cap: int) -> tuple[torch.Tensor, torch.Tensor]:
    """Rank-order the union of every rank's records and keep the first `cap`.
    Returns (merged [cap, NUM_FIELDS], count int64 [1]) where count is the
    number of present (non-padding) records kept."""
    order = torch.sort(gathered[:, KEY2], stable=True).indices
    order = order[torch.sort(gathered[order, KEY1], stable=True).indices]
    merged = gathered[order[:cap]]
    count = (gathered[:, KEY1] != ABSENT).sum().clamp(max=cap).reshape(1)
    return merged, count


def placement(src: torch.Tensor, world: int):
    """Where each child (global acceptance order) lives next level.

    Rank r keeps its own children (those whose parent it holds) up to its
    quota - A // world, plus one for the first A % world ranks - in order;
    the rest go, in order, to the ranks with room, lowest rank first.
    Returns (dest [A], pair_counts [world, world]) with pair_counts[s, d] the
    children moving from rank s to rank d (the diagonal: kept)."""
    a = src.numel()
    ranks = torch.arange(world, device=src.device)
    quota = a // world + (ranks < a % world).long()
    onehot = torch.nn.functional.one_hot(src, world)
    position = (onehot.cumsum(0) * onehot).sum(1) - 1           # index among same-source
    keep = position < quota[src]
    kept = torch.bincount(src[keep], minlength=world)
    room = (quota - kept).cumsum(0)
    over = (~keep).long()
    slot = over.cumsum(0) - 1
    dest_over = torch.searchsorted(room, slot, right=True)
    dest = torch.where(keep, src, dest_over)
    pairs = torch.bincount(src * world + dest, minlength=world * world).view(world, world)
    return dest, pairs


# ---- packed beam rows ------------------------------------------------------
def _as_bytes(t: torch.Tensor) -> torch.Tensor:
    n = t.shape[0]
    return t.contiguous().view(n, -1).view(torch.uint8) if t.numel() else torch.empty(
        n, 0, dtype=torch.uint8, device=t.device)


def row_bytes(fields: list[torch.Tensor]) -> list[int]:
    return [math.prod(f.shape[1:]) * f.element_size() for f in fields]


def _rows(state: TopologyState, lo: int, hi: int) -> TopologyState:
    """Rows lo..hi of a topology view (views of the same storage)."""
    return TopologyState(*(getattr(state, f)[lo:hi] for f in (
        "types", "out_node", "out_port", "in_node", "in_port", "touched", "preferred",
        "distance", "next_slot", "streak", "gate", "fingerprint")))


class ShardedBeamSearch(DeviceBeamSearch):
    """``DeviceBeamSearch`` over this rank's slice of a beam whose global
    width is ``config.beam_size``; every rank runs the same step sequence.
    Requires an initialised default process group."""

    def __init__(self, *args, group=None, **kwargs):
        super().__init__(*args, **kwargs)
        self.group = group
        self.world = dist.get_world_size(group)
        self.rank = dist.get_rank(group)
        self.dst_len = self.table.view(-1, _lib.lib().grs_topology_table_width())[:, 1].long()

    # ---- state ------------------------------------------------------------------
    def reset(self) -> None:
        super().reset()
        self.rows_global = []
        if self.rank != 0:                      # the start state lives on rank 0
            self._empty_beams(self.slots)
        self.global_index = torch.arange(self.beams, device=self.device, dtype=torch.int64)
        self.global_count = 1

    def global_beams(self) -> int:
        return self.global_count

    def _empty_beams(self, slots: int) -> None:
        dev, m = self.device, self.model
        self.states = torch.empty(0, slots, m.width, device=dev, dtype=m.compute_dtype)
        self.live = torch.empty(0, slots, device=dev, dtype=torch.bool)
        self.types = torch.empty(0, slots, device=dev, dtype=torch.int64)
        self.block_table = torch.zeros(0, max(1, self.block_table.shape[1]), device=dev,
                                       dtype=torch.int32)
        self.lengths = torch.zeros(0, device=dev, dtype=torch.int32)
        self.topo = self.topology[self.current].state(0, slots)
        self.beams = 0

    # ---- collectives --------------------------------------------------------
    def _all_gather(self, t: torch.Tensor) -> torch.Tensor:
        out = [torch.empty_like(t) for _ in range(self.world)]
        dist.all_gather(out, t.contiguous(), group=self.group)
        return torch.stack(out)

    # ---- one level ----------------------------------------------------------
    def _records(self, prop) -> torch.Tensor:
        gcap = self.cfg.global_cap
        rows = prop.ranked.rows
        present = torch.arange(gcap, device=self.device) < prop.ranked.count
        safe = rows.clamp(min=0)
        parent = prop.cand["batch_ids"][safe]
        key1, key2 = pack_keys(prop.ranked.next_gate, prop.cand["probabilities"][safe],
                               self.topo.gate[parent], self.global_index[parent],
                               prop.ranked.xfer_ids, safe % prop.k)
        child_next = self.topo.next_slot[parent].long() + self.dst_len[prop.ranked.xfer_ids.clamp(min=0)]
        rec = torch.stack((key1, key2, prop.valid.long(), prop.fp, child_next,
                           torch.full_like(key1, self.rank),
                           torch.arange(gcap, device=self.device)), dim=1)
        rec[~present, KEY1] = ABSENT
        return rec

    def _step(self) -> StepRow | None:
        cfg, dev = self.cfg, self.device
        gcap, s, depth = cfg.global_cap, self.slots, self.depth
        i64 = dict(device=dev, dtype=torch.int64)
        prop = None
        if self.beams:
            prop = self._propose()
            rec = self._records(prop)
            metrics = torch.cat((prop.ranked.count, prop.ranked.metrics,
                                 self.cache.allocated_pages_tensor().long()))
        else:
            rec = torch.zeros(gcap, NUM_FIELDS, **i64)
            rec[:, KEY1] = ABSENT
            metrics = torch.cat((torch.zeros(3, **i64), self.cache.allocated_pages_tensor().long()))
        self._mark("exchange_records")
        gathered = self._all_gather(rec).view(-1, NUM_FIELDS)
        metrics = self._all_gather(metrics).sum(0)
        merged, count = merge_records(gathered, gcap)
        # 4. the accept loop on the merged list (identical on every rank)
        self._mark("accept")
        valid = merged[:, VALID].to(torch.uint8)
        fp = merged[:, FP].contiguous()
        next_gate = (merged[:, KEY1] >> (PROB_BITS + GATE_BITS)).contiguous()
        classes = torch.empty(gcap, device=dev, dtype=torch.uint8)
        child_proposal = torch.empty(cfg.beam_size, **i64)
        _lib.check(_lib.lib().grs_topology_accept(
            gcap, count.data_ptr(), valid.data_ptr(), fp.data_ptr(), next_gate.data_ptr(),
            cfg.beam_size, self.step_keys.data_ptr(), self.step_first.data_ptr(),
            self.step_capacity, self.seen.data_ptr(), self.seen_capacity, classes.data_ptr(),
            child_proposal.data_ptr(), self.summary.data_ptr(), None, None, None, None, None,
            self.status.data_ptr(), K.stream()), "topology_accept")
        self._mark("host_sync")
        metrics[0] = count[0]                       # proposals kept after the global cap
        host = torch.cat((self.summary, metrics, self.status.long(),
                          self.cache.status_tensor().long())).cpu().tolist()
        (accepted, attempted, invalid, dup, _, best, proposals, predicted, eligible_n,
         allocated, status, cache_status) = host
        if status:
            self.status.zero_()
            _lib.check(int(status), "beam search step")
        if cache_status:
            self.cache.check_status()
        row = StepRow(depth + 1, self.global_count, accepted, best, predicted, eligible_n,
                      proposals, attempted, accepted, invalid, dup, allocated, 0, 0.0)
        if not accepted:
            self.rows.append(row)
            return None
        # children in global order: where they come from and where they go
        chosen = merged[child_proposal[:accepted]]
        src, local_index = chosen[:, RANK], chosen[:, INDEX]
        dest, pairs = placement(src, self.world)
        plan = torch.cat((pairs.flatten(), chosen[:, CHILD_NEXT].max().reshape(1))).cpu().tolist()
        pairs_host = [plan[r * self.world:(r + 1) * self.world] for r in range(self.world)]
        s_new = max(s, _round_up(int(plan[-1]), 8))
        me = self.rank
        mine = torch.nonzero(src == me).flatten()                 # ascending global order
        stay = dest[mine] == me
        keep_j = mine[stay]
        leave = torch.nonzero(~stay).flatten()
        leave = leave[torch.sort(dest[mine[leave]], stable=True).indices]   # by destination
        out_j = mine[leave]
        in_j = torch.nonzero((dest == me) & (src != me)).flatten()
        in_j = in_j[torch.sort(src[in_j], stable=True).indices]   # by source, as received
        # 5a. children that change GPU: their proposal and their parent travel
        self._mark("rebalance")
        moved = self._exchange_parents(prop, local_index[out_j], pairs_host)
        # 5b-6. every GPU materialises and advances exactly its share
        self._children_sharded(prop, local_index[keep_j], moved, s_new)
        self._reorder(torch.cat((keep_j, in_j)))
        self.global_count = accepted
        row.logical_cache_pages = accepted * self.block_table.shape[1]
        self._mark("end")
        self.rows.append(row)
        return row

    # ---- moving children between GPUs ------------------------------------------
    def _move_fields(self, prop, ranked_index: torch.Tensor):
        """What a child that changes GPU carries: its proposal (xfer, next
        gate, fingerprint, anchor, bindings) and its parent's beam row
        (model state, topology, length); empty rows of the right shapes when
        nothing leaves."""
        dev, m = self.device, self.model
        i64 = dict(device=dev, dtype=torch.int64)
        n = 0 if prop is None else ranked_index.numel()
        t = self.topo
        parent = [self.states, self.live, self.types, t.types, t.out_node, t.out_port, t.in_node,
                  t.in_port, t.touched, t.preferred, t.next_slot, t.streak, self.lengths]
        if n == 0:
            proposal = [torch.empty(0, **i64) for _ in range(4)] + [
                torch.empty(0, m.max_pattern, **i64)]
            parent = [torch.empty(0, *f.shape[1:], device=dev, dtype=f.dtype) for f in parent]
            return proposal + parent, None
        rows = prop.ranked.rows[ranked_index]
        proposal = [prop.ranked.xfer_ids[ranked_index], prop.ranked.next_gate[ranked_index],
                    prop.fp[ranked_index], prop.cand["anchors"][rows], prop.cand["bindings"][rows]]
        parent_rows = prop.cand["batch_ids"][rows]
        return proposal + [f.index_select(0, parent_rows) for f in parent], parent_rows

    def _exchange_parents(self, prop, ranked_index: torch.Tensor, pairs) -> dict:
        """Send the children leaving this GPU (proposal + parent row + the
        parent's cache pages) and receive the ones arriving; the received
        pages are copied into pages of this cache."""
        dev, world, me = self.device, self.world, self.rank
        fields, parent_rows = self._move_fields(prop, ranked_index)
        widths = row_bytes(fields)
        cols = -(-self.depth // self.cfg.page_size)               # parent pages in use
        page_bytes = self.cache.page_bytes
        row_size = sum(widths) + cols * page_bytes
        send_counts = [pairs[me][d] if d != me else 0 for d in range(world)]
        recv_counts = [pairs[r][me] if r != me else 0 for r in range(world)]
        if parent_rows is not None:
            parts = [_as_bytes(f) for f in fields]
            if cols:
                pages = self.block_table.index_select(0, parent_rows)[:, :cols].flatten()
                parts.append(self.cache.export_pages(pages).view(parent_rows.numel(), -1))
            send = torch.cat(parts, dim=1)
        else:
            send = torch.empty(0, row_size, device=dev, dtype=torch.uint8)
        n_in = sum(recv_counts)
        recv = torch.empty(n_in, row_size, device=dev, dtype=torch.uint8)
        if world > 1:                              # collective: every rank, every level
            dist.all_to_all_single(recv.view(-1), send.contiguous().view(-1),
                                   [c * row_size for c in recv_counts],
                                   [c * row_size for c in send_counts], group=self.group)
        out, offset = [], 0
        for f, w in zip(fields, widths):
            if n_in:
                # a fresh, aligned copy: field offsets inside a row are not
                # multiples of the field's element size
                part = recv[:, offset:offset + w].flatten().clone()
                out.append(part.view(f.dtype).view(n_in, *f.shape[1:]))
            else:
                out.append(torch.empty(0, *f.shape[1:], device=dev, dtype=f.dtype))
            offset += w
        table = torch.zeros(n_in, max(1, self.block_table.shape[1]), device=dev,
                            dtype=torch.int32)
        if n_in and cols:
            data = recv[:, offset:].flatten().clone().view(-1, page_bytes)
            table[:, :cols] = self.cache.import_pages(data).view(n_in, cols)
        (xfer, next_gate, fp, anchor, bindings, states, live, types, t_types, out_node, out_port,
         in_node, in_port, touched, preferred, next_slot, streak, lengths) = out
        parent = TopologyState(t_types, out_node, out_port, in_node, in_port, touched, preferred,
                               torch.empty_like(touched), next_slot, streak,
                               torch.empty(n_in, device=dev, dtype=torch.int64),
                               torch.empty(n_in, device=dev, dtype=torch.int64))
        return {"n": n_in, "xfer": xfer, "next_gate": next_gate, "fp": fp, "anchor": anchor,
                "bindings": bindings, "states": states, "live": live, "types": types,
                "topo": parent, "table": table, "lengths": lengths}

    def _children_sharded(self, prop, keep_index: torch.Tensor, moved: dict, s_new: int) -> None:
        """Materialise this GPU's children - its own kept ones from the local
        ranked proposals and parents, then the received ones from their
        travelling proposals and parents - advance them in one batch, append
        to the cache and release every parent."""
        cfg, model, dev = self.cfg, self.model, self.device
        s, depth = self.slots, self.depth
        n_keep, n_in = keep_index.numel(), moved["n"]
        n = n_keep + n_in
        i64 = dict(device=dev, dtype=torch.int64)
        self._mark("materialize")
        nxt = self.topology[1 - self.current].state(n, s_new)
        acts = []
        if n_keep:
            summary = torch.zeros(6, **i64)
            summary[0] = n_keep
            acts.append(self._materialize(
                n_keep, keep_index.contiguous(), summary, prop.ranked.rows, prop.ranked.xfer_ids,
                prop.ranked.next_gate, prop.fp, prop.cand["batch_ids"], prop.cand["anchors"],
                prop.cand["bindings"], self.topo, s, _rows(nxt, 0, n_keep), s_new))
        if n_in:
            summary = torch.zeros(6, **i64)
            summary[0] = n_in
            ident = torch.arange(n_in, **i64)
            acts.append(self._materialize(
                n_in, ident, summary, ident, moved["xfer"].contiguous(),
                moved["next_gate"].contiguous(), moved["fp"].contiguous(), ident,
                moved["anchor"].contiguous(), moved["bindings"].contiguous(), moved["topo"], s,
                _rows(nxt, n_keep, n), s_new))
        if len(acts) == 2:
            a_parent, a_xfer, a_source, a_src, a_dst, a_dst_types = (
                torch.cat(parts) for parts in zip(*acts))
        elif acts:
            a_parent, a_xfer, a_source, a_src, a_dst, a_dst_types = acts[0]
        # 6. gather the parents (local, then received), advance, append, release
        self._mark("advance")
        w = model.width
        child_cols = -(-(depth + 1) // cfg.page_size)
        if n:
            cols = self.block_table.shape[1]
            states_par = torch.empty(n, s_new, w, device=dev, dtype=model.compute_dtype)
            live_par = torch.empty(n, s_new, device=dev, dtype=torch.bool)
            types_par = torch.empty(n, s_new, **i64)
            table_par = torch.empty(n, cols, device=dev, dtype=torch.int32)
            lengths_par = torch.empty(n, device=dev, dtype=torch.int32)
            for lo, hi, st, lv, ty, tb, ln in (
                    (0, n_keep, self.states, self.live, self.types, self.block_table,
                     self.lengths),
                    (n_keep, n, moved["states"], moved["live"], moved["types"], moved["table"],
                     moved["lengths"])):
                if hi > lo:
                    idx = a_parent[lo:hi]
                    K.gather_beams(st, idx, states_par[lo:hi])
                    K.gather_beams(lv, idx, live_par[lo:hi])
                    K.gather_beams(ty, idx, types_par[lo:hi], fill_byte=0xFF)
                    K.gather_beams(tb, idx, table_par[lo:hi])
                    K.gather_beams(ln, idx, lengths_par[lo:hi])
            states, live, types, new_k, new_v, action = model.advance_device(
                states_par, live_par, types_par, a_xfer, a_source, a_src, a_dst, a_dst_types,
                self.cache.keys, self.cache.values, table_par, lengths_par)
            rk, rv = model.project_action_readout_kv(action)
            self._mark("cache_append_release")
            child_table, child_lengths = self.cache.append_device(
                table_par, lengths_par, new_k, new_v, action, rk, rv, child_cols=child_cols)
        else:
            states = torch.empty(0, s_new, w, device=dev, dtype=model.compute_dtype)
            live = torch.empty(0, s_new, device=dev, dtype=torch.bool)
            types = torch.empty(0, s_new, **i64)
            child_table = torch.zeros(0, child_cols, device=dev, dtype=torch.int32)
            child_lengths = torch.zeros(0, device=dev, dtype=torch.int32)
        if self.beams:
            self.cache.release_device(self.block_table, self.lengths)
        if n_in:
            self.cache.release_device(moved["table"], moved["lengths"])
        self.states, self.live, self.types = states, live, types
        self.block_table, self.lengths = child_table, child_lengths
        self.topo, self.current = nxt, 1 - self.current
        self.beams, self.slots, self.depth = n, s_new, depth + 1

    def _reorder(self, global_index: torch.Tensor) -> None:
        """Put this GPU's children in global order (the order the ranking's
        ties follow), copying the topology into the spare buffer."""
        order = torch.sort(global_index).indices
        self.global_index = global_index[order]
        n, s = self.beams, self.slots
        self.states = self.states.index_select(0, order)
        self.live = self.live.index_select(0, order)
        self.types = self.types.index_select(0, order)
        self.block_table = self.block_table.index_select(0, order)
        self.lengths = self.lengths.index_select(0, order)
        src = self.topo
        dst = self.topology[1 - self.current].state(n, s)
        for name in ("types", "out_node", "out_port", "in_node", "in_port", "touched",
                     "preferred", "distance", "next_slot", "streak", "gate", "fingerprint"):
            torch.index_select(getattr(src, name), 0, order, out=getattr(dst, name))
        self.topo, self.current = dst, 1 - self.current

    # ---- results ------------------------------------------------------------
    def global_fingerprints(self) -> list[int]:
        """Fingerprints of the whole beam in global order (a collective)."""
        n = torch.tensor([self.beams], device=self.device)
        counts = self._all_gather(n).flatten().tolist()
        width = max(counts) if counts else 0
        pad = torch.zeros(width, 2, device=self.device, dtype=torch.int64)
        pad[: self.beams, 0] = self.global_index
        pad[: self.beams, 1] = self.topo.fingerprint
        rows = self._all_gather(pad)
        pairs = []
        for r, c in enumerate(counts):
            pairs.extend(rows[r, :c].tolist())
        return [fp & ((1 << 64) - 1) for _, fp in sorted(pairs)]

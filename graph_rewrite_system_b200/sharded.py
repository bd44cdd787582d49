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
   beam; the overflow moves (deterministically, lowest rank with room first)
   with one all-to-all of packed rows: model state, topology and the
   contents of the child's cache pages, which the receiver copies into pages
   it allocates from its own free list.

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
def _row_fields(states, live, types, topo: TopologyState, lengths):
    """The per-beam tensors that travel with a beam (first dim = beams)."""
    return [states, live, types, topo.types, topo.out_node, topo.out_port, topo.in_node,
            topo.in_port, topo.touched, topo.preferred, topo.distance, topo.next_slot,
            topo.streak, topo.gate, topo.fingerprint, lengths]


def _as_bytes(t: torch.Tensor) -> torch.Tensor:
    n = t.shape[0]
    return t.contiguous().view(n, -1).view(torch.uint8) if t.numel() else torch.empty(
        n, 0, dtype=torch.uint8, device=t.device)


def pack_rows(fields: list[torch.Tensor], rows: torch.Tensor) -> torch.Tensor:
    return torch.cat([_as_bytes(f.index_select(0, rows)) for f in fields], dim=1)


def row_bytes(fields: list[torch.Tensor]) -> list[int]:
    return [math.prod(f.shape[1:]) * f.element_size() for f in fields]


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
        mine = torch.nonzero(src == self.rank).flatten()          # ascending global order
        n_local = sum(pairs_host[self.rank])
        if n_local:
            local_summary = torch.zeros(6, **i64)
            local_summary[0] = n_local
            self._children(prop, local_index[mine].contiguous(), local_summary, n_local, s_new)
        else:
            if self.beams:
                self.cache.release_device(self.block_table, self.lengths)
            self._empty_beams(s_new)
            self.slots, self.depth = s_new, depth + 1
            self.block_table = torch.zeros(0, -(-(depth + 1) // cfg.page_size), device=dev,
                                           dtype=torch.int32)
        self._mark("rebalance")
        self._rebalance(src, mine, dest, pairs_host, accepted)
        self.global_count = accepted
        row.logical_cache_pages = accepted * self.block_table.shape[1]
        self._mark("end")
        self.rows.append(row)
        return row

    def _rebalance(self, src: torch.Tensor, mine: torch.Tensor, dest: torch.Tensor,
                   pairs: list[list[int]], accepted: int) -> None:
        """Move the children this rank holds but does not keep, receive the
        ones it gains, and order the result by global child index."""
        dev, world, me = self.device, self.world, self.rank
        s_new, cols = self.slots, self.block_table.shape[1]
        my_dest = dest[mine]
        fields = _row_fields(self.states, self.live, self.types, self.topo, self.lengths)
        widths = row_bytes(fields)
        page_bytes = self.cache.page_bytes
        row_size = sum(widths) + cols * page_bytes
        # outgoing rows in (destination, global index) order
        out_mask = my_dest != me
        out_rows = torch.nonzero(out_mask).flatten()
        out_rows = out_rows[torch.sort(my_dest[out_rows], stable=True).indices]
        send_counts = [pairs[me][d] if d != me else 0 for d in range(world)]
        recv_counts = [pairs[s][me] if s != me else 0 for s in range(world)]
        send = torch.empty(0, row_size, device=dev, dtype=torch.uint8)
        if out_rows.numel():
            pages = self.block_table.index_select(0, out_rows)[:, :cols].flatten()
            page_data = self.cache.export_pages(pages).view(out_rows.numel(), -1)
            send = torch.cat((pack_rows(fields, out_rows), page_data), dim=1)
        recv = torch.empty(sum(recv_counts), row_size, device=dev, dtype=torch.uint8)
        if world > 1:                              # collective: every rank, every level
            dist.all_to_all_single(recv.view(-1), send.contiguous().view(-1),
                                   [c * row_size for c in recv_counts],
                                   [c * row_size for c in send_counts], group=self.group)
        if out_rows.numel():
            self.cache.release_device(self.block_table.index_select(0, out_rows),
                                      self.lengths.index_select(0, out_rows))
        # global indices of what this rank holds next: kept rows + received rows
        keep_rows = torch.nonzero(~out_mask).flatten()
        keep_global = mine[keep_rows]
        # received children: by source rank, then global index (the senders'
        # packing order)
        incoming = torch.nonzero((dest == me) & (src != me)).flatten()
        incoming = incoming[torch.sort(src[incoming], stable=True).indices]
        n_final = keep_rows.numel() + incoming.numel()
        order = torch.sort(torch.cat((keep_global, incoming))).indices
        # unpack received rows
        n_in = recv.shape[0]
        recv_fields, offset = [], 0
        for f, w in zip(fields, widths):
            if n_in:
                # a fresh, aligned copy: field offsets inside a row are not
                # multiples of the field's element size
                part = recv[:, offset:offset + w].flatten().clone()
                recv_fields.append(part.view(f.dtype).view(n_in, *f.shape[1:]))
            else:
                recv_fields.append(torch.empty(0, *f.shape[1:], device=dev, dtype=f.dtype))
            offset += w
        recv_pages = (recv[:, offset:].flatten().clone().view(-1, page_bytes) if n_in else
                      torch.empty(0, page_bytes, device=dev, dtype=torch.uint8))
        new_pages = self.cache.import_pages(recv_pages).view(recv.shape[0], cols)
        table_in = torch.zeros(recv.shape[0], self.block_table.shape[1], device=dev,
                               dtype=torch.int32)
        table_in[:, :cols] = new_pages
        # assemble the next beam in global order
        merged_fields = [torch.cat((f.index_select(0, keep_rows), r))[order]
                         for f, r in zip(fields, recv_fields)]
        table = torch.cat((self.block_table.index_select(0, keep_rows), table_in))[order]
        nxt = self.topology[1 - self.current].state(n_final, s_new)
        (states, live, types, t_types, out_node, out_port, in_node, in_port, touched,
         preferred, distance, next_slot, streak, gate, fingerprint, lengths) = merged_fields
        for dst, src in ((nxt.types, t_types), (nxt.out_node, out_node),
                         (nxt.out_port, out_port), (nxt.in_node, in_node),
                         (nxt.in_port, in_port), (nxt.touched, touched),
                         (nxt.preferred, preferred), (nxt.distance, distance),
                         (nxt.next_slot, next_slot), (nxt.streak, streak), (nxt.gate, gate),
                         (nxt.fingerprint, fingerprint)):
            dst.copy_(src)
        self.states, self.live, self.types = states, live, types
        self.block_table, self.lengths = table.contiguous(), lengths.contiguous()
        self.topo, self.current = nxt, 1 - self.current
        self.global_index = torch.cat((keep_global, incoming))[order]
        self.beams = n_final

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

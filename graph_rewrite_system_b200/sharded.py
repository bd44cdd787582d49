"""Beam search sharded over the GPUs of one node, one process per GPU.

The reference search (paged_rollout_benchmark.py:898-1207) runs on one GPU.
Its beams are independent within a level except for three couplings: the
global proposal ranking and cap, the global dedup set, and the fixed global
beam width.  Each rank here holds a slice of the beams with its own paged
cache, model state and port graph, and a level runs as:

1. locally: readout, match logits, candidates, per-parent-capped ranking and
   the rewrite plan (child fingerprint and validity) of its own beams
   (``DeviceBeamSearch._propose``);
2. every rank publishes its ranked records with one all-gather, padded to
   the most a rank can hold (ceil(global beams / world) parents times the
   per-parent cap, at most ``global_cap``, so nothing the global cap would
   keep is dropped); the records carry the reference's full ranking
   key - next gate count ascending, probability descending, parent gate count
   ascending, then the position of the proposal in the single-GPU expansion
   order (global parent, xfer, candidate row);
3. every rank merges the gathered lists identically (each list arrives
   sorted; ``grs_shard_merge`` places every record by binary searches in the
   other lists) and runs the accept loop on the merged list, so the dedup
   sets stay identical and the accepted children - and their order, the
   global beam order of the next level - equal the single-GPU search on the
   same records;
4. children stay on their parent's rank up to an even share of the new
   beam; for the overflow (placed deterministically, lowest rank with room
   first, by ``grs_shard_route``) the child's proposal and its parent's row - model state,
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
# grs_shard_records packs a GPU's ranked list into int64 records, field-major
# [KEY1 | KEY2 | FP | AUX] x width followed by REC_METRICS values; the order
# of (KEY1, KEY2) is the reference ranking order.
REC_FIELDS, REC_METRICS = 4, 4


# ---- beam rows -------------------------------------------------------------
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
        if kwargs.get("exploration_model") is not None:
            raise NotImplementedError("the sharded search runs one model; the exploration "
                                      "model runs on the single-GPU search")
        super().__init__(*args, **kwargs)
        self.group = group
        self.world = dist.get_world_size(group)
        self.rank = dist.get_rank(group)
        self.moved_children = 0                 # children that changed GPU, all levels
        self.moved_bytes = 0                    # bytes this GPU sent for them

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
        out = torch.empty(self.world * t.shape[0], *t.shape[1:], device=t.device, dtype=t.dtype)
        dist.all_gather_into_tensor(out, t.contiguous(), group=self.group)
        return out.view(self.world, *t.shape)

    # ---- one level ----------------------------------------------------------
    def _send_block(self, prop, width: int) -> torch.Tensor:
        """This GPU's ranked proposals as a record block (padding past the
        ranked count), followed by its metrics."""
        dev, lib = self.device, _lib.lib()
        block = torch.empty(REC_FIELDS * width + REC_METRICS, device=dev, dtype=torch.int64)
        free_count = self.cache.free_count_tensor()
        if prop is None:
            zero = torch.zeros(1, device=dev, dtype=torch.int64)
            _lib.check(lib.grs_shard_records(
                width, zero.data_ptr(), None, None, None, None, None, 1, None, None, None, None,
                None, None, None, free_count.data_ptr(), self.cache.capacity, block.data_ptr(),
                self.status.data_ptr(), K.stream()), "shard_records")
            return block
        r, cand, t = prop.ranked, prop.cand, self.topo
        _lib.check(lib.grs_shard_records(
            width, r.count.data_ptr(), r.rows.data_ptr(), r.xfer_ids.data_ptr(),
            r.next_gate.data_ptr(), cand["probabilities"].data_ptr(),
            cand["batch_ids"].data_ptr(), prop.k, t.gate.data_ptr(),
            self.global_index.data_ptr(), t.next_slot.data_ptr(), self.table.data_ptr(),
            prop.valid.data_ptr(), prop.fp.data_ptr(), r.metrics.data_ptr(),
            free_count.data_ptr(), self.cache.capacity, block.data_ptr(),
            self.status.data_ptr(), K.stream()), "shard_records")
        return block

    def _step(self) -> StepRow | None:
        cfg, dev, lib = self.cfg, self.device, _lib.lib()
        s, depth, world, me = self.slots, self.depth, self.world, self.rank
        i64 = dict(device=dev, dtype=torch.int64)
        # 1-2. local proposals; a rank holds at most ceil(global beams / world)
        # parents with at most parent_cap() proposals each, so blocks of that
        # many records lose nothing the global cap would keep
        width = min(cfg.global_cap, -(-self.global_count // world) * self.parent_cap())
        prop = self._propose() if self.beams else None
        block = self._send_block(prop, width)
        # 3. one all-gather of every GPU's block, then the merged ranking
        self._mark("exchange_records")
        gathered = self._all_gather(block)
        cap = min(cfg.global_cap, world * width)
        count = torch.empty(1, **i64)
        metrics = torch.empty(REC_METRICS, **i64)
        valid = torch.empty(cap, device=dev, dtype=torch.uint8)
        fp, next_gate, src, index, child_next = (torch.empty(cap, **i64) for _ in range(5))
        _lib.check(lib.grs_shard_merge(
            gathered.data_ptr(), world, width, block.numel(), cap, count.data_ptr(),
            metrics.data_ptr(), valid.data_ptr(), fp.data_ptr(), next_gate.data_ptr(),
            src.data_ptr(), index.data_ptr(), child_next.data_ptr(), self.status.data_ptr(),
            K.stream()), "shard_merge")
        # 4. the accept loop on the merged list (identical on every rank)
        self._mark("accept")
        classes = torch.empty(cap, device=dev, dtype=torch.uint8)
        child_proposal = torch.zeros(cfg.beam_size, **i64)
        _lib.check(lib.grs_topology_accept(
            cap, count.data_ptr(), valid.data_ptr(), fp.data_ptr(), next_gate.data_ptr(),
            cfg.beam_size, self.step_keys.data_ptr(), self.step_first.data_ptr(),
            self.step_capacity, self.seen.data_ptr(), self.seen_capacity, classes.data_ptr(),
            child_proposal.data_ptr(), self.summary.data_ptr(), None, None, None, None, None,
            self.status.data_ptr(), K.stream()), "topology_accept")
        # where every child lives next level, and this GPU's index lists
        pairs = torch.empty(world * world, **i64)
        extent = torch.empty(1, **i64)
        keep_local, keep_global, in_global = (torch.empty(cfg.beam_size, **i64)
                                               for _ in range(3))
        out_local = torch.zeros(cfg.beam_size, **i64)   # zero tail: safe gather indexes
        _lib.check(lib.grs_shard_route(
            child_proposal.data_ptr(), self.summary.data_ptr(), src.data_ptr(),
            index.data_ptr(), child_next.data_ptr(), cap, cfg.beam_size, world, me,
            pairs.data_ptr(), extent.data_ptr(), keep_local.data_ptr(), keep_global.data_ptr(),
            out_local.data_ptr(), in_global.data_ptr(), self.status.data_ptr(), K.stream()),
            "shard_route")
        # leaving children's rows packed while the host waits below
        send = None
        if world > 1:
            n_out_dev = pairs.view(world, world)[me].sum(0, keepdim=True) - pairs[
                me * world + me:me * world + me + 1]
            max_out = min(cfg.beam_size, width) if prop is not None else 0
            send = self._pack_outgoing(prop, out_local, n_out_dev, max_out)
        # the level's one host read
        self._mark("host_sync")
        host = torch.cat((self.summary, count, metrics[1:], self.status.long(),
                          self.cache.status_tensor().long(), pairs, extent)).cpu().tolist()
        (accepted, attempted, invalid, dup, _, best, proposals, predicted, eligible_n,
         allocated, status, cache_status) = host[:12]
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
        pairs_host = [host[12 + r * world:12 + (r + 1) * world] for r in range(world)]
        s_new = max(s, _round_up(int(host[-1]), 8))
        n_keep = pairs_host[me][me]
        n_in = sum(pairs_host[r][me] for r in range(world)) - n_keep
        # 5a. children that change GPU: their proposal and their parent travel
        self._mark("rebalance")
        moves = sum(sum(row) for row in pairs_host) - sum(pairs_host[r][r] for r in range(world))
        self.moved_children += moves
        moved = self._exchange_parents(send, pairs_host, moves > 0)
        # 5b-6. every GPU materialises and advances exactly its share
        self._children_sharded(prop, keep_local[:n_keep], moved, s_new)
        self._reorder(torch.cat((keep_global[:n_keep], in_global[:n_in])), n_in)
        self.global_count = accepted
        row.logical_cache_pages = accepted * self.block_table.shape[1]
        self._mark("end")
        self.rows.append(row)
        return row

    # ---- moving children between GPUs ------------------------------------------
    PARENT_FIELDS = ("states", "live", "types", "t_types", "out_node", "out_port", "in_node",
                     "in_port", "touched", "preferred", "next_slot", "streak", "lengths")
    PROPOSAL_FIELDS = ("xfer", "next_gate", "fp", "anchor", "bindings")

    def _parent_tensors(self) -> list[torch.Tensor]:
        t = self.topo
        return [self.states, self.live, self.types, t.types, t.out_node, t.out_port, t.in_node,
                t.in_port, t.touched, t.preferred, t.next_slot, t.streak, self.lengths]

    def _row_layout(self):
        """What a child that changes GPU carries, as one byte row: its
        proposal (xfer, next gate, fingerprint, anchor, bindings), its
        parent's beam row (model state, topology, length) and the parent's
        cache pages in use.  Returns ([(name, dtype, row shape, offset,
        bytes)], [(arena, offset, page bytes)], pages per row, row bytes);
        every piece starts 16-byte aligned.  The layout is the same on every
        GPU (same slot count, depth and cache geometry)."""
        i64 = torch.int64
        specs = [(n, i64, ()) for n in self.PROPOSAL_FIELDS[:4]]
        specs.append(("bindings", i64, (self.model.max_pattern,)))
        specs += [(n, f.dtype, tuple(f.shape[1:]))
                  for n, f in zip(self.PARENT_FIELDS, self._parent_tensors())]
        fields, offset = [], 0
        for name, dtype, shape in specs:
            nbytes = math.prod(shape) * torch.empty((), dtype=dtype).element_size()
            fields.append((name, dtype, shape, offset, nbytes))
            offset += _round_up(nbytes, 16)
        cols = -(-self.depth // self.cfg.page_size)                # parent pages in use
        pages = []
        for arena in self.cache.arenas():
            nbytes = arena.shape[1] * arena.element_size()
            pages.append((arena, offset, nbytes))
            offset += _round_up(nbytes * cols, 16)
        return fields, pages, cols, _round_up(offset, 16)

    def _staging(self, name: str, nbytes: int) -> torch.Tensor:
        """A persistent byte buffer of at least `nbytes` (grown by half again
        when too small): the packed rows change size with the slot count, and
        a fresh multi-hundred-megabyte allocation per level can stall a level
        while the allocator maps memory."""
        buf = getattr(self, name, None)
        if buf is None or buf.numel() < nbytes:
            size = max(nbytes, int(1.5 * buf.numel()) if buf is not None else 0)
            buf = torch.empty(size, device=self.device, dtype=torch.uint8)
            setattr(self, name, buf)
        return buf[:nbytes]

    def _pack_outgoing(self, prop, out_local: torch.Tensor, n_out: torch.Tensor,
                       max_out: int):
        """Before the level's host read: copy the rows of this GPU's leaving
        children (out_local, device count n_out <= max_out) into send rows
        with one grs_rows_copy launch."""
        fields, pages, cols, row_size = self._row_layout()
        send = self._staging("_send_buf", max_out * row_size).view(max_out, row_size)
        if max_out == 0:
            return send
        ranked_index = out_local[:max_out]
        rows = prop.ranked.rows.index_select(0, ranked_index).clamp_(min=0)
        parent = prop.cand["batch_ids"].index_select(0, rows)
        sources = [(prop.ranked.xfer_ids, ranked_index), (prop.ranked.next_gate, ranked_index),
                   (prop.fp, ranked_index), (prop.cand["anchors"], rows),
                   (prop.cand["bindings"], rows)]
        sources += [(f, parent) for f in self._parent_tensors()]
        flat = send.view(-1)
        segments = []
        for (src, index), (_, _, _, offset, nbytes) in zip(sources, fields):
            stride = src.stride(0) * src.element_size()
            segments.append((src, 0, stride, index, flat[offset:], row_size, 0, None, nbytes, 1))
        if cols:
            page_ids = self.block_table.index_select(0, parent)[:, :cols].long().contiguous()
            for arena, offset, nbytes in pages:
                segments.append((arena, 0, arena.stride(0) * arena.element_size(), page_ids,
                                 flat[offset:], row_size, nbytes, None, nbytes, cols))
        K.rows_copy(segments, max_out, n_out)
        return send

    def _exchange_parents(self, send: torch.Tensor, pairs, any_moves: bool) -> dict:
        """Send the packed rows of the children leaving this GPU and unpack
        the arriving ones: fields into fresh tensors, page contents into
        pages allocated from this cache.  `any_moves` (the same on every
        rank) skips the collective when no child changes GPU."""
        dev, world, me = self.device, self.world, self.rank
        fields, pages, cols, row_size = self._row_layout()
        send_counts = [pairs[me][d] if d != me else 0 for d in range(world)]
        recv_counts = [pairs[r][me] if r != me else 0 for r in range(world)]
        n_out, n_in = sum(send_counts), sum(recv_counts)
        self.moved_bytes += n_out * row_size
        recv = self._staging("_recv_buf", n_in * row_size).view(n_in, row_size)
        if send is None:
            send = torch.empty(0, row_size, device=dev, dtype=torch.uint8)
        if world > 1 and any_moves:                # collective: every rank alike
            dist.all_to_all_single(recv.view(-1), send[:n_out].reshape(-1),
                                   [c * row_size for c in recv_counts],
                                   [c * row_size for c in send_counts], group=self.group)
        out = {name: torch.empty(n_in, *shape, device=dev, dtype=dtype)
               for name, dtype, shape, _, _ in fields}
        table = torch.zeros(n_in, max(1, self.block_table.shape[1]), device=dev,
                            dtype=torch.int32)
        if n_in:
            flat = recv.view(-1)
            segments = [(flat[offset:], row_size, 0, None, out[name], nbytes, 0, None, nbytes, 1)
                        for name, _, _, offset, nbytes in fields]
            if cols:
                page_ids = self.cache.alloc_pages(n_in * cols)
                table[:, :cols] = page_ids.view(n_in, cols)
                index = page_ids.long()
                for arena, offset, nbytes in pages:
                    segments.append((flat[offset:], row_size, nbytes, None, arena, 0,
                                     arena.stride(0) * arena.element_size(), index, nbytes,
                                     cols))
            K.rows_copy(segments, n_in)
        parent = TopologyState(out["t_types"], out["out_node"], out["out_port"], out["in_node"],
                               out["in_port"], out["touched"], out["preferred"],
                               torch.empty_like(out["touched"]), out["next_slot"],
                               out["streak"], torch.empty(n_in, device=dev, dtype=torch.int64),
                               torch.empty(n_in, device=dev, dtype=torch.int64))
        out.update(n=n_in, topo=parent, table=table)
        return out

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
            states, live, types, new_k, new_v, action, rk, rv = model.advance_device(
                states_par, live_par, types_par, a_xfer, a_source, a_src, a_dst, a_dst_types,
                self.cache.keys, self.cache.values, table_par, lengths_par,
                return_readout_kv=True, graphed=True)
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
        if n:       # parents index this GPU's kept parents, then the received rows
            self.last_actions = (a_parent, a_xfer, a_src, a_dst)
        else:
            self.last_actions = (torch.empty(0, **i64), torch.empty(0, **i64),
                                 torch.empty(0, self.max_src, **i64),
                                 torch.empty(0, max(self.max_dst, 1), **i64))
        self.states, self.live, self.types = states, live, types
        self.block_table, self.lengths = child_table, child_lengths
        self.topo, self.current = nxt, 1 - self.current
        self.beams, self.slots, self.depth = n, s_new, depth + 1

    def _reorder(self, global_index: torch.Tensor, received: int) -> None:
        """Put this GPU's children in global order (the order the ranking's
        ties follow) with one grs_rows_copy launch, the topology into the
        spare buffer; the kept children are already in order, so nothing
        moves when none arrived."""
        if not received:
            self.global_index = global_index
            return
        order = torch.sort(global_index).indices
        self.global_index = global_index[order]
        n, s = self.beams, self.slots
        src = self.topo
        dst = self.topology[1 - self.current].state(n, s)
        names = ("types", "out_node", "out_port", "in_node", "in_port", "touched", "preferred",
                 "distance", "next_slot", "streak", "gate", "fingerprint")
        pairs = [(getattr(src, name), getattr(dst, name)) for name in names]
        beam = [self.states, self.live, self.types, self.block_table, self.lengths]
        fresh = [torch.empty_like(t) for t in beam]
        segments = []
        for a, b in pairs + list(zip(beam, fresh)):
            nbytes = a[0].numel() * a.element_size() if a.numel() else 0
            segments.append((a, 0, a.stride(0) * a.element_size(), order, b,
                             b.stride(0) * b.element_size(), 0, None, nbytes, 1))
        K.rows_copy(segments, n)
        self.states, self.live, self.types, self.block_table, self.lengths = fresh
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

"""Oracle of the sharded search's record exchange (NumPy; test infrastructure).

The reference ranks all proposals of a level on one GPU - next gate count
ascending, probability descending, parent gate count ascending, ties in
expansion order: parent, xfer, candidate (gpu_proposals.py:128-154) - and
accepts in that order (paged_rollout_benchmark.py:1013-1046).  A sharded
search ranks every GPU's beams separately and must rebuild that one list.
This module states, with plain sorts and loops, what the CUDA record
kernels compute:

* ``pack_records`` - one GPU's ranked list as records whose lexicographic
  (KEY1, KEY2) order is the reference ranking order;
* ``merge_records`` - the first ``cap`` records of the union in that order;
* ``route`` - where every accepted child lives next level: each GPU keeps
  its own children up to an even share, the overflow goes in acceptance
  order to the GPUs with room, lowest first.
"""
from __future__ import annotations

import numpy as np

ABSENT = (1 << 63) - 1
FIELDS = 4                 # KEY1, KEY2, FP, AUX
METRICS = 4                # ranked count, predicted, eligible, allocated pages


def pack_keys(next_gate, prob, parent_gate, global_parent, xfer, candidate_in_parent):
    """KEY1 = next_gate << 44 | (0xffffffff - float32 bits of prob) << 12 |
    parent_gate; KEY2 = global_parent << 27 | xfer << 11 | candidate.  For
    non-negative float32 probabilities the bit patterns order like the
    values, so ascending KEY1 is descending probability within a gate count."""
    bits = np.asarray(prob, np.float32).view(np.uint32).astype(np.int64)
    ng = np.asarray(next_gate, np.int64)
    key1 = (ng << 44) | ((0xFFFFFFFF - bits) << 12) | np.asarray(parent_gate, np.int64)
    key2 = ((np.asarray(global_parent, np.int64) << 27) | (np.asarray(xfer, np.int64) << 11)
            | np.asarray(candidate_in_parent, np.int64))
    return key1, key2


def pack_records(width, count, rows, xfers, next_gate, probs, cand_batch, k, gate, global_index,
                 next_slot, dst_len, valid, fp, metrics):
    """One GPU's record block: int64 [FIELDS * width + METRICS], field-major.
    ``dst_len[x]`` is the destination pattern length of xfer x; ``metrics``
    the four trailing values."""
    out = np.zeros(FIELDS * width + METRICS, np.int64)
    out[:width] = ABSENT
    n = min(int(count), width)
    if n:
        row = np.asarray(rows[:n], np.int64)
        parent = np.asarray(cand_batch, np.int64)[row]
        x = np.asarray(xfers[:n], np.int64)
        key1, key2 = pack_keys(np.asarray(next_gate[:n]), np.asarray(probs)[row],
                               np.asarray(gate)[parent], np.asarray(global_index)[parent], x,
                               row % k)
        out[:n] = key1
        out[width:width + n] = key2
        out[2 * width:2 * width + n] = np.asarray(fp[:n], np.int64)
        child_next = np.asarray(next_slot, np.int64)[parent] + np.asarray(dst_len, np.int64)[x]
        out[3 * width:3 * width + n] = child_next | (np.asarray(valid[:n]) != 0).astype(
            np.int64) << 32
    out[FIELDS * width:] = np.asarray(metrics, np.int64)
    return out


def merge_records(blocks, width, cap):
    """The first ``cap`` records of the union of the blocks in (KEY1, KEY2)
    order (equal keys: lower block first).  Returns a dict of per-position
    arrays (rows past the count: zero, src = len(blocks)), the count and
    the summed metrics."""
    world = len(blocks)
    key1 = np.concatenate([b[:width] for b in blocks])
    key2 = np.concatenate([b[width:2 * width] for b in blocks])
    fp = np.concatenate([b[2 * width:3 * width] for b in blocks])
    aux = np.concatenate([b[3 * width:4 * width] for b in blocks])
    src = np.repeat(np.arange(world), width)
    index = np.tile(np.arange(width), world)
    present = np.nonzero(key1 != ABSENT)[0]
    order = present[np.lexsort((src[present], key2[present], key1[present]))][:cap]
    count = order.size
    out = {"valid": np.zeros(cap, np.uint8), "fp": np.zeros(cap, np.int64),
           "next_gate": np.zeros(cap, np.int64), "src": np.full(cap, world, np.int64),
           "index": np.zeros(cap, np.int64), "child_next": np.zeros(cap, np.int64)}
    out["valid"][:count] = (aux[order] >> 32) & 1
    out["fp"][:count] = fp[order]
    out["next_gate"][:count] = key1[order] >> 44
    out["src"][:count] = src[order]
    out["index"][:count] = index[order]
    out["child_next"][:count] = aux[order] & 0xFFFFFFFF
    metrics = np.sum([b[FIELDS * width:FIELDS * width + METRICS] for b in blocks], axis=0)
    return out, count, metrics


def route(child_proposal, accepted, merged, world, me):
    """Placement of the ``accepted`` children (merged positions, global
    order).  Returns pairs [world, world] (moves s -> d; diagonal kept),
    extent, and GPU ``me``'s keep_local / keep_global / out_local /
    in_global lists."""
    src = [int(merged["src"][p]) for p in child_proposal[:accepted]]
    quota = [accepted // world + (1 if r < accepted % world else 0) for r in range(world)]
    seen = [0] * world
    dest = []
    overflow = []
    for j, s in enumerate(src):
        if seen[s] < quota[s]:
            dest.append(s)
        else:
            dest.append(-1)
            overflow.append(j)
        seen[s] += 1
    room = [quota[r] - min(seen[r], quota[r]) for r in range(world)]
    r = 0
    for j in overflow:
        while room[r] == 0:
            r += 1
        dest[j] = r
        room[r] -= 1
    pairs = np.zeros((world, world), np.int64)
    for s, d in zip(src, dest):
        pairs[s, d] += 1
    extent = max([int(merged["child_next"][p]) for p in child_proposal[:accepted]], default=0)
    index = [int(merged["index"][p]) for p in child_proposal[:accepted]]
    keep = [j for j in range(accepted) if src[j] == me and dest[j] == me]
    out = sorted((j for j in range(accepted) if src[j] == me and dest[j] != me),
                 key=lambda j: (dest[j], j))
    arriving = sorted((j for j in range(accepted) if dest[j] == me and src[j] != me),
                      key=lambda j: (src[j], j))
    return {"pairs": pairs, "extent": extent,
            "keep_local": np.asarray([index[j] for j in keep], np.int64),
            "keep_global": np.asarray(keep, np.int64),
            "out_local": np.asarray([index[j] for j in out], np.int64),
            "in_global": np.asarray(arriving, np.int64)}

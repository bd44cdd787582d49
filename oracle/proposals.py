"""Oracle proposal expansion and bounded ranking (NumPy, stable sorts).

Restates ``gpu_proposals.py``: the CSR source->allowed-xfer index keeps the
xfers of each source whose gate delta is at most ``max_gate_increase``
(``:20-50``); every candidate expands into its allowed xfers in index order
(``:102-118``); ``next_gate = parent_gate + delta`` (``:119-124``); a stable
lexicographic order (parent asc, next_gate asc, probability desc, xfer asc)
keeps the first ``per_parent_cap`` actions of each parent (``:128-143``); a
stable order (next_gate asc, probability desc, parent_gate asc) over the
survivors keeps the first ``global_cap`` (``:147-154``).  Ties left by every
key fall back to expansion order (stable sorts), i.e. ties break by index.
"""
from __future__ import annotations

import numpy as np


def build_rule_index(source_to_xfers: dict[int, list[int]], gate_deltas,
                     num_sources: int, max_gate_increase: int):
    allowed, offsets, counts, all_counts = [], [], [], []
    for source in range(num_sources):
        xs = source_to_xfers.get(source, [])
        sel = [x for x in xs if gate_deltas[x] <= max_gate_increase]
        offsets.append(len(allowed))
        allowed.extend(sel)
        counts.append(len(sel))
        all_counts.append(len(xs))
    return {
        "xfer_offsets": np.asarray(offsets, np.int64),
        "xfer_counts": np.asarray(counts, np.int64),
        "xfer_ids": np.asarray(allowed, np.int64),
        "gate_deltas": np.asarray(gate_deltas, np.int64),
        "all_xfer_counts": np.asarray(all_counts, np.int64),
    }


def rank_proposals(batch_ids, sources, anchors, bindings, probabilities,
                   parent_gate_counts, index, *, per_parent_cap: int,
                   global_cap: int):
    """Returns (selected expanded rows as dict of arrays, metrics)."""
    sources = np.asarray(sources, np.int64)
    counts = index["xfer_counts"][sources]
    predicted = int(index["all_xfer_counts"][sources].sum()) if sources.size else 0
    expanded = int(counts.sum()) if sources.size else 0
    if not expanded:
        empty = np.zeros(0, np.int64)
        return {"parent": empty, "xfer": empty, "anchor": empty,
                "binding": np.zeros((0, bindings.shape[1]), np.int64),
                "probability": np.zeros(0, np.float32), "next_gate": empty,
                "row": empty, "candidate": empty}, {"predicted_actions": predicted, "eligible_actions": 0}
    rows = np.repeat(np.arange(sources.size), counts)
    starts = np.cumsum(counts) - counts
    within = np.arange(expanded) - np.repeat(starts, counts)
    xfer = index["xfer_ids"][index["xfer_offsets"][sources[rows]] + within]
    parent = np.asarray(batch_ids, np.int64)[rows]
    prob = np.asarray(probabilities, np.float32)[rows]
    pgc = np.asarray(parent_gate_counts, np.int64)
    next_gate = pgc[parent] + index["gate_deltas"][xfer]
    # np.lexsort: last key is primary; stable.  Descending probability via
    # negation (exact for float32).
    order = np.lexsort((xfer, -prob, next_gate, parent))
    op = parent[order]
    new = np.ones(expanded, bool)
    new[1:] = op[1:] != op[:-1]
    pos = np.arange(expanded)
    start = np.maximum.accumulate(np.where(new, pos, 0))
    keep = order[(pos - start) < per_parent_cap]
    g = np.lexsort((pgc[parent[keep]], -prob[keep], next_gate[keep]))
    sel = keep[g[:global_cap]]
    return {
        "parent": parent[sel], "xfer": xfer[sel],
        "anchor": np.asarray(anchors, np.int64)[rows[sel]],
        "binding": np.asarray(bindings, np.int64)[rows[sel]],
        "probability": prob[sel], "next_gate": next_gate[sel], "row": sel,
        "candidate": rows[sel],
    }, {"predicted_actions": predicted, "eligible_actions": expanded}


def rank_proposals_exploration(primary: dict, exploration: dict, parent_gate_counts, index, *,
                               per_parent_cap: int, exploration_per_parent: int,
                               global_cap: int):
    """Proposals from a primary and an exploration model's candidates with a
    per-parent exploration quota: build_legacy_proposals
    (paged_rollout_benchmark.py:101-210) over candidates expanded like
    expand_action_rows (:88-98).

    `primary` / `exploration`: dicts of candidate arrays (batch_ids,
    sources, anchors, bindings [n, P] -1 padded, probabilities), each in its
    model's candidate order.  Per parent: each model's actions with an
    allowed gate delta, stably sorted by (next_gate, -probability, xfer); the
    first cap - quota primary actions, then exploration actions whose
    (xfer, anchor, binding) is not yet taken, then the remaining primary
    ones, until the cap; the parent's list stably re-sorted by the same key.
    All parents' lists, in parent order, stably sorted by (next_gate,
    -probability, parent gate) and cut at global_cap.  Returned rows index
    the concatenated candidate table [primary rows | exploration rows]."""
    pgc = np.asarray(parent_gate_counts, np.int64)
    quota = min(exploration_per_parent, per_parent_cap)
    primary_limit = per_parent_cap - quota

    def expand(cand, offset):
        """Per parent: (next_gate, -prob, xfer, anchor, binding, prob, row, parent) in
        expansion order, allowed deltas only; plus the predicted count."""
        per, predicted = {}, 0
        batch = np.asarray(cand["batch_ids"], np.int64)
        sources = np.asarray(cand["sources"], np.int64)
        for r in range(batch.size):
            s = int(sources[r])
            predicted += int(index["all_xfer_counts"][s])
            start, count = int(index["xfer_offsets"][s]), int(index["xfer_counts"][s])
            b = int(batch[r])
            binding = tuple(int(v) for v in cand["bindings"][r] if v >= 0)
            prob = float(np.float32(cand["probabilities"][r]))
            for x in index["xfer_ids"][start:start + count].tolist():
                ng = int(pgc[b] + index["gate_deltas"][x])
                per.setdefault(b, []).append((ng, -prob, x, int(cand["anchors"][r]), binding,
                                              prob, offset + r, b))
        for rows in per.values():
            rows.sort(key=lambda t: (t[0], t[1], t[2]))
        return per, predicted

    n_primary = np.asarray(primary["batch_ids"]).size
    p_rows, p_pred = expand(primary, 0)
    e_rows, e_pred = expand(exploration, n_primary)
    proposals, eligible, e_eligible, selected_exploration = [], 0, 0, 0
    for parent in range(pgc.size):
        prim, expl = p_rows.get(parent, []), e_rows.get(parent, [])
        eligible += len(prim)
        e_eligible += len(expl)
        chosen = list(prim[:primary_limit])
        keys = {(t[2], t[3], t[4]) for t in chosen}
        # the cap is checked after an append (:172-180): with no quota and a
        # full primary list one exploration proposal still joins
        for t in expl:
            key = (t[2], t[3], t[4])
            if key in keys:
                continue
            chosen.append(t)
            keys.add(key)
            selected_exploration += 1
            if len(chosen) >= per_parent_cap:
                break
        if len(chosen) < per_parent_cap:
            for t in prim[primary_limit:]:
                key = (t[2], t[3], t[4])
                if key in keys:
                    continue
                chosen.append(t)
                keys.add(key)
                if len(chosen) >= per_parent_cap:
                    break
        chosen.sort(key=lambda t: (t[0], t[1], t[2]))
        proposals.extend(chosen)
    proposals.sort(key=lambda t: (t[0], t[1], int(pgc[t[7]])))
    proposals = proposals[:global_cap]
    sel = {
        "parent": np.asarray([t[7] for t in proposals], np.int64),
        "xfer": np.asarray([t[2] for t in proposals], np.int64),
        "anchor": np.asarray([t[3] for t in proposals], np.int64),
        "binding": [t[4] for t in proposals],
        "probability": np.asarray([t[5] for t in proposals], np.float32),
        "next_gate": np.asarray([t[0] for t in proposals], np.int64),
        "candidate": np.asarray([t[6] for t in proposals], np.int64),
    }
    return sel, {"predicted_actions": p_pred, "exploration_predicted_actions": e_pred,
                 "eligible_actions": eligible, "exploration_eligible_actions": e_eligible,
                 "selected_exploration_proposals": selected_exploration}

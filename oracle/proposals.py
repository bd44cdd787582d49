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

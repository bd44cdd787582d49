"""Oracle candidate selection (threshold_inference.py:208-297).

Near/far affine calibration by rewrite distance (near = distance <= 2),
threshold mask on the raw logits, per-state top-k of the calibrated scores
over the flattened (slot, source) grid, sigmoid probabilities, then the
structural decoder's validity filter.  Ties among equal scores are broken by
the lower flat index (the CUDA kernel's rule; the reference leaves them to
``torch.topk``).
"""
from __future__ import annotations

import torch


def threshold_candidates(model, types, live, distance, edges, logits, eligible, config, *,
                         max_candidates_per_state: int, batch_offset: int = 0):
    near = distance.le(2)
    g = config["groups"]
    scale = torch.where(near, torch.tensor(g["near"]["scale"]), torch.tensor(g["far"]["scale"]))
    bias = torch.where(near, torch.tensor(g["near"]["bias"]), torch.tensor(g["far"]["bias"]))
    thr = torch.where(near, torch.tensor(g["near"]["raw_threshold"]),
                      torch.tensor(g["far"]["raw_threshold"]))
    calibrated = logits.float() * scale.unsqueeze(-1) + bias.unsqueeze(-1)
    selected = eligible & logits.ge(thr.unsqueeze(-1))
    flat = calibrated.flatten(1).masked_fill(~selected.flatten(1), -torch.inf)
    b, n = flat.shape
    k = min(max_candidates_per_state, n)
    # sort by (score desc, index asc)
    idx = torch.arange(n).expand(b, n)
    order = torch.argsort(flat, dim=1, descending=True, stable=True)[:, :k]
    scores = torch.gather(flat, 1, order)
    present = scores.isfinite()
    batch_ids = torch.arange(b).unsqueeze(1).expand_as(order)[present]
    scores, positions = scores[present], order[present]
    anchors = positions // model.num_sources
    sources = positions % model.num_sources
    probabilities = scores.sigmoid()
    bindings, valid = model.structural_decode(types, live, edges, batch_ids, sources, anchors)
    return {"batch_ids": batch_ids[valid] + batch_offset, "sources": sources[valid],
            "anchors": anchors[valid], "bindings": bindings[valid],
            "probabilities": probabilities[valid]}

"""Device layouts restated as the oracle's inputs (test infrastructure).

The device search keeps the port graph as per-slot port arrays and the
action history in paged arenas; the oracle (like the reference's
``InitialGraphLayer.forward``, model.py:26-53, and the dense-history branch of
``advance_incremental``, paged_model.py:444-613) takes edge lists and dense
per-beam histories.  These helpers convert one into the other on the host.
"""
from __future__ import annotations

import torch


def port_edges(out_node: torch.Tensor, out_port: torch.Tensor):
    """[B, S, 4] out-port arrays (-1 = unconnected) -> (batch, src, dst,
    relation) int64 edge lists with relation = src_port * 4 + dst_port
    (tensorized_batch.py:128)."""
    out_node = out_node.long().cpu()
    out_port = out_port.long().cpu()
    b, s, p = (out_node >= 0).nonzero(as_tuple=True)
    return b, s, out_node[b, s, p], p * 4 + out_port[b, s, p]


def dense_history(pages: torch.Tensor, table: torch.Tensor, lengths: torch.Tensor):
    """The first `length` token rows of every beam's block-table pages,
    [..., pages, page, H, D] -> [..., B, H, T, D] fp32 on the host (every beam
    of a search level has the same length)."""
    t = int(lengths.max()) if lengths.numel() else 0
    assert lengths.numel() == 0 or int(lengths.min()) == t, "ragged lengths"
    page = pages.shape[-3]
    pos = torch.arange(t, device=table.device)
    ids = table[:, pos // page].long()                        # [B, T]
    rows = pages[..., ids, pos % page, :, :]                  # [..., B, T, H, D]
    return rows.transpose(-3, -2).float().cpu()

"""Seeded device workloads for the benchmarks (no oracle dependency).

``decode_attention_workload`` builds the shared-prefix paged decode
microbenchmark: B beams, one query token each, H heads x 32, bf16; a
beam-invariant prefix of ``num_shared`` s0 node keys/values; ``tokens``
action K/V entries per beam in pages of ``page_size``; block tables from a
random prefix tree (each level expands every beam into ``branching``
children and samples B survivors uniformly), so the full pages completed by a
common ancestor are shared exactly as the copy-on-write cache shares them.
"""
from __future__ import annotations

from dataclasses import dataclass

import numpy as np
import torch


@dataclass
class DecodeAttentionWorkload:
    query: torch.Tensor          # [B, H, 1, D]
    key_cache: torch.Tensor      # [pages, page, H, D]
    value_cache: torch.Tensor
    block_table: torch.Tensor    # int32 [B, blocks]
    lengths: torch.Tensor        # int32 [B]
    shared_key: torch.Tensor     # [N, H, D]
    shared_value: torch.Tensor
    distinct_pages: int

    @property
    def logical_bytes(self) -> int:
        """Q + O + shared K/V once + every beam's history K/V counted per beam
        (pages shared through the prefix tree counted once per beam that
        reads them) + block table + lengths."""
        e = self.query.element_size()
        b, h, q, d = self.query.shape
        history = int(self.lengths.sum().item()) * h * d * e * 2
        return (2 * b * h * q * d * e + 2 * self.shared_key.numel() * e + history
                + self.block_table.numel() * 4 + self.lengths.numel() * 4)

    @property
    def unique_bytes(self) -> int:
        """Algorithmic HBM bytes of one launch: Q + O + shared K/V once +
        every distinct referenced page (K and V) + block table + lengths."""
        e = self.query.element_size()
        b, h, q, d = self.query.shape
        page_bytes = self.key_cache.shape[1] * h * d * e * 2
        return (2 * b * h * q * d * e + 2 * self.shared_key.numel() * e
                + self.distinct_pages * page_bytes + self.block_table.numel() * 4
                + self.lengths.numel() * 4)


def prefix_tree_tables(beams: int, tokens: int, page_size: int, branching: int,
                       seed: int) -> tuple[np.ndarray, int]:
    """Block tables of `beams` survivors after `tokens` levels of a random
    prefix tree.  Page j of a beam is the copy completed by its ancestor at
    level page_size*(j+1); beams sharing that ancestor share the page."""
    rng = np.random.default_rng(seed)
    blocks = -(-tokens // page_size)
    # ancestor id of every survivor at each completed-page level
    node_ids = np.arange(beams)           # ids of current survivors
    next_id = beams
    page_owner = np.zeros((beams, blocks), np.int64)
    for level in range(1, tokens + 1):
        children_parent = np.repeat(np.arange(beams), branching)
        pick = np.sort(rng.choice(beams * branching, size=beams, replace=False))
        parent = children_parent[pick]
        page_owner = page_owner[parent]
        node_ids = np.arange(next_id, next_id + beams)
        next_id += beams
        if level % page_size == 0 or level == tokens:
            page_owner[:, (level - 1) // page_size] = node_ids
    uniq, inverse = np.unique(page_owner, return_inverse=True)
    # scatter distinct pages over the arena in a seeded order
    physical = rng.permutation(len(uniq))
    table = physical[inverse.reshape(beams, blocks)].astype(np.int32)
    return table, len(uniq)


def decode_attention_workload(device, *, beams=512, heads=8, head_width=32, tokens=64,
                              page_size=16, num_shared=381, branching=4, seed=0,
                              dtype=torch.bfloat16) -> DecodeAttentionWorkload:
    table, distinct = prefix_tree_tables(beams, tokens, page_size, branching, seed)
    g = torch.Generator(device="cpu").manual_seed(seed)
    shape = (distinct, page_size, heads, head_width)
    key_cache = torch.randn(shape, generator=g).to(device, dtype)
    value_cache = torch.randn(shape, generator=g).to(device, dtype)
    query = torch.randn(beams, heads, 1, head_width, generator=g).to(device, dtype)
    shared_key = torch.randn(num_shared, heads, head_width, generator=g).to(device, dtype)
    shared_value = torch.randn(num_shared, heads, head_width, generator=g).to(device, dtype)
    lengths = torch.full((beams,), tokens, dtype=torch.int32, device=device)
    return DecodeAttentionWorkload(query, key_cache, value_cache,
                                   torch.from_numpy(table).to(device), lengths, shared_key,
                                   shared_value, distinct)

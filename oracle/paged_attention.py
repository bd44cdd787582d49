"""Oracle paged attention: gather pages, then masked softmax attention.

Restates ``paged_attention.py:162-214`` (``_contiguous_from_pages`` and
``paged_attention_reference``) and the kernel semantics of
``paged_attention.py:101-145``: a query attends to the first ``lengths[b]``
tokens of its block-table pages plus, optionally, the current token at
position ``lengths[b]`` when ``current_valid[b]``; rows with no valid key
return zeros.  The shared-prefix form prepends ``shared_key/value`` [N, H, D]
(the same for every beam) to each beam's keys.
"""
from __future__ import annotations

import math

import torch


def contiguous_from_pages(cache: torch.Tensor, block_table: torch.Tensor,
                          max_length: int) -> torch.Tensor:
    """[pages, page, H, D] -> [B, H, T, D] (paged_attention.py:162-179)."""
    batch = block_table.shape[0]
    page = cache.shape[1]
    if not max_length:
        return cache.new_zeros(batch, cache.shape[2], 0, cache.shape[3])
    positions = torch.arange(max_length)
    columns = positions // page
    pages = block_table.long().index_select(1, columns)
    tokens = pages * page + positions % page
    flat = cache.reshape(-1, cache.shape[2], cache.shape[3])
    return flat[tokens].transpose(1, 2)


def paged_attention(query, key_cache, value_cache, block_table, lengths, *,
                    current_key=None, current_value=None, current_valid=None,
                    shared_key=None, shared_value=None) -> torch.Tensor:
    """fp64 accumulation reference; returns float32 [B, H, Q, D]."""
    if (current_key is None) != (current_value is None) or (
        (current_key is None) != (current_valid is None)
    ):
        raise ValueError("current key/value/valid must be supplied together")
    q = query.double()
    lengths = lengths.long()
    max_past = int(lengths.max()) if lengths.numel() else 0
    keys = contiguous_from_pages(key_cache.double(), block_table, max_past)
    values = contiguous_from_pages(value_cache.double(), block_table, max_past)
    mask = torch.arange(max_past).unsqueeze(0) < lengths.unsqueeze(1)
    if current_key is not None:
        keys = torch.cat((keys, current_key.double().unsqueeze(2)), dim=2)
        values = torch.cat((values, current_value.double().unsqueeze(2)), dim=2)
        mask = torch.cat((mask, current_valid.bool().unsqueeze(1)), dim=1)
    if shared_key is not None:
        b = q.shape[0]
        sk = shared_key.double().permute(1, 0, 2).unsqueeze(0).expand(b, -1, -1, -1)
        sv = shared_value.double().permute(1, 0, 2).unsqueeze(0).expand(b, -1, -1, -1)
        keys = torch.cat((sk, keys), dim=2)
        values = torch.cat((sv, values), dim=2)
        mask = torch.cat((torch.ones(b, shared_key.shape[0], dtype=torch.bool), mask), 1)
    if not keys.shape[2]:
        return torch.zeros(query.shape, dtype=torch.float32)
    scores = torch.einsum("bhqd,bhtd->bhqt", q, keys) / math.sqrt(q.shape[-1])
    scores = scores.masked_fill(~mask[:, None, None, :], float("-inf"))
    any_valid = mask.any(1)
    scores = torch.where(any_valid[:, None, None, None], scores, torch.zeros_like(scores))
    probs = torch.softmax(scores, dim=-1)
    out = torch.einsum("bhqt,bhtd->bhqd", probs, values)
    out = out * any_valid[:, None, None, None]
    return out.float()

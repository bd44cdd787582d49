"""Oracle PagedKVCache: host refcounts + LIFO free list + CPU arenas.

Restates ``paged_cache.py:16-238``: the free list starts as
``[capacity-1, ..., 0]`` and allocation pops from its end (``:75``, ``:85-92``);
``append_batch`` walks parents in order, retaining shared pages before it
allocates the child's page, copying the valid rows of a partial tail page
(COW) and writing one new row per arena (``:140-207``); ``release`` decrements
each page of a handle and appends pages that reach zero in scan order
(``:99-105``); ``block_table`` pads rows with page 0 to at least one column
(``:210-238``).  Error messages match the reference.
"""
from __future__ import annotations

from dataclasses import dataclass

import torch


@dataclass(frozen=True)
class PrefixHandle:
    blocks: tuple[int, ...]
    length: int


class OraclePagedKVCache:
    def __init__(self, *, layers, capacity, page_size, heads, head_width,
                 model_width, dtype=torch.float32):
        if min(layers, capacity, page_size, heads, head_width, model_width) <= 0:
            raise ValueError("all cache dimensions must be positive")
        self.layers, self.capacity, self.page_size = layers, capacity, page_size
        self.heads, self.head_width, self.model_width = heads, head_width, model_width
        self.keys = torch.zeros(layers, capacity, page_size, heads, head_width, dtype=dtype)
        self.values = torch.zeros_like(self.keys)
        self.actions = torch.zeros(capacity, page_size, model_width, dtype=dtype)
        self.readout_keys = torch.zeros(capacity, page_size, heads, head_width, dtype=dtype)
        self.readout_values = torch.zeros_like(self.readout_keys)
        self.refcounts = [0] * capacity
        self.free = list(range(capacity - 1, -1, -1))

    @property
    def allocated_pages(self) -> int:
        return self.capacity - len(self.free)

    @staticmethod
    def empty_handle() -> PrefixHandle:
        return PrefixHandle((), 0)

    def _allocate(self) -> int:
        if not self.free:
            raise RuntimeError("paged KV cache exhausted")
        page = self.free.pop()
        if self.refcounts[page] != 0:
            raise RuntimeError("free-list corruption")
        self.refcounts[page] = 1
        return page

    def _retain(self, page: int) -> None:
        if self.refcounts[page] <= 0:
            raise RuntimeError("retaining an unallocated page")
        self.refcounts[page] += 1

    def release(self, handle: PrefixHandle) -> None:
        for page in handle.blocks:
            self.refcounts[page] -= 1
            if self.refcounts[page] < 0:
                raise RuntimeError("negative page reference count")
            if self.refcounts[page] == 0:
                self.free.append(page)

    def append_batch(self, parents, keys, values, actions, readout_keys=None,
                     readout_values=None):
        n = len(parents)
        expected = (self.layers, n, self.heads, self.head_width)
        if tuple(keys.shape) != expected or tuple(values.shape) != expected:
            raise ValueError(f"expected KV shape {expected}")
        if tuple(actions.shape) != (n, self.model_width):
            raise ValueError("invalid action-state shape")
        if (readout_keys is None) != (readout_values is None):
            raise ValueError("readout keys and values must be supplied together")
        children, pages, offsets, copies = [], [], [], []
        for parent in parents:
            offset = parent.length % self.page_size
            if offset == 0:
                for page in parent.blocks:
                    self._retain(page)
                page = self._allocate()
                blocks = parent.blocks + (page,)
            else:
                for page in parent.blocks[:-1]:
                    self._retain(page)
                tail = parent.blocks[-1]
                page = self._allocate()
                copies.append((tail, page, offset))
                blocks = parent.blocks[:-1] + (page,)
            children.append(PrefixHandle(blocks, parent.length + 1))
            pages.append(page)
            offsets.append(offset)
        for tail, page, offset in copies:
            self.keys[:, page, :offset] = self.keys[:, tail, :offset]
            self.values[:, page, :offset] = self.values[:, tail, :offset]
            self.actions[page, :offset] = self.actions[tail, :offset]
            if readout_keys is not None:
                self.readout_keys[page, :offset] = self.readout_keys[tail, :offset]
                self.readout_values[page, :offset] = self.readout_values[tail, :offset]
        for i, (page, offset) in enumerate(zip(pages, offsets)):
            self.keys[:, page, offset] = keys[:, i].to(self.keys.dtype)
            self.values[:, page, offset] = values[:, i].to(self.keys.dtype)
            self.actions[page, offset] = actions[i].to(self.keys.dtype)
            if readout_keys is not None:
                self.readout_keys[page, offset] = readout_keys[i].to(self.keys.dtype)
                self.readout_values[page, offset] = readout_values[i].to(self.keys.dtype)
        return children

    def block_table(self, handles):
        max_blocks = max([len(h.blocks) for h in handles] + [1])
        rows, lengths = [], []
        for h in handles:
            if (h.length + self.page_size - 1) // self.page_size != len(h.blocks):
                raise RuntimeError("prefix handle length/block table mismatch")
            rows.append(list(h.blocks) + [0] * (max_blocks - len(h.blocks)))
            lengths.append(h.length)
        return (torch.tensor(rows, dtype=torch.int32).reshape(len(handles), max_blocks),
                torch.tensor(lengths, dtype=torch.int32))

    def gather(self, handles):
        """Contiguous [L,B,H,T,D] K/V, [B,T,W] actions, [B,T] mask (``:240-344``)."""
        n = len(handles)
        t = max([h.length for h in handles] + [0])
        keys = torch.zeros(self.layers, n, self.heads, t, self.head_width, dtype=self.keys.dtype)
        values = torch.zeros_like(keys)
        actions = torch.zeros(n, t, self.model_width, dtype=self.keys.dtype)
        mask = torch.zeros(n, t, dtype=torch.bool)
        for b, h in enumerate(handles):
            for pos in range(h.length):
                page = h.blocks[pos // self.page_size]
                row = pos % self.page_size
                keys[:, b, :, pos] = self.keys[:, page, row]
                values[:, b, :, pos] = self.values[:, page, row]
                actions[b, pos] = self.actions[page, row]
                mask[b, pos] = True
        return keys, values, actions, mask

"""PagedKVCache with the reference's Python API, run in place on the device.

Mirrors ``paged_cache.py:16-386``: constructor arguments, attributes
(``keys, values, actions, readout_keys, readout_values, refcounts, free,
capacity, page_size``), ``empty_handle``, ``append_batch``, ``release``,
``block_table``, ``allocated_pages``, ``gather`` and ``gather_actions``, with
the same exceptions and messages.  Page ownership (refcounts, the LIFO free
list) lives in device memory and is updated by the kernels of
``csrc/paged_cache.cu``; the allocation order is bit-exact with the
reference's host lists.

Two layers:

* the reference API, with immutable ``PrefixHandle(blocks, length)`` values;
  each call checks the device status word (one synchronisation, as the
  reference's host loop raises immediately);
* a device-native API (``append_device`` / ``release_device``) over int32
  block-table tensors that never synchronises; ``check_status`` raises the
  first recorded error once per step.
"""
from __future__ import annotations

from dataclasses import dataclass

import numpy as np
import torch

from . import _lib



@dataclass(frozen=True)
class PrefixHandle:
    """Logical ownership of one paged causal prefix (paged_cache.py:8-13)."""

    blocks: tuple[int, ...]
    length: int


class PagedKVCache:
    """Fixed-size device KV/action pool with prefix sharing and COW tail pages."""

    def __init__(self, *, layers: int, capacity: int, page_size: int, heads: int,
                 head_width: int, model_width: int, device, dtype: torch.dtype,
                 gather_backend: str = "vectorized"):
        if min(layers, capacity, page_size, heads, head_width, model_width) <= 0:
            raise ValueError("all cache dimensions must be positive")
        if gather_backend not in {"loop", "vectorized"}:
            raise ValueError("gather_backend must be 'loop' or 'vectorized'")
        device = torch.device(device)
        if device.type != "cuda":
            raise RuntimeError("PagedKVCache lives in CUDA memory (no CPU fallback)")
        if dtype not in (torch.bfloat16, torch.float32):
            raise ValueError("PagedKVCache arenas are bf16 or fp32")
        self.layers, self.capacity, self.page_size = layers, capacity, page_size
        self.heads, self.head_width, self.model_width = heads, head_width, model_width
        self.device, self.dtype, self.gather_backend = device, dtype, gather_backend
        self.keys = torch.empty(layers, capacity, page_size, heads, head_width,
                                device=device, dtype=dtype)
        self.values = torch.empty_like(self.keys)
        self.actions = torch.empty(capacity, page_size, model_width, device=device, dtype=dtype)
        self.readout_keys = torch.empty(capacity, page_size, heads, head_width,
                                        device=device, dtype=dtype)
        self.readout_values = torch.empty_like(self.readout_keys)
        i32 = dict(device=device, dtype=torch.int32)
        self._refcounts = torch.empty(capacity, **i32)
        self._free = torch.empty(capacity, **i32)
        self._free_count = torch.empty(1, **i32)
        self._last_pos = torch.empty(capacity, **i32)
        self._status = torch.zeros(1, **i32)
        _lib.check(_lib.lib().grs_cache_init(
            self._refcounts.data_ptr(), self._free.data_ptr(), self._free_count.data_ptr(),
            self._last_pos.data_ptr(), capacity, self._stream()), "PagedKVCache")

    def reset(self) -> None:
        """Return every page to the free list (the state of a new cache)."""
        self._status.zero_()
        _lib.check(_lib.lib().grs_cache_init(
            self._refcounts.data_ptr(), self._free.data_ptr(), self._free_count.data_ptr(),
            self._last_pos.data_ptr(), self.capacity, self._stream()), "PagedKVCache")

    def status_tensor(self) -> torch.Tensor:
        """The device status word (0 = ok) without synchronising."""
        return self._status

    # ---- state views (device -> host) -------------------------------------
    def _stream(self) -> int:
        return torch.cuda.current_stream(self.device).cuda_stream

    @property
    def refcounts(self) -> list[int]:
        return self._refcounts.tolist()

    @property
    def free(self) -> list[int]:
        count = int(self._free_count.item())
        return self._free[:count].tolist()

    @property
    def allocated_pages(self) -> int:
        return self.capacity - int(self._free_count.item())

    def free_count_tensor(self) -> torch.Tensor:
        """The device free-page count (int32 [1]) itself, no synchronisation."""
        return self._free_count

    def allocated_pages_tensor(self) -> torch.Tensor:
        """Allocated page count as a device scalar (no synchronisation)."""
        return self.capacity - self._free_count

    @staticmethod
    def empty_handle() -> PrefixHandle:
        return PrefixHandle((), 0)

    def check_status(self) -> None:
        """Raise the first error recorded by a kernel since the last check."""
        code = int(self._status.item())
        if code:
            self._status.zero_()
            _lib.check(code, "PagedKVCache")

    # ---- device-native API ------------------------------------------------
    def append_device(self, parent_table: torch.Tensor, parent_lengths: torch.Tensor,
                      keys: torch.Tensor, values: torch.Tensor, actions: torch.Tensor,
                      readout_keys: torch.Tensor | None = None,
                      readout_values: torch.Tensor | None = None,
                      child_cols: int | None = None):
        """Append one token to each parent row; returns (child_table, child_lengths).

        ``parent_table`` int32 [n, cols], ``parent_lengths`` int32 [n].  No
        host synchronisation; errors land in the status word.
        """
        n = parent_lengths.shape[0]
        expected = (self.layers, n, self.heads, self.head_width)
        if tuple(keys.shape) != expected or tuple(values.shape) != expected:
            raise ValueError(f"expected KV shape {expected}")
        if tuple(actions.shape) != (n, self.model_width):
            raise ValueError("invalid action-state shape")
        readout_shape = (n, self.heads, self.head_width)
        if (readout_keys is None) != (readout_values is None):
            raise ValueError("readout keys and values must be supplied together")
        if readout_keys is not None and (tuple(readout_keys.shape) != readout_shape
                                         or tuple(readout_values.shape) != readout_shape):
            raise ValueError(f"expected readout KV shape {readout_shape}")
        cols = parent_table.shape[1] if parent_table.dim() == 2 else 0
        child_cols = child_cols or max(1, cols + 1)
        child_table = torch.empty(n, child_cols, device=self.device, dtype=torch.int32)
        child_lengths = torch.empty(n, device=self.device, dtype=torch.int32)
        if n == 0:
            return child_table, child_lengths
        parent_table = parent_table.to(torch.int32)
        if parent_table.stride(-1) != 1:
            parent_table = parent_table.contiguous()
        parent_lengths = parent_lengths.to(torch.int32).contiguous()
        conv = lambda t: None if t is None else t.to(self.dtype).contiguous()
        keys, values, actions = conv(keys), conv(values), conv(actions)
        readout_keys, readout_values = conv(readout_keys), conv(readout_values)
        status = _lib.lib().grs_cache_append(
            self.keys.element_size(), self._refcounts.data_ptr(), self._free.data_ptr(),
            self._free_count.data_ptr(), self.capacity, parent_table.data_ptr(),
            parent_table.stride(0), parent_lengths.data_ptr(), n, self.page_size,
            child_table.data_ptr(), child_table.stride(0), child_lengths.data_ptr(),
            child_cols, self.keys.data_ptr(), self.values.data_ptr(), self.layers,
            self.heads * self.head_width, keys.data_ptr(), values.data_ptr(),
            self.actions.data_ptr(), self.model_width, actions.data_ptr(),
            self.readout_keys.data_ptr(), self.readout_values.data_ptr(),
            _lib.ptr(readout_keys), _lib.ptr(readout_values), self._status.data_ptr(),
            self._stream())
        _lib.check(status, "append_batch")
        return child_table, child_lengths

    def release_device(self, table: torch.Tensor, lengths: torch.Tensor) -> None:
        """Release handles given as device rows, in row order (no sync)."""
        n = lengths.shape[0]
        if n == 0:
            return
        table = table.to(torch.int32)
        if table.stride(-1) != 1:
            table = table.contiguous()
        lengths = lengths.to(torch.int32).contiguous()
        _lib.check(_lib.lib().grs_cache_release(
            self._refcounts.data_ptr(), self._free.data_ptr(), self._free_count.data_ptr(),
            self._last_pos.data_ptr(), self.capacity, table.data_ptr(), table.stride(0),
            lengths.data_ptr(), n, table.shape[1], self.page_size, self._status.data_ptr(),
            self._stream()), "release")

    # ---- moving rows between caches (sharded beam search) -------------------
    def arenas(self) -> list[torch.Tensor]:
        """Every arena as a [capacity, page elements] view (page-major), per
        layer for the K/V arenas."""
        cap = self.capacity
        return ([self.keys[l].view(cap, -1) for l in range(self.layers)]
                + [self.values[l].view(cap, -1) for l in range(self.layers)]
                + [self.actions.view(cap, -1), self.readout_keys.view(cap, -1),
                   self.readout_values.view(cap, -1)])

    @property
    def page_bytes(self) -> int:
        """Bytes one page holds across all arenas."""
        return sum(a.shape[1] * a.element_size() for a in self.arenas())

    def alloc_pages(self, n: int) -> torch.Tensor:
        """Allocate n pages (refcount 1, free-list order) for contents copied
        in from another cache; returns their ids (device int32)."""
        pages = torch.empty(n, device=self.device, dtype=torch.int32)
        if n:
            _lib.check(_lib.lib().grs_cache_alloc(
                self._refcounts.data_ptr(), self._free.data_ptr(), self._free_count.data_ptr(),
                self.capacity, n, pages.data_ptr(), self._status.data_ptr(), self._stream()),
                "alloc_pages")
        return pages

    # ---- reference API ----------------------------------------------------
    def _handle_rows(self, handles: list[PrefixHandle], min_cols: int = 1):
        cols = max([len(h.blocks) for h in handles] + [min_cols])
        rows = np.zeros((len(handles), cols), dtype=np.int32)
        lengths = np.empty(len(handles), dtype=np.int32)
        for i, h in enumerate(handles):
            if (h.length + self.page_size - 1) // self.page_size != len(h.blocks):
                raise RuntimeError("prefix handle length/block table mismatch")
            if any(not 0 <= p < self.capacity for p in h.blocks):
                raise ValueError("prefix handle names a page outside the cache")
            rows[i, : len(h.blocks)] = h.blocks
            lengths[i] = h.length
        table = torch.from_numpy(rows).to(self.device, non_blocking=True)
        length_tensor = torch.from_numpy(lengths).to(self.device, non_blocking=True)
        return table, length_tensor

    def release(self, handle: PrefixHandle) -> None:
        if not handle.blocks:
            return
        table, lengths = self._handle_rows([handle])
        self.release_device(table, lengths)
        self.check_status()

    def append_batch(self, parents: list[PrefixHandle], keys: torch.Tensor,
                     values: torch.Tensor, actions: torch.Tensor,
                     readout_keys: torch.Tensor | None = None,
                     readout_values: torch.Tensor | None = None) -> list[PrefixHandle]:
        """Append one causal token to each parent (keys/values [L, B, H, D])."""
        n = len(parents)
        expected = (self.layers, n, self.heads, self.head_width)
        if tuple(keys.shape) != expected or tuple(values.shape) != expected:
            raise ValueError(f"expected KV shape {expected}")
        if not n:
            return []
        table, lengths = self._handle_rows(parents)
        child_table, child_lengths = self.append_device(
            table, lengths, keys, values, actions, readout_keys, readout_values,
            child_cols=table.shape[1] + 1)
        self.check_status()
        rows = child_table.cpu().numpy()
        out = []
        for i, parent in enumerate(parents):
            length = parent.length + 1
            nb = (length + self.page_size - 1) // self.page_size
            out.append(PrefixHandle(tuple(int(p) for p in rows[i, :nb]), length))
        return out

    def block_table(self, handles: list[PrefixHandle]) -> tuple[torch.Tensor, torch.Tensor]:
        """Padded physical page ids (>= 1 column) and logical lengths (int32)."""
        return self._handle_rows(handles, min_cols=1)

    def _token_indices(self, handles):
        n = len(handles)
        t = max([h.length for h in handles] + [0])
        if not n or not t:
            return (torch.empty((n, t), device=self.device, dtype=torch.long),
                    torch.zeros((n, t), device=self.device, dtype=torch.bool))
        table, lengths = self.block_table(handles)
        positions = torch.arange(t, device=self.device)
        pages = table.long().index_select(1, positions // self.page_size)
        tokens = pages * self.page_size + positions % self.page_size
        mask = positions.unsqueeze(0) < lengths.unsqueeze(1)
        return tokens, mask

    def gather(self, handles: list[PrefixHandle]):
        """Contiguous K/V [L,B,H,T,D], actions [B,T,W] and mask (API compatibility;
        the decode path reads pages in place and never gathers)."""
        tokens, mask = self._token_indices(handles)
        flat_k = self.keys.reshape(self.layers, -1, self.heads, self.head_width)
        flat_v = self.values.reshape_as(flat_k)
        keys = flat_k[:, tokens].permute(0, 1, 3, 2, 4)
        values = flat_v[:, tokens].permute(0, 1, 3, 2, 4)
        m = mask[None, :, None, :, None]
        keys = keys.masked_fill(~m, 0)
        values = values.masked_fill(~m, 0)
        actions = self.actions.reshape(-1, self.model_width)[tokens]
        actions = actions.masked_fill(~mask.unsqueeze(-1), 0)
        return keys, values, actions, mask

    def gather_actions(self, handles: list[PrefixHandle]):
        tokens, mask = self._token_indices(handles)
        actions = self.actions.reshape(-1, self.model_width)[tokens]
        return actions.masked_fill(~mask.unsqueeze(-1), 0), mask

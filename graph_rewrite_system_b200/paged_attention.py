"""Paged attention with the reference's Python API (paged_attention.py:217-306).

``paged_attention(query, key_cache, value_cache, block_table, lengths, *,
current_key=None, current_value=None, current_valid=None)`` attends each
(beam, head, query) row to the first ``lengths[b]`` tokens of the beam's
block-table pages plus, when given, the current token at position
``lengths[b]`` (``current_valid[b]``).  Rows with no valid key are zero.
The sm_100a kernels live in ``csrc/paged_attention.cu``; CPU tensors raise.

``shared_key``/``shared_value`` ([N, H, D], beam-invariant) extend the
reference API for the shared-prefix decode microbenchmark; ``status`` (device
int32) receives in-kernel errors of the decode kernels (default: a
per-device word read by ``check_decode_status``).

bf16 one-query decode runs on ``grs_decode_causal`` (page-staged, one CTA per
beam) or, with a shared prefix, ``grs_decode_attention_shared`` (one CTA
per 32 beams and head); other shapes and fp32 on ``grs_paged_attention``.
"""
from __future__ import annotations

import torch

from . import _lib


_STATUS: dict[torch.device, torch.Tensor] = {}


def _status_word(device: torch.device) -> torch.Tensor:
    """Device int32 that the shared-prefix decode kernel sets to a negative
    status when one of its bounded in-kernel waits gives up."""
    if device not in _STATUS:
        _STATUS[device] = torch.zeros(1, dtype=torch.int32, device=device)
    return _STATUS[device]


def check_decode_status(device: torch.device | str = "cuda") -> None:
    """Raise if a shared-prefix decode launch on `device` reported an error
    (reads the device status word: one synchronisation), then clear it."""
    device = torch.device(device)
    if device.index is None:
        device = torch.device(device.type, torch.cuda.current_device())
    word = _status_word(device)
    code = int(word.item())
    word.zero_()
    _lib.check(code, "shared-prefix decode attention")


def paged_attention(
    query: torch.Tensor,
    key_cache: torch.Tensor,
    value_cache: torch.Tensor,
    block_table: torch.Tensor,
    lengths: torch.Tensor,
    *,
    current_key: torch.Tensor | None = None,
    current_value: torch.Tensor | None = None,
    current_valid: torch.Tensor | None = None,
    shared_key: torch.Tensor | None = None,
    shared_value: torch.Tensor | None = None,
    out: torch.Tensor | None = None,
    status: torch.Tensor | None = None,
) -> torch.Tensor:
    has_current = current_key is not None
    if has_current != (current_value is not None and current_valid is not None):
        raise ValueError("current key/value/valid must be supplied together")
    if (shared_key is None) != (shared_value is None):
        raise ValueError("shared key/value must be supplied together")
    _lib.require_cuda(query, key_cache, value_cache, block_table, lengths,
                      current_key, current_value, current_valid, shared_key, shared_value)
    if query.dtype not in _lib.DTYPE_CODES or key_cache.dtype != query.dtype:
        raise ValueError("paged_attention supports bf16 or fp32 query and cache of one dtype")
    batch, heads, query_length, head_width = query.shape
    if key_cache.shape[2:] != (heads, head_width) or value_cache.shape != key_cache.shape:
        raise ValueError("cache must be [pages, page, heads, head_width]")
    if key_cache.stride() != value_cache.stride() or key_cache.stride(3) != 1:
        raise ValueError("key/value caches must share a layout with contiguous head_width")
    if shared_key is not None and (shared_key.dim() != 3
                                   or shared_key.shape[1:] != (heads, head_width)
                                   or shared_value.shape != shared_key.shape):
        raise ValueError("shared key/value must be [num_shared, heads, head_width]")
    if has_current and (current_key.shape != (batch, heads, head_width)
                        or current_value.shape != current_key.shape
                        or current_valid.shape != (batch,)):
        raise ValueError("current key/value must be [batch, heads, head_width], valid [batch]")
    if out is not None and (out.shape != query.shape or out.dtype != query.dtype
                            or out.stride(3) != 1):
        raise ValueError("out must match the query's shape and dtype with contiguous head_width")
    if query.stride(3) != 1:
        query = query.contiguous()
    block_table = block_table.to(torch.int32)
    lengths = lengths.to(torch.int32).contiguous()
    if block_table.dim() != 2 or block_table.shape[0] != batch or block_table.stride(1) != 1:
        block_table = block_table.reshape(batch, -1).contiguous()
    output = torch.empty_like(query) if out is None else out
    if not query_length or not batch:
        return output.zero_() if out is not None else torch.zeros_like(query)
    ck = cv = valid = None
    ck_sb = ck_sh = 0
    if has_current:
        ck = current_key.to(query.dtype)
        cv = current_value.to(query.dtype)
        if ck.stride(2) != 1 or cv.stride() != ck.stride():
            ck, cv = ck.contiguous(), cv.contiguous()
        ck_sb, ck_sh = ck.stride(0), ck.stride(1)
        valid = current_valid
        if valid.dtype not in (torch.uint8, torch.bool) or not valid.is_contiguous():
            valid = valid.to(torch.uint8).contiguous()
    status_word = _status_word(query.device) if status is None else status
    if (shared_key is None and query.dtype == torch.bfloat16 and query_length == 1
            and head_width == 32):
        # one query per (beam, head) over the beam's pages (+ the current
        # token): the page-staged causal decode kernel
        code = _lib.lib().grs_decode_causal(
            query.data_ptr(), query.stride(0), query.stride(1), key_cache.data_ptr(),
            value_cache.data_ptr(), key_cache.stride(0), key_cache.stride(1),
            key_cache.stride(2), block_table.data_ptr(), block_table.stride(0),
            lengths.data_ptr(), key_cache.shape[0], _lib.ptr(ck), _lib.ptr(cv), ck_sb, ck_sh,
            _lib.ptr(valid), output.data_ptr(), output.stride(0), output.stride(1), batch, heads,
            key_cache.shape[1], status_word.data_ptr(), _lib.stream_of(query))
        if code == 0:
            return output
        # only a layout the kernel does not take (nothing launched) goes on to
        # the general kernel; a failed launch raises
        if code != _lib.GRS_ERR_SHAPE:
            _lib.check(code, "causal decode attention")
    sk = sv = None
    num_shared = 0
    if shared_key is not None:
        sk = shared_key.to(query.dtype).contiguous()
        sv = shared_value.to(query.dtype).contiguous()
        num_shared = sk.shape[0]
    if (shared_key is not None and query.dtype == torch.bfloat16 and query_length == 1
            and head_width == 32 and heads <= 8 and query.stride(3) == 1
            and key_cache.stride(3) == 1 and value_cache.stride() == key_cache.stride()):
        code = _lib.lib().grs_decode_attention_shared(
            query.data_ptr(), query.stride(0), query.stride(1), key_cache.data_ptr(),
            value_cache.data_ptr(), key_cache.stride(0), key_cache.stride(1),
            key_cache.stride(2), block_table.data_ptr(), block_table.stride(0),
            block_table.shape[1], lengths.data_ptr(), key_cache.shape[0], _lib.ptr(ck),
            _lib.ptr(cv), ck_sb, ck_sh,
            _lib.ptr(valid), sk.data_ptr(), sv.data_ptr(), num_shared, output.data_ptr(),
            output.stride(0), output.stride(1), batch, heads, key_cache.shape[1],
            status_word.data_ptr(), _lib.stream_of(query))
        if code == 0:
            return output
        # only a layout the grouped kernel does not take (nothing launched)
        # goes on to the general kernel; a failed launch raises
        if code != _lib.GRS_ERR_SHAPE:
            _lib.check(code, "shared-prefix decode attention")
    code = _lib.lib().grs_paged_attention(
        _lib.DTYPE_CODES[query.dtype],
        query.data_ptr(), query.stride(0), query.stride(1), query.stride(2),
        key_cache.data_ptr(), value_cache.data_ptr(),
        key_cache.stride(0), key_cache.stride(1), key_cache.stride(2),
        block_table.data_ptr(), block_table.stride(0), lengths.data_ptr(),
        _lib.ptr(ck), _lib.ptr(cv), ck_sb, ck_sh, _lib.ptr(valid),
        _lib.ptr(sk), _lib.ptr(sv), num_shared,
        output.data_ptr(), output.stride(0), output.stride(1), output.stride(2),
        batch, heads, query_length, head_width, key_cache.shape[1], block_table.shape[1],
        key_cache.shape[0], _lib.stream_of(query),
    )
    _lib.check(code, "paged_attention")
    return output

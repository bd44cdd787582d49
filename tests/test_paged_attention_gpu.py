"""CUDA paged attention vs the oracle (tolerances: fp32 1e-5 relative; bf16 2e-2)."""
from __future__ import annotations

import numpy as np
import pytest
import torch

from conftest import load_golden
from oracle import paged_attention as oracle

pytestmark = pytest.mark.gpu


def _run(dev, g, dtype, with_current):
    from graph_rewrite_system_b200.paged_attention import paged_attention

    t = lambda k: torch.from_numpy(g[k]).to(dev)
    kwargs = {}
    if with_current:
        kwargs = dict(current_key=t("current_key").to(dtype), current_value=t("current_value").to(dtype),
                      current_valid=t("current_valid"))
    return paged_attention(t("query").to(dtype), t("keys").to(dtype), t("values").to(dtype),
                           t("block_table"), t("lengths"), **kwargs)


@pytest.mark.parametrize("name,with_current", [("paged_attention_history.npz", False),
                                               ("paged_attention_current.npz", True)])
def test_golden_fp32(cuda_device, name, with_current):
    g = load_golden(name)
    out = _run(cuda_device, g, torch.float32, with_current).cpu().numpy()
    np.testing.assert_allclose(out, g["output"], rtol=1e-5, atol=1e-5)
    if not with_current:
        assert not out[0].any()


@pytest.mark.parametrize("name,with_current", [("paged_attention_history.npz", False),
                                               ("paged_attention_current.npz", True)])
def test_golden_bf16(cuda_device, name, with_current):
    g = load_golden(name)
    out = _run(cuda_device, g, torch.bfloat16, with_current).float().cpu().numpy()
    # the reference's own bf16 tolerance (test_paged_attention.py:57)
    np.testing.assert_allclose(out, g["output"], rtol=2e-2, atol=2e-2)


def _random_case(seed, batch, heads, hw, page, cap, q, max_len, dtype, dev, shared=0,
                 current=False):
    g = torch.Generator().manual_seed(seed)
    keys = torch.randn(cap, page, heads, hw, generator=g)
    values = torch.randn(cap, page, heads, hw, generator=g)
    lengths = torch.randint(0, max_len + 1, (batch,), generator=g, dtype=torch.int32)
    lengths[0] = 0
    lengths[-1] = max_len
    cols = max(1, -(-max_len // page))
    table = torch.randint(0, cap, (batch, cols), generator=g, dtype=torch.int32)
    query = torch.randn(batch, heads, q, hw, generator=g)
    kw = {}
    if shared:
        kw["shared_key"] = torch.randn(shared, heads, hw, generator=g)
        kw["shared_value"] = torch.randn(shared, heads, hw, generator=g)
    if current:
        kw["current_key"] = torch.randn(batch, heads, hw, generator=g)
        kw["current_value"] = torch.randn(batch, heads, hw, generator=g)
        kw["current_valid"] = torch.rand(batch, generator=g) > 0.2
    # round inputs to the kernel dtype so both sides see the same values
    rnd = lambda x: x.to(dtype).float()
    query, keys, values = rnd(query), rnd(keys), rnd(values)
    kw = {k: (rnd(v) if v.is_floating_point() else v) for k, v in kw.items()}
    expected = oracle.paged_attention(query, keys, values, table, lengths, **kw)
    from graph_rewrite_system_b200.paged_attention import paged_attention

    dkw = {k: v.to(dev).to(dtype) if v.is_floating_point() else v.to(dev) for k, v in kw.items()}
    out = paged_attention(query.to(dev, dtype), keys.to(dev, dtype), values.to(dev, dtype),
                          table.to(dev), lengths.to(dev), **dkw)
    return out.float().cpu(), expected


@pytest.mark.parametrize("hw", [8, 32, 64])
def test_random_decode_with_current(cuda_device, hw):
    out, exp = _random_case(1, 37, 6, hw, 8, 40, 1, 70, torch.float32, cuda_device, current=True)
    np.testing.assert_allclose(out.numpy(), exp.numpy(), rtol=1e-5, atol=1e-5)


def test_readout_mma_bf16(cuda_device):
    # node readout shape: Q=381 queries per beam, T<=64, head width 32 -> tensor-core path
    out, exp = _random_case(2, 24, 8, 32, 16, 120, 381, 64, torch.bfloat16, cuda_device)
    np.testing.assert_allclose(out.numpy(), exp.numpy(), rtol=2e-2, atol=2e-2)
    assert not out[0].any()  # zero-length history row


@pytest.mark.parametrize("heads,max_len", [(3, 64), (16, 64), (16, 100)])
def test_readout_mma_head_counts_bf16(cuda_device, heads, max_len):
    # odd and the largest head counts of the tensor-core readout, one staged
    # tile (swizzled rows) and several (padded rows)
    out, exp = _random_case(5, 11, heads, 32, 16, 60, 40, max_len, torch.bfloat16, cuda_device)
    np.testing.assert_allclose(out.numpy(), exp.numpy(), rtol=2e-2, atol=2e-2)


def test_readout_mma_multi_tile_bf16(cuda_device):
    out, exp = _random_case(3, 9, 6, 32, 8, 90, 45, 150, torch.bfloat16, cuda_device)
    np.testing.assert_allclose(out.numpy(), exp.numpy(), rtol=2e-2, atol=2e-2)


def test_readout_fp32_rows(cuda_device):
    out, exp = _random_case(4, 7, 4, 32, 4, 30, 50, 20, torch.float32, cuda_device)
    np.testing.assert_allclose(out.numpy(), exp.numpy(), rtol=1e-5, atol=1e-5)


def test_shared_prefix_decode_bf16(cuda_device):
    out, exp = _random_case(5, 64, 8, 32, 16, 300, 1, 64, torch.bfloat16, cuda_device, shared=381)
    np.testing.assert_allclose(out.numpy(), exp.numpy(), rtol=2e-2, atol=2e-2)


def test_shared_prefix_decode_fp32(cuda_device):
    out, exp = _random_case(6, 16, 8, 32, 16, 64, 1, 64, torch.float32, cuda_device, shared=37)
    np.testing.assert_allclose(out.numpy(), exp.numpy(), rtol=1e-5, atol=1e-5)


def test_partial_current_triple_rejected(cuda_device):
    from graph_rewrite_system_b200.paged_attention import paged_attention

    q = torch.zeros(1, 1, 1, 32, device=cuda_device)
    kc = torch.zeros(1, 4, 1, 32, device=cuda_device)
    with pytest.raises(ValueError):
        paged_attention(q, kc, kc, torch.zeros(1, 1, dtype=torch.int32, device=cuda_device),
                        torch.zeros(1, dtype=torch.int32, device=cuda_device),
                        current_key=torch.zeros(1, 1, 32, device=cuda_device))


@pytest.mark.parametrize("batch,shared,current", [(37, 381, False), (16, 381, True),
                                                  (5, 17, True), (48, 0, False),
                                                  (40, 700, True)])
def test_shared_decode_shared_prefix(cuda_device, batch, shared, current):
    """The shared-prefix decode vs the oracle (700 shared keys: two staged
    chunks of the prefix per CTA)."""
    from graph_rewrite_system_b200.paged_attention import check_decode_status

    out, exp = _random_case(7 + batch, batch, 8, 32, 16, 200, 1, 64, torch.bfloat16, cuda_device,
                            shared=shared, current=current)
    np.testing.assert_allclose(out.numpy(), exp.numpy(), rtol=2e-2, atol=2e-2)
    check_decode_status(cuda_device)


@pytest.mark.parametrize("batch,heads,cap,max_len,page", [(40, 6, 6, 64, 16), (33, 8, 3, 96, 32),
                                                          (24, 5, 9, 61, 16), (70, 8, 400, 64, 16),
                                                          (33, 8, 3, 50, 8), (16, 4, 12, 17, 4)])
def test_shared_decode_shared_pages(cuda_device, batch, heads, cap, max_len, page):
    """Heavily shared pages (small arenas) exercise the per-column page dedup
    of the shared-prefix decode; ragged lengths, odd head counts (the general
    kernel), pages of 32 rows, partial beam groups and near-private pages (a
    400-page arena: several staging rounds per CTA) included (page sizes 8
    and 4 take the rows kernel)."""
    from graph_rewrite_system_b200.paged_attention import check_decode_status

    out, exp = _random_case(100 + batch, batch, heads, 32, page, cap, 1, max_len, torch.bfloat16,
                            cuda_device, shared=50, current=True)
    np.testing.assert_allclose(out.numpy(), exp.numpy(), rtol=2e-2, atol=2e-2)
    check_decode_status(cuda_device)


def test_shared_decode_prefix_tree(cuda_device):
    """The decode microbenchmark's own prefix-tree tables at a small size."""
    from graph_rewrite_system_b200.paged_attention import paged_attention
    from graph_rewrite_system_b200.workloads import decode_attention_workload

    w = decode_attention_workload(cuda_device, beams=48, num_shared=381, seed=5)
    got = paged_attention(w.query, w.key_cache, w.value_cache, w.block_table, w.lengths,
                          shared_key=w.shared_key, shared_value=w.shared_value)
    f = lambda t: t.float().cpu()
    exp = oracle.paged_attention(f(w.query), f(w.key_cache), f(w.value_cache),
                                 w.block_table.cpu(), w.lengths.cpu(), shared_key=f(w.shared_key),
                                 shared_value=f(w.shared_value))
    np.testing.assert_allclose(got.float().cpu().numpy(), exp.numpy(), rtol=2e-2, atol=2e-2)


@pytest.mark.parametrize("entry", ["grs_decode_attention_shared",
                                   "grs_decode_attention_shared_cluster"])
@pytest.mark.parametrize("beams,current", [(40, False), (512, True)])
def test_shared_decode_entry_points(cuda_device, entry, beams, current):
    """Both shared-prefix decode kernels, called through the C ABI on the
    decode microbenchmark's prefix-tree layout, accept it (a non-zero return
    would mean the rows-kernel fallback) and match the oracle."""
    from graph_rewrite_system_b200 import _lib
    from graph_rewrite_system_b200.paged_attention import check_decode_status
    from graph_rewrite_system_b200.workloads import decode_attention_workload

    w = decode_attention_workload(cuda_device, beams=beams, num_shared=381, seed=9 + beams)
    out = torch.empty_like(w.query)
    status = torch.zeros(1, dtype=torch.int32, device=cuda_device)
    q, kc = w.query, w.key_cache
    g = torch.Generator().manual_seed(beams)
    ck = cv = valid = None
    if current:
        ck = torch.randn(beams, q.shape[1], 32, generator=g).to(cuda_device, q.dtype)
        cv = torch.randn(beams, q.shape[1], 32, generator=g).to(cuda_device, q.dtype)
        valid = (torch.rand(beams, generator=g) > 0.3).to(cuda_device)
    rc = getattr(_lib.lib(), entry)(
        q.data_ptr(), q.stride(0), q.stride(1), kc.data_ptr(), w.value_cache.data_ptr(),
        kc.stride(0), kc.stride(1), kc.stride(2), w.block_table.data_ptr(),
        w.block_table.stride(0), w.block_table.shape[1], w.lengths.data_ptr(), kc.shape[0],
        _lib.ptr(ck), _lib.ptr(cv), ck.stride(0) if current else 0,
        ck.stride(1) if current else 0, _lib.ptr(valid), w.shared_key.data_ptr(),
        w.shared_value.data_ptr(), w.shared_key.shape[0], out.data_ptr(), out.stride(0),
        out.stride(1), q.shape[0], q.shape[1], kc.shape[1], status.data_ptr(),
        torch.cuda.current_stream().cuda_stream)
    assert rc == 0
    assert int(status.item()) == 0
    f = lambda t: t.float().cpu()
    kw = {}
    if current:
        kw = dict(current_key=f(ck), current_value=f(cv), current_valid=valid.cpu())
    exp = oracle.paged_attention(f(w.query), f(w.key_cache), f(w.value_cache),
                                 w.block_table.cpu(), w.lengths.cpu(), shared_key=f(w.shared_key),
                                 shared_value=f(w.shared_value), **kw)
    np.testing.assert_allclose(out.float().cpu().numpy(), exp.numpy(), rtol=2e-2, atol=2e-2)
    check_decode_status(cuda_device)


@pytest.mark.parametrize("batch,heads,page,cap,max_len,current", [
    (1000, 8, 16, 300, 63, True), (37, 6, 8, 90, 64, True), (21, 16, 4, 200, 150, True),
    (33, 8, 16, 100, 129, False), (5, 1, 16, 10, 16, True), (64, 8, 16, 64, 1, True)])
def test_causal_decode_bf16(cuda_device, batch, heads, page, cap, max_len, current):
    """One query per (beam, head) with the current token: the page-staged
    causal decode kernel (lengths 0, chunk-sized, multi-chunk)."""
    out, exp = _random_case(11 + batch, batch, heads, 32, page, cap, 1, max_len, torch.bfloat16,
                            cuda_device, current=current)
    np.testing.assert_allclose(out.numpy(), exp.numpy(), rtol=2e-2, atol=2e-2)


def _causal_abi(dev, q, kc, vc, table, lengths, ck, cv, valid, out, status):
    from graph_rewrite_system_b200 import _lib

    return _lib.lib().grs_decode_causal(
        q.data_ptr(), q.stride(0), q.stride(1), kc.data_ptr(), vc.data_ptr(), kc.stride(0),
        kc.stride(1), kc.stride(2), table.data_ptr(), table.stride(0), lengths.data_ptr(),
        kc.shape[0], ck.data_ptr(), cv.data_ptr(), ck.stride(0), ck.stride(1), valid.data_ptr(),
        out.data_ptr(), out.stride(0), out.stride(1), q.shape[0], q.shape[1], kc.shape[1],
        status.data_ptr(), torch.cuda.current_stream().cuda_stream)


def test_causal_decode_takes_the_kernel_and_flags_bad_pages(cuda_device):
    """The rollout's layout (8 heads x 32, page 16, query and current rows
    strided inside a QKV buffer) is accepted by grs_decode_causal itself; a
    page id outside the arena sets GRS_ERR_BAD_PAGE and its tokens are
    skipped, leaving the other beams exact."""
    dev = cuda_device
    g = torch.Generator().manual_seed(5)
    b, h, page, cap = 64, 8, 16, 40
    qkv = torch.randn(b, 3, h, 32, generator=g).bfloat16()
    kc = torch.randn(cap, page, h, 32, generator=g).bfloat16()
    vc = torch.randn(cap, page, h, 32, generator=g).bfloat16()
    table = torch.randint(0, cap, (b, 4), generator=g, dtype=torch.int32)
    lengths = torch.randint(0, 64, (b,), generator=g, dtype=torch.int32)
    valid = torch.rand(b, generator=g) > 0.1
    q, k, v = qkv.unbind(1)
    exp = oracle.paged_attention(q.float().unsqueeze(2), kc.float(), vc.float(), table, lengths,
                                 current_key=k.float(), current_value=v.float(),
                                 current_valid=valid).squeeze(2)
    qkv_d = qkv.to(dev)
    qd, kd, vd = qkv_d.unbind(1)
    out = torch.empty(b, h, 32, device=dev, dtype=torch.bfloat16)
    status = torch.zeros(1, dtype=torch.int32, device=dev)
    rc = _causal_abi(dev, qd, kc.to(dev), vc.to(dev), table.to(dev), lengths.to(dev), kd, vd,
                     valid.to(dev), out, status)
    assert rc == 0
    torch.cuda.synchronize()
    assert int(status.item()) == 0
    np.testing.assert_allclose(out.float().cpu().numpy(), exp.numpy(), rtol=2e-2, atol=2e-2)
    # beam 3 points one used page at an id past the arena
    lengths[3] = 40
    table[3, 1] = cap + 7
    good = torch.ones(b, dtype=torch.bool)
    good[3] = False
    rc = _causal_abi(dev, qd, kc.to(dev), vc.to(dev), table.to(dev), lengths.to(dev), kd, vd,
                     valid.to(dev), out, status)
    assert rc == 0
    torch.cuda.synchronize()
    assert int(status.item()) == -2                     # GRS_ERR_BAD_PAGE
    np.testing.assert_allclose(out.float().cpu().numpy()[good.numpy()],
                               exp.numpy()[good.numpy()], rtol=2e-2, atol=2e-2)
    assert torch.isfinite(out.float()).all()

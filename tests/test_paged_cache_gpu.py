"""Device PagedKVCache vs the reference's recorded churn (bit-exact state)."""
from __future__ import annotations

import numpy as np
import pytest
import torch

from conftest import load_golden
from test_oracle_golden import replay_churn

pytestmark = pytest.mark.gpu


class _DeviceAdapter:
    """Feeds host tensors to the device cache so replay_churn can drive it."""

    def __init__(self, cache, device):
        self.cache, self.device = cache, device

    def empty_handle(self):
        return self.cache.empty_handle()

    def append_batch(self, parents, *tensors):
        return self.cache.append_batch(parents, *[t.to(self.device) for t in tensors])

    def release(self, h):
        self.cache.release(h)

    def __getattr__(self, name):
        return getattr(self.cache, name)


@pytest.mark.parametrize("name", ["paged_cache_churn_p4.npz", "paged_cache_churn_p3.npz"])
def test_churn_bit_exact(cuda_device, name):
    from graph_rewrite_system_b200.paged_cache import PagedKVCache

    g = load_golden(name)

    def make(g):
        return _DeviceAdapter(PagedKVCache(
            layers=int(g["layers"]), capacity=int(g["capacity"]), page_size=int(g["page"]),
            heads=int(g["heads"]), head_width=int(g["hw"]), model_width=int(g["width"]),
            device=cuda_device, dtype=torch.float32), cuda_device)

    def check(step, cache, handles):
        table = g[f"s{step}_table"]
        for i, h in enumerate(handles):
            assert list(h.blocks) == [int(p) for p in table[i, : len(h.blocks)]]
        assert [h.length for h in handles] == g[f"s{step}_lengths"].tolist()
        assert cache.refcounts == g[f"s{step}_refcounts"].tolist()
        assert cache.free == g[f"s{step}_free"].tolist()
        _, values, actions, _ = cache.gather(handles)
        np.testing.assert_array_equal(values.cpu().numpy(), g[f"s{step}_gather_values"])
        np.testing.assert_array_equal(actions.cpu().numpy(), g[f"s{step}_gather_actions"])

    cache = replay_churn(g, make, check)
    assert cache.allocated_pages == 0


def test_exhaustion_and_refcount_errors(cuda_device):
    from graph_rewrite_system_b200.paged_cache import PagedKVCache, PrefixHandle

    cache = PagedKVCache(layers=1, capacity=2, page_size=2, heads=1, head_width=2, model_width=2,
                         device=cuda_device, dtype=torch.float32)
    root = cache.empty_handle()
    kv = torch.zeros(1, 3, 1, 2, device=cuda_device)
    with pytest.raises(RuntimeError, match="exhausted"):
        cache.append_batch([root] * 3, kv, kv, torch.zeros(3, 2, device=cuda_device))
    cache2 = PagedKVCache(layers=1, capacity=4, page_size=2, heads=1, head_width=2, model_width=2,
                          device=cuda_device, dtype=torch.float32)
    with pytest.raises(RuntimeError, match="negative page reference count"):
        cache2.release(PrefixHandle((1,), 1))
    with pytest.raises(RuntimeError, match="mismatch"):
        cache2.block_table([PrefixHandle((1, 2), 1)])


@pytest.mark.parametrize("beams,depth,checked", [(64, 40, 8), (1000, 64, 40)])
def test_bf16_churn_matches_oracle(cuda_device, beams, depth, checked):
    """Cache churn with bf16 arenas through the device-native API, bit-exact
    against the oracle: each step forks every beam into 5 children with
    seeded uniform scores, keeps the top `beams` (stable, ties by index),
    appends one token per survivor in all arenas (COW on partial tail pages)
    and releases the old handles (refcount reclaim).  The second case is the
    full churn workload: 1000 beams, 4 layers x 8 heads x 32, page 16, depth
    64.  Block tables, refcounts and the free list are compared in full, arena
    rows at every valid position of `checked` handles spread over the beam."""
    from graph_rewrite_system_b200.paged_cache import PagedKVCache
    from oracle.paged_cache import OraclePagedKVCache

    layers, heads, hw, width, page = 4, 8, 32, 256, 16
    cap = beams * (-(-depth // page) + 3)
    dev = PagedKVCache(layers=layers, capacity=cap, page_size=page, heads=heads, head_width=hw,
                       model_width=width, device=cuda_device, dtype=torch.bfloat16)
    ref = OraclePagedKVCache(layers=layers, capacity=cap, page_size=page, heads=heads,
                             head_width=hw, model_width=width, dtype=torch.bfloat16)
    gen = torch.Generator().manual_seed(0)
    handles = [ref.empty_handle()]
    table = torch.zeros(1, 1, dtype=torch.int32, device=cuda_device)
    lengths = torch.zeros(1, dtype=torch.int32, device=cuda_device)
    for step in range(depth):
        scores = torch.rand(len(handles) * 5, generator=gen)
        parents = (torch.sort(scores, descending=True, stable=True).indices[:beams] // 5)
        n = parents.numel()
        kv = torch.randn(layers, n, heads, hw, generator=gen).bfloat16()
        act = torch.randn(n, width, generator=gen).bfloat16()
        rk = torch.randn(n, heads, hw, generator=gen).bfloat16()
        new = ref.append_batch([handles[p] for p in parents.tolist()], kv, kv, act, rk, rk)
        for h in handles:
            ref.release(h)
        handles = new
        pidx = parents.to(cuda_device)
        ct, cl = dev.append_device(table[pidx], lengths[pidx], kv.to(cuda_device),
                                   kv.to(cuda_device), act.to(cuda_device), rk.to(cuda_device),
                                   rk.to(cuda_device))
        dev.release_device(table, lengths)
        table, lengths = ct, cl
    dev.check_status()
    assert dev.refcounts == ref.refcounts
    assert dev.free == ref.free
    rows = table.cpu()
    for i, h in enumerate(handles):
        assert rows[i, : len(h.blocks)].tolist() == list(h.blocks)
    assert dev.allocated_pages == ref.allocated_pages
    assert cl.tolist() == [h.length for h in handles]
    # arena contents at every valid token position
    stride = max(1, len(handles) // checked)
    for h in handles[::stride][:checked]:
        for pos in range(h.length):
            p, r = h.blocks[pos // page], pos % page
            assert torch.equal(dev.keys[:, p, r].cpu(), ref.keys[:, p, r])
            assert torch.equal(dev.actions[p, r].cpu(), ref.actions[p, r])
            assert torch.equal(dev.readout_values[p, r].cpu(), ref.readout_values[p, r])

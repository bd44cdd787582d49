"""The sharded search's record kernels (grs_shard_records / grs_shard_merge /
grs_shard_route) against the oracle restatement, bit-exact, on seeded inputs
with ties, empty lists, padding and the size limits."""
from __future__ import annotations

import numpy as np
import pytest
import torch

from oracle import sharded as oracle

pytestmark = pytest.mark.gpu

DEV = torch.device("cuda", 0)


def _lib():
    from graph_rewrite_system_b200 import _lib

    return _lib


def _t(a, dtype=torch.int64):
    return torch.as_tensor(np.asarray(a), dtype=dtype, device=DEV)


def _stream():
    return torch.cuda.current_stream(DEV).cuda_stream


@pytest.mark.parametrize("parents,k,n,width,seed", [(6, 5, 20, 24, 0), (40, 16, 300, 300, 1),
                                                     (3, 2, 0, 8, 2), (50, 8, 200, 120, 3)])
def test_records_match_oracle(parents, k, n, width, seed):
    lib = _lib()
    rng = np.random.default_rng(seed)
    tw = lib.lib().grs_topology_table_width()
    xfers_total = 30
    table = rng.integers(0, 5, size=(xfers_total, tw)).astype(np.int32)
    cand_batch = np.repeat(np.arange(parents), k)
    probs = (rng.integers(0, 6, size=parents * k) / 6.0).astype(np.float32)
    rows = rng.integers(0, parents * k, size=max(n, 1))[:n]
    xfers = rng.integers(0, xfers_total, size=n)
    next_gate = rng.integers(10, 4000, size=n)
    gate = rng.integers(0, 4095, size=parents)
    global_index = rng.integers(0, 1 << 23, size=parents)
    next_slot = rng.integers(0, 500, size=parents).astype(np.int32)
    valid = rng.integers(0, 2, size=n).astype(np.uint8)
    fp = rng.integers(-(1 << 62), 1 << 62, size=n)
    metrics = rng.integers(0, 1000, size=2)
    capacity, free = 5000, 1234
    gcap = max(n, width) + 7                       # ranked arrays are global_cap long
    pad = lambda a, dt: np.concatenate([np.asarray(a, dt), np.zeros(gcap - len(a), dt)])
    out = torch.empty(4 * width + 4, dtype=torch.int64, device=DEV)
    status = torch.zeros(1, dtype=torch.int32, device=DEV)
    args = [_t([n]), _t(pad(rows, np.int64)), _t(pad(xfers, np.int64)),
            _t(pad(next_gate, np.int64)), _t(probs, torch.float32), _t(cand_batch), None,
            _t(gate), _t(global_index), _t(next_slot, torch.int32), _t(table, torch.int32),
            _t(pad(valid, np.uint8), torch.uint8), _t(pad(fp, np.int64)), _t(metrics),
            _t([free], torch.int32)]
    ptr = [a.data_ptr() if a is not None else None for a in args]
    ptr[6] = k
    lib.check(lib.lib().grs_shard_records(width, *ptr, capacity, out.data_ptr(),
                                          status.data_ptr(), _stream()))
    torch.cuda.synchronize()
    assert int(status.item()) == 0
    expected = oracle.pack_records(width, n, rows, xfers, next_gate, probs, cand_batch, k, gate,
                                   global_index, next_slot, table[:, 1], valid, fp,
                                   [n, metrics[0], metrics[1], capacity - free])
    np.testing.assert_array_equal(out.cpu().numpy(), expected)


def test_records_empty_gpu_block():
    lib = _lib()
    width = 16
    out = torch.full((4 * width + 4,), 7, dtype=torch.int64, device=DEV)
    zero = torch.zeros(1, dtype=torch.int64, device=DEV)
    free = torch.tensor([40], dtype=torch.int32, device=DEV)
    lib.check(lib.lib().grs_shard_records(width, zero.data_ptr(), None, None, None, None, None, 1,
                                          None, None, None, None, None, None, None,
                                          free.data_ptr(), 100, out.data_ptr(), None,
                                          _stream()))
    got = out.cpu().numpy()
    assert (got[:width] == oracle.ABSENT).all() and (got[width:4 * width] == 0).all()
    assert got[4 * width:].tolist() == [0, 0, 0, 60]


def _sorted_blocks(rng, world, width, present, tie_keys=False):
    """Per-GPU record blocks, each sorted by (KEY1, KEY2), unique keys overall."""
    total = sum(present)
    key1 = rng.integers(0, 6 if tie_keys else 1 << 40, size=total) << 12
    key2 = rng.permutation(1 << 20)[:total]                  # unique
    blocks, at = [], 0
    for r in range(world):
        n = present[r]
        k1, k2 = key1[at:at + n], key2[at:at + n]
        at += n
        order = np.lexsort((k2, k1))
        b = np.zeros(4 * width + 4, np.int64)
        b[:width] = oracle.ABSENT
        b[:n] = k1[order]
        b[width:width + n] = k2[order]
        b[2 * width:2 * width + n] = rng.integers(-(1 << 62), 1 << 62, size=n)
        b[3 * width:3 * width + n] = rng.integers(0, 600, size=n) | (
            rng.integers(0, 2, size=n) << 32)
        b[4 * width:] = rng.integers(0, 100, size=4)
        blocks.append(b)
    return blocks


def _merge(blocks, width, cap):
    lib = _lib()
    world = len(blocks)
    gathered = _t(np.stack(blocks))
    count = torch.empty(1, dtype=torch.int64, device=DEV)
    metrics = torch.empty(4, dtype=torch.int64, device=DEV)
    valid = torch.empty(cap, dtype=torch.uint8, device=DEV)
    arrays = [torch.empty(cap, dtype=torch.int64, device=DEV) for _ in range(5)]
    status = torch.zeros(1, dtype=torch.int32, device=DEV)
    lib.check(lib.lib().grs_shard_merge(
        gathered.data_ptr(), world, width, gathered.shape[1], cap, count.data_ptr(),
        metrics.data_ptr(), valid.data_ptr(), *(a.data_ptr() for a in arrays),
        status.data_ptr(), _stream()))
    torch.cuda.synchronize()
    got = dict(zip(("fp", "next_gate", "src", "index", "child_next"),
                   (a.cpu().numpy() for a in arrays)))
    got["valid"] = valid.cpu().numpy()
    return got, int(count.item()), metrics.cpu().numpy(), int(status.item())


@pytest.mark.parametrize("world,width,present,cap,ties,seed", [
    (2, 50, [50, 31], 100, False, 0), (4, 300, [300, 0, 120, 299], 600, True, 1),
    (8, 64, [64, 64, 0, 1, 17, 64, 3, 40], 512, True, 2), (3, 10, [0, 0, 0], 30, False, 3),
    (5, 2000, [2000, 1500, 1999, 7, 2000], 4000, True, 4), (1, 40, [33], 40, False, 5)])
def test_merge_matches_oracle(world, width, present, cap, ties, seed):
    rng = np.random.default_rng(seed)
    blocks = _sorted_blocks(rng, world, width, present, ties)
    got, count, metrics, status = _merge(blocks, width, cap)
    assert status == 0
    expected, e_count, e_metrics = oracle.merge_records(blocks, width, cap)
    assert count == e_count
    np.testing.assert_array_equal(metrics, e_metrics)
    for name, value in expected.items():
        np.testing.assert_array_equal(got[name], value, err_msg=name)


def test_merge_flags_unsorted_block():
    rng = np.random.default_rng(7)
    blocks = _sorted_blocks(rng, 2, 20, [20, 12])
    blocks[1][[3, 4]] = blocks[1][[4, 3]]                   # swap two KEY1s
    blocks[1][[23, 24]] = blocks[1][[24, 23]]
    _, _, _, status = _merge(blocks, 20, 40)
    assert status == -11


def _route(merged, child_proposal, accepted, world, me, beam):
    lib = _lib()
    cap = len(merged["src"])
    summary = _t([accepted, 0, 0, 0, 0, 0])
    cp = torch.zeros(beam, dtype=torch.int64, device=DEV)
    cp[:len(child_proposal)] = _t(child_proposal)
    pairs = torch.empty(world * world, dtype=torch.int64, device=DEV)
    extent = torch.empty(1, dtype=torch.int64, device=DEV)
    lists = [torch.full((beam,), -1, dtype=torch.int64, device=DEV) for _ in range(4)]
    status = torch.zeros(1, dtype=torch.int32, device=DEV)
    src, index, cn = _t(merged["src"]), _t(merged["index"]), _t(merged["child_next"])
    lib.check(lib.lib().grs_shard_route(
        cp.data_ptr(), summary.data_ptr(), src.data_ptr(), index.data_ptr(), cn.data_ptr(), cap,
        beam, world, me, pairs.data_ptr(), extent.data_ptr(), *(x.data_ptr() for x in lists),
        status.data_ptr(), _stream()))
    torch.cuda.synchronize()
    return pairs.cpu().numpy().reshape(world, world), int(extent.item()), [
        x.cpu().numpy() for x in lists], int(status.item())


@pytest.mark.parametrize("world,accepted,beam,skew,seed", [
    (2, 12, 12, 0.5, 0), (4, 4000, 4000, 0.3, 1), (8, 8000, 8000, 0.05, 2),
    (3, 1000, 1024, 0.6, 3), (8, 8192, 8192, 0.9, 4), (1, 500, 500, 0.0, 5),
    (5, 3, 10, 0.5, 6), (64, 4096, 4096, 0.2, 7)])
def test_route_matches_oracle(world, accepted, beam, skew, seed):
    rng = np.random.default_rng(seed)
    cap = accepted * 3 + 5
    # children concentrated on a few GPUs (skew) so that many overflow
    weights = np.exp(-skew * np.arange(world))
    src = rng.choice(world, size=cap, p=weights / weights.sum())
    merged = {"src": src, "index": rng.integers(0, 1 << 20, size=cap),
              "child_next": rng.integers(0, 900, size=cap)}
    child_proposal = rng.permutation(cap)[:accepted]
    for me in sorted({0, world - 1, world // 2}):
        pairs, extent, lists, status = _route(merged, child_proposal, accepted, world, me, beam)
        assert status == 0
        expected = oracle.route(child_proposal, accepted, merged, world, me)
        np.testing.assert_array_equal(pairs, expected["pairs"])
        assert extent == expected["extent"]
        n_keep, n_out = pairs[me, me], pairs[me].sum() - pairs[me, me]
        n_in = pairs[:, me].sum() - pairs[me, me]
        for got, name, n in zip(lists, ("keep_local", "keep_global", "out_local", "in_global"),
                                (n_keep, n_keep, n_out, n_in)):
            np.testing.assert_array_equal(got[:n], expected[name], err_msg=name)


@pytest.mark.parametrize("seed,n,n_dev", [(0, 7, None), (1, 40, 13), (2, 300, 300), (3, 5, 0)])
def test_rows_copy_matches_numpy(seed, n, n_dev):
    """Gather (indexed source), scatter (indexed destination) and multi-unit
    segments with 1-, 4-, 8- and 16-byte aligned rows."""
    from graph_rewrite_system_b200 import kernels as K

    rng = np.random.default_rng(seed)
    src_rows = n + 11
    a = rng.integers(0, 255, size=(src_rows, 37), dtype=np.uint8)       # odd row bytes
    b = rng.integers(-1000, 1000, size=(src_rows, 6), dtype=np.int32)
    c = rng.integers(-(1 << 40), 1 << 40, size=(src_rows, 8))            # 64-byte rows
    pages = rng.standard_normal((50, 24)).astype(np.float32)            # 96-byte pages
    gather = rng.integers(0, src_rows, size=n)
    page_ids = rng.choice(50, size=(n, 2), replace=False) if n * 2 <= 50 else \
        rng.integers(0, 50, size=(n, 2))
    layout = [(0, 37), (48, 24), (80, 64), (144, 192)]                  # packed row offsets
    row = 336
    ta, tb, tc, tp = _t(a, torch.uint8), _t(b, torch.int32), _t(c), _t(pages, torch.float32)
    ti, tpi = _t(gather), _t(page_ids.reshape(-1))
    packed = torch.zeros(n, row, dtype=torch.uint8, device=DEV)
    flat = packed.view(-1)
    count = None if n_dev is None else _t([n_dev])
    K.rows_copy([(ta, 0, 37, ti, flat[0:], row, 0, None, 37, 1),
                 (tb, 0, 24, ti, flat[48:], row, 0, None, 24, 1),
                 (tc, 0, 64, ti, flat[80:], row, 0, None, 64, 1),
                 (tp, 0, 96, tpi, flat[144:], row, 96, None, 96, 2)], n, count)
    rows = n if n_dev is None else min(n, n_dev)
    expected = np.zeros((n, row), np.uint8)
    for i in range(rows):
        g = gather[i]
        expected[i, 0:37] = a[g]
        expected[i, 48:72] = b[g].view(np.uint8)
        expected[i, 80:144] = c[g].view(np.uint8)
        expected[i, 144:336] = pages[page_ids[i]].reshape(-1).view(np.uint8)
    np.testing.assert_array_equal(packed.cpu().numpy(), expected)
    # scatter the packed pages back into a fresh arena at new page ids
    arena = torch.zeros(60, 24, dtype=torch.float32, device=DEV)
    targets = rng.choice(60, size=rows * 2, replace=False) if rows * 2 <= 60 else None
    if targets is not None and rows:
        K.rows_copy([(flat[144:], row, 96, None, arena, 0, 96, _t(targets), 96, 2)], rows)
        got = arena.cpu().numpy()
        for i in range(rows):
            for k in range(2):
                np.testing.assert_array_equal(got[targets[i * 2 + k]], pages[page_ids[i, k]])

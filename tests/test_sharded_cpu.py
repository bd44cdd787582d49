"""Host logic of the sharded beam search on CPU (gloo, world size 2).

The merged ranking of the per-rank ranked records must equal the single-GPU
ranking (the oracle's ``rank_proposals`` over the union of candidates, which
restates gpu_proposals.py) bit-exactly, ties included; the child placement
must keep every rank within its quota and move as few children as possible.
"""
from __future__ import annotations

import multiprocessing as mp
import os
import socket

import numpy as np
import pytest
import torch

from oracle import proposals as oracle


def _candidates(seed: int, parents: int, k: int, num_sources: int):
    rng = np.random.default_rng(seed)
    sources = rng.integers(0, num_sources, size=(parents, k))
    # quantised probabilities and few gate deltas: plenty of exact ties
    probs = (rng.integers(0, 8, size=(parents, k)) / 8.0).astype(np.float32)
    gates = rng.integers(20, 24, size=parents)
    return sources, probs, gates


def _rule_index(num_sources: int, seed: int):
    rng = np.random.default_rng(seed + 1)
    source_to_xfers = {s: sorted(rng.choice(40, size=rng.integers(1, 5), replace=False).tolist())
                       for s in range(num_sources)}
    deltas = rng.integers(-2, 2, size=40)
    return oracle.build_rule_index(source_to_xfers, deltas, num_sources, max_gate_increase=1)


def _local_records(rank, world, parents, k, cap, per_parent_cap, seed):
    from oracle import sharded

    sources, probs, gates = _candidates(seed, parents, k, 7)
    index = _rule_index(7, seed)
    mine = np.arange(parents)[rank::world]                  # this rank's parents (global ids)
    src = sources[mine].reshape(-1)
    pr = probs[mine].reshape(-1)
    local_batch = np.repeat(np.arange(len(mine)), k)
    sel, _ = oracle.rank_proposals(local_batch, src, np.zeros_like(src),
                                   np.zeros((src.size, 1), np.int64), pr, gates[mine], index,
                                   per_parent_cap=per_parent_cap, global_cap=cap)
    n = sel["parent"].size
    identity = mine[sel["parent"]] * 1000 + sel["xfer"]           # payload in the FP field
    return sharded.pack_records(
        cap, n, sel["candidate"], sel["xfer"], sel["next_gate"], pr, local_batch, k,
        gates[mine], mine, np.zeros(len(mine), np.int64), np.zeros(64, np.int64),
        np.ones(n, np.uint8), identity, [n, rank, 0, 0])


def _worker(rank, world, port, args, queue):
    import torch.distributed as dist

    from oracle import sharded

    dist.init_process_group("gloo", init_method=f"tcp://127.0.0.1:{port}", rank=rank,
                            world_size=world)
    try:
        block = torch.from_numpy(_local_records(rank, world, *args))
        out = torch.empty(world * block.numel(), dtype=torch.int64)
        dist.all_gather_into_tensor(out, block)
        merged, count, metrics = sharded.merge_records(list(out.view(world, -1).numpy()),
                                                       args[2], args[2])
        queue.put((rank, merged["fp"][:count].tolist(), metrics.tolist()))
    finally:
        dist.destroy_process_group()


def _free_port() -> int:
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


@pytest.mark.parametrize("parents,k,cap,per_parent_cap,seed", [(10, 6, 25, 3, 0),
                                                               (9, 5, 200, 4, 1),
                                                               (12, 8, 40, 16, 2)])
def test_merged_ranking_equals_single_gpu_ranking(parents, k, cap, per_parent_cap, seed):
    world = 2
    ctx = mp.get_context("spawn")
    queue = ctx.Queue()
    port = _free_port()
    args = (parents, k, cap, per_parent_cap, seed)
    procs = [ctx.Process(target=_worker, args=(r, world, port, args, queue)) for r in range(world)]
    for p in procs:
        p.start()
    results = {r: rest for r, *rest in (queue.get(timeout=120) for _ in range(world))}
    for p in procs:
        p.join(timeout=60)
        assert p.exitcode == 0
    assert results[0] == results[1]                      # every rank merges identically
    assert results[0][1][1] == sum(range(world))         # metrics summed over ranks
    # the single-GPU ranking of the union
    sources, probs, gates = _candidates(seed, parents, k, 7)
    index = _rule_index(7, seed)
    batch = np.repeat(np.arange(parents), k)
    sel, _ = oracle.rank_proposals(batch, sources.reshape(-1), np.zeros(parents * k, np.int64),
                                   np.zeros((parents * k, 1), np.int64), probs.reshape(-1),
                                   gates, index, per_parent_cap=per_parent_cap, global_cap=cap)
    expected = (sel["parent"] * 1000 + sel["xfer"]).tolist()
    assert results[0][0] == expected


@pytest.mark.parametrize("world,sources", [(2, [0, 0, 0, 1, 0, 0]), (4, [0] * 9),
                                           (3, [2, 1, 0, 2, 2, 2, 1, 0]), (2, [1, 0])])
def test_placement_keeps_quota_and_minimises_moves(world, sources):
    from oracle import sharded

    a = len(sources)
    merged = {"src": np.asarray(sources), "index": np.arange(a) + 100,
              "child_next": np.arange(a) % 5}
    quota = [a // world + (r < a % world) for r in range(world)]
    lists = [sharded.route(np.arange(a), a, merged, world, me) for me in range(world)]
    pairs = lists[0]["pairs"]
    assert all((x["pairs"] == pairs).all() for x in lists)
    assert pairs.sum(0).tolist() == quota                # every rank ends at its share
    assert pairs.sum(1).tolist() == [sources.count(r) for r in range(world)]
    for r in range(world):
        own = [j for j, s in enumerate(sources) if s == r]
        assert lists[r]["keep_global"].tolist() == own[: min(len(own), quota[r])]
        assert lists[r]["keep_local"].tolist() == [100 + j for j in own[: quota[r]]]
        assert len(lists[r]["out_local"]) == max(0, len(own) - quota[r])
    # a child only moves when its own rank is over quota, and every moved
    # child is sent once and received once
    moves = pairs.sum() - np.trace(pairs)
    assert moves == sum(max(0, sources.count(r) - quota[r]) for r in range(world))
    sent = sorted(j - 100 for x in lists for j in x["out_local"])
    received = sorted(j for x in lists for j in x["in_global"])
    assert sent == received
    assert lists[0]["extent"] == max(j % 5 for j in range(a))

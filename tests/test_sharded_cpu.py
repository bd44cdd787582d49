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
    from graph_rewrite_system_b200.sharded import ABSENT, KEY1, NUM_FIELDS, pack_keys

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
    t = lambda a: torch.as_tensor(np.asarray(a, np.int64))
    key1, key2 = pack_keys(t(sel["next_gate"]), torch.as_tensor(sel["probability"]),
                           t(gates[mine][sel["parent"]]), t(mine[sel["parent"]]),
                           t(sel["xfer"]), t(sel["candidate"] % k))
    rec = torch.zeros(cap, NUM_FIELDS, dtype=torch.int64)
    rec[:, KEY1] = ABSENT
    rec[:n, 0], rec[:n, 1] = key1, key2
    rec[:n, 3] = t(mine[sel["parent"]] * 1000 + sel["xfer"])      # payload: identity
    rec[:n, 5] = rank
    rec[:n, 6] = torch.arange(n)
    return rec


def _worker(rank, world, port, args, queue):
    import torch.distributed as dist

    from graph_rewrite_system_b200.sharded import merge_records

    dist.init_process_group("gloo", init_method=f"tcp://127.0.0.1:{port}", rank=rank,
                            world_size=world)
    try:
        rec = _local_records(rank, world, *args)
        out = [torch.empty_like(rec) for _ in range(world)]
        dist.all_gather(out, rec)
        merged, count = merge_records(torch.cat(out), args[2])
        queue.put((rank, merged[: int(count)].tolist()))
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
    results = dict(queue.get(timeout=120) for _ in range(world))
    for p in procs:
        p.join(timeout=60)
        assert p.exitcode == 0
    assert results[0] == results[1]                      # every rank merges identically
    # the single-GPU ranking of the union
    sources, probs, gates = _candidates(seed, parents, k, 7)
    index = _rule_index(7, seed)
    batch = np.repeat(np.arange(parents), k)
    sel, _ = oracle.rank_proposals(batch, sources.reshape(-1), np.zeros(parents * k, np.int64),
                                   np.zeros((parents * k, 1), np.int64), probs.reshape(-1),
                                   gates, index, per_parent_cap=per_parent_cap, global_cap=cap)
    expected = (sel["parent"] * 1000 + sel["xfer"]).tolist()
    got = [row[3] for row in results[0]]
    assert got == expected


@pytest.mark.parametrize("world,sources", [(2, [0, 0, 0, 1, 0, 0]), (4, [0] * 9),
                                           (3, [2, 1, 0, 2, 2, 2, 1, 0]), (2, [1, 0])])
def test_placement_keeps_quota_and_minimises_moves(world, sources):
    from graph_rewrite_system_b200.sharded import placement

    src = torch.tensor(sources)
    dest, pairs = placement(src, world)
    a = len(sources)
    quota = [a // world + (r < a % world) for r in range(world)]
    assert torch.bincount(dest, minlength=world).tolist() == quota
    assert pairs.sum().item() == a
    for r in range(world):
        own = [j for j, s in enumerate(sources) if s == r]
        kept = [j for j in own if dest[j] == r]
        assert kept == own[: min(len(own), quota[r])]    # first children stay, in order
    # a child only moves when its own rank is over quota
    assert int((dest != src).sum()) == sum(max(0, sources.count(r) - quota[r])
                                           for r in range(world))

"""Sharded beam search over 1, 2 and 4 GPUs (NCCL, one process per GPU)
against the single-GPU search with the same global beam, fp32: the
per-level decisions (accepted / attempted / invalid / duplicate counts,
proposals, best gate) and the final global fingerprints must match, the beam
must stay evenly split, and every rank's cache must hand back all pages.
Cases that need more GPUs than present are skipped."""
from __future__ import annotations

import multiprocessing as mp
import socket

import pytest
import torch

pytestmark = pytest.mark.gpu

SMALL = dict(width=64, retrieval_width=32, graph_layers=1, action_layers=2, action_heads=2,
             max_sequence_length=64, readout_graph_layers=2)
FIELDS = ("input_states", "output_states", "best_speculative_gate_count", "predicted_actions",
          "eligible_actions_before_parent_cap", "proposals_after_caps", "attempted_actions",
          "accepted_actions", "invalid_structural_actions", "duplicate_speculative_successors")


def _search_parts(dev, seed, beam, depth):
    from graph_rewrite_system_b200 import synthetic
    from test_paged_model_gpu import build_model

    cfg = synthetic.ModelConfig(**SMALL)
    rules = synthetic.synthetic_rules()
    model = build_model(dev, torch.float32, rules, cfg, seed)
    circuit = synthetic.random_circuit(4, 30, seed + 1)
    rc = synthetic.RolloutConfig(beam_size=beam, depth=depth, page_size=4,
                                 max_candidates_per_state=400, per_parent_cap=4,
                                 proposal_factor=4)
    return model, rules, circuit, rc


def _worker(rank, world, port, seed, beam, depth, queue):
    import os
    import sys

    import torch.distributed as dist

    sys.path.insert(0, os.path.dirname(os.path.abspath(__file__)))
    sys.path.insert(0, os.path.dirname(os.path.dirname(os.path.abspath(__file__))))

    dev = torch.device("cuda", rank)
    torch.cuda.set_device(dev)
    import datetime

    dist.init_process_group("nccl", init_method=f"tcp://127.0.0.1:{port}", rank=rank,
                            world_size=world, device_id=dev,
                            timeout=datetime.timedelta(seconds=60))
    try:
        _run_worker(rank, dev, seed, beam, depth, queue)
    except Exception:
        import traceback

        queue.put((rank, "error", traceback.format_exc(), None))
        raise
    finally:
        dist.destroy_process_group()


def _run_worker(rank, dev, seed, beam, depth, queue):
    from graph_rewrite_system_b200.sharded import ShardedBeamSearch

    model, rules, circuit, rc = _search_parts(dev, seed, beam, depth)
    search = ShardedBeamSearch(model, rules, circuit, rc, dev)
    search.reset()
    rows = []
    for _ in range(depth):
        row = search.step()
        if row is None:
            break
        rows.append([getattr(row, f) for f in FIELDS] + [search.beams])
    search.check()
    fps = search.global_fingerprints()
    search.cache.release_device(search.block_table, search.lengths)
    search.cache.check_status()
    queue.put((rank, rows, fps, search.cache.allocated_pages))


def _free_port() -> int:
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


@pytest.mark.parametrize("world,seed", [(1, 3), (2, 3), (2, 4), (4, 5)])
def test_sharded_search_matches_single_gpu(world, seed):
    if torch.cuda.device_count() < world:
        pytest.skip(f"needs {world} GPUs")
    from graph_rewrite_system_b200.rollout import DeviceBeamSearch

    beam, depth = 12, 5
    ctx = mp.get_context("spawn")
    queue = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=_worker, args=(r, world, port, seed, beam, depth, queue))
             for r in range(world)]
    for p in procs:
        p.start()
    results = {}
    for _ in range(world):
        r, *rest = queue.get(timeout=300)
        if rest[0] == "error":
            for p in procs:
                p.join(timeout=90)
            pytest.fail(f"rank {r} failed:\n{rest[1]}")
        results[r] = rest
    for p in procs:
        p.join(timeout=120)
        assert p.exitcode == 0
    rows0, fps0, _ = results[0]
    for r in range(world):
        assert [x[:-1] for x in results[r][0]] == [x[:-1] for x in rows0]  # same decisions
        assert results[r][1] == fps0
        assert results[r][2] == 0                                # every page came back
    # the beam is split evenly after every level
    for level, a in enumerate(rows0):
        held = [results[r][0][level][-1] for r in range(world)]
        assert max(held) - min(held) <= 1
        assert sum(held) == a[FIELDS.index("output_states")]
    # single GPU, same global beam
    dev = torch.device("cuda", 0)
    model, rules, circuit, rc = _search_parts(dev, seed, beam, depth)
    single = DeviceBeamSearch(model, rules, circuit, rc, dev)
    single.reset()
    expected = []
    for _ in range(depth):
        row = single.step()
        if row is None:
            break
        expected.append([getattr(row, f) for f in FIELDS])
    single.check()
    assert [r[:-1] for r in rows0] == expected
    assert fps0 == [int(x) & ((1 << 64) - 1) for x in single.topo.fingerprint.tolist()]

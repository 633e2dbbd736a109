"""Multi-process host logic on CPU (gloo, world size 2): request sharding is a
partition of the workload, balanced, identical on every rank; the end-of-run
reduction sums committed tokens and takes the max time."""
from __future__ import annotations

import os
import socket

import pytest
import torch.multiprocessing as mp


def _free_port() -> int:
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _worker(rank, world, port, out):
    import sys
    root = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
    sys.path.insert(0, os.path.join(root, "paged-speculative-engine_b200"))
    import datetime

    import torch.distributed as dist

    from pse import dist as pd
    from pse import workload as wl
    from pse.scheduler import Request

    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    dist.init_process_group("gloo", rank=rank, world_size=world, timeout=datetime.timedelta(seconds=60))
    w = wl.WORKLOADS["llama-1b"]
    prompts = wl.prompts(w, seed=0, n=64)
    reqs = [Request(f"r{i}", p, w.max_new_tokens) for i, p in enumerate(prompts)]
    mine = pd.shard_requests(reqs, world, rank)
    tokens = sum(r.max_new_tokens for r in mine)
    total, secs, per = pd.reduce_stats(tokens, 1.0 + rank, extra={"ids": [r.request_id for r in mine]})
    out.put((rank, [r.request_id for r in mine], total, secs, per))
    dist.barrier()
    dist.destroy_process_group()


@pytest.mark.timeout(120)
def test_sharding_and_stats_reduce_two_ranks():
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=_worker, args=(r, 2, port, q)) for r in range(2)]
    for p in procs:
        p.start()
    got = [q.get(timeout=100) for _ in range(2)]
    for p in procs:
        p.join(timeout=60)
        assert p.exitcode == 0
    got.sort()
    ids0, ids1 = set(got[0][1]), set(got[1][1])
    assert not ids0 & ids1 and len(ids0 | ids1) == 64
    assert abs(len(ids0) - len(ids1)) <= 8
    for rank, _, total, secs, per in got:
        assert total == 64 * 512
        assert secs == 2.0
        assert [set(p[2]["ids"]) for p in per] == [ids0, ids1]


def test_lpt_sharding_balances_expected_tokens():
    import sys
    root = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
    sys.path.insert(0, os.path.join(root, "paged-speculative-engine_b200"))
    from pse import dist as pd
    from pse import workload as wl
    from pse.scheduler import Request
    w = wl.WORKLOADS["llama-1b"]
    reqs = [Request(f"r{i}", p, w.max_new_tokens) for i, p in enumerate(wl.prompts(w, seed=1, n=2048))]
    for world in (2, 4, 8):
        loads = [sum(len(r.prompt_ids) + r.max_new_tokens for r in pd.shard_requests(reqs, world, k))
                 for k in range(world)]
        assert max(loads) / min(loads) < 1.01

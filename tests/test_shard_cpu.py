"""Batch-shard planning and the multi-rank driver on CPU (gloo, world size 2),
including a rank that fails before the gather."""
from __future__ import annotations

import os
import socket

import pytest
import torch
import torch.multiprocessing as mp

from persistent_lstm_hip_b200.shard import distributed_forward, plan_shards, shard_balance


def test_plan_uniform_is_contiguous_and_complete():
    plan = plan_shards(4096, 8)
    assert [int(p.numel()) for p in plan] == [512] * 8
    assert torch.equal(torch.cat(plan), torch.arange(4096))
    plan = plan_shards(10, 3)
    assert sorted(torch.cat(plan).tolist()) == list(range(10))


def test_plan_varlen_balances_rows_and_lengths():
    g = torch.Generator().manual_seed(2)
    lens = torch.randint(200, 1001, (4096,), generator=g)
    for n in (1, 2, 4, 8):
        plan = plan_shards(4096, n, lens.tolist())
        assert sorted(torch.cat(plan).tolist()) == list(range(4096))
        rep = shard_balance(plan, lens.tolist())["shards"]
        assert {r["rows"] for r in rep} == {4096 // n}
        sums = [r["sum_len"] for r in rep]
        assert max(sums) - min(sums) <= 800  # one row's worth of length
        assert max(r["max_len"] for r in rep) - min(r["max_len"] for r in rep) <= 10


def _free_port() -> int:
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _row_fn(x, lengths):
    v = x.double().sum(dim=(1, 2))
    if lengths is not None:
        v = v + lengths.double()
    return torch.stack([v, 2 * v], dim=1)


def _worker(rank, world, port, varlen, fail_rank, q):
    import datetime

    import torch.distributed as dist

    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    dist.init_process_group("gloo", rank=rank, world_size=world, timeout=datetime.timedelta(seconds=6))
    try:
        g = torch.Generator().manual_seed(0)
        x = torch.randn(64, 7, 3, generator=g)
        lens = torch.randint(1, 8, (64,), generator=g) if varlen else None
        plan = plan_shards(64, world, None if lens is None else lens.tolist())
        mine = plan[rank]
        if rank == fail_rank:
            raise RuntimeError("injected rank failure before the gather")
        out = distributed_forward(_row_fn, x[mine], plan, None if lens is None else lens[mine])
        q.put((rank, "ok", torch.allclose(out, _row_fn(x, lens))))
    except Exception as exc:  # reported to the parent, not swallowed
        q.put((rank, "error", type(exc).__name__ + ": " + str(exc)[:200]))
    finally:
        try:
            dist.destroy_process_group()
        except Exception:
            pass


def _run(world, varlen, fail_rank=-1):
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=_worker, args=(r, world, port, varlen, fail_rank, q)) for r in range(world)]
    for p in procs:
        p.start()
    res = [q.get(timeout=120) for _ in range(world)]
    for p in procs:
        p.join(timeout=60)
    return sorted(res)


@pytest.mark.parametrize("varlen", [False, True])
def test_distributed_forward_gloo_world2(varlen):
    res = _run(2, varlen)
    assert res == [(0, "ok", True), (1, "ok", True)]


def test_rank_failure_is_detected_by_the_survivor():
    res = _run(2, False, fail_rank=1)
    assert res[1][1] == "error" and "injected" in res[1][2]
    assert res[0][1] == "error"  # the gather fails (peer gone / timeout) instead of hanging

"""The multi-GPU path is replicas (one process per GPU, own request stream): the only
cross-rank work is the host-side reduction of timings in woodcock_b200.replicas, run here as
two gloo ranks on the CPU."""

from __future__ import annotations

import os
import socket

import pytest
import torch.multiprocessing as mp


def _free_port() -> int:
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _rank(rank, world, port, q):
    import torch.distributed as dist
    from datetime import timedelta

    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
    dist.init_process_group("gloo", rank=rank, world_size=world, timeout=timedelta(seconds=60))
    try:
        from woodcock_b200.replicas import aggregate

        # rank r timed (10 + r) ms of device work for 30 tokens, its wall clock 1 + r s
        out = aggregate(10.0 + rank, 30.0, 1.0 + rank)
        dist.barrier()
        q.put((rank, out))
    finally:
        dist.destroy_process_group()


def test_two_gloo_ranks_aggregate_as_replicas():
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=_rank, args=(r, 2, port, q)) for r in range(2)]
    for p in procs:
        p.start()
    res = dict(q.get(timeout=120) for _ in procs)
    for p in procs:
        p.join(timeout=60)
        assert p.exitcode == 0
    for r in range(2):
        out = res[r]
        assert out["world"] == 2
        assert out["device_ms"] == pytest.approx(11.0)  # the slowest rank
        assert out["wall_s"] == pytest.approx(2.0)
        assert out["tokens"] == pytest.approx(60.0)     # both ranks' tokens
        assert out["value"] == pytest.approx(60.0 / 0.011)


def test_single_process_is_its_own_job():
    from woodcock_b200.replicas import aggregate

    out = aggregate(20.0, 10.0)
    assert out["world"] == 1 and out["value"] == pytest.approx(500.0)

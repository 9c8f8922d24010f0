"""Multi-GPU runs are replicas: one process per GPU, each decoding its own request stream
(batch-1 decoding does not shard, and the reference has no collective on this path). The
only cross-rank steps are host-side: a start barrier and this reduction of the timings,
over a CPU (gloo) process group — no device collective, no peer memory."""

from __future__ import annotations


def aggregate(device_ms: float, tokens: float, wall_s: float = 0.0) -> dict:
    """Whole-job figures from every rank's own: the job's device time is the slowest rank's,
    tokens add up; value = tokens / job time. Needs an initialised process group when the
    world is larger than one; every rank must call it (it is a collective)."""
    import torch
    import torch.distributed as dist

    world = dist.get_world_size() if dist.is_available() and dist.is_initialized() else 1
    if world > 1:
        t = torch.tensor([device_ms, wall_s], dtype=torch.float64)
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
        n = torch.tensor([tokens], dtype=torch.float64)
        dist.all_reduce(n, op=dist.ReduceOp.SUM)
        device_ms, wall_s, tokens = float(t[0]), float(t[1]), float(n[0])
    return {"world": world, "device_ms": device_ms, "wall_s": wall_s, "tokens": tokens,
            "value": tokens / (device_ms / 1e3) if device_ms > 0 else 0.0}

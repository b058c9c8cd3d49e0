"""Data-parallel layer: one process per GPU, each op sharded along its natural axis.

The reference has no multi-GPU code. Here every headline workload partitions into
independent units, and the only exchange steps are the ones the math needs:

    reduce_sum        contiguous chunks; local fp32 partial -> all_reduce(SUM)
    softmax           row blocks; no collective (all_gather only to assemble)
    matmul            M-blocks of A (B replicated); all_gather of C only to assemble
    attention(_causal) (B*H) slices; all_gather of O only to assemble

Ops are passed in as callables so the same host logic runs the CUDA kernels on GPUs
(NCCL) and the PyTorch CPU baseline in multi-process tests (gloo).
"""

from __future__ import annotations

import datetime
import os
from collections.abc import Callable
from dataclasses import dataclass

import torch
import torch.distributed as dist


@dataclass(frozen=True)
class Rank:
    rank: int
    world: int
    local_rank: int

    @property
    def is_main(self) -> bool:
        return self.rank == 0


def env_rank() -> Rank:
    return Rank(int(os.environ.get("RANK", 0)), int(os.environ.get("WORLD_SIZE", 1)),
                int(os.environ.get("LOCAL_RANK", 0)))


def init(backend: str | None = None, timeout_s: float = 120.0) -> Rank:
    """Join the process group described by the torchrun environment (no-op at world 1)."""
    r = env_rank()
    if r.world > 1 and not dist.is_initialized():
        if backend is None:
            backend = "nccl" if torch.cuda.is_available() else "gloo"
        if backend == "nccl":
            torch.cuda.set_device(r.local_rank)
        os.environ.setdefault("MASTER_ADDR", "127.0.0.1")
        kw = {}
        if backend == "nccl":
            kw["device_id"] = torch.device("cuda", r.local_rank)
        dist.init_process_group(backend, timeout=datetime.timedelta(seconds=timeout_s), **kw)
    return r


def shard_range(n: int, rank: int, world: int) -> tuple[int, int]:
    """Contiguous [start, stop) of ``n`` units for ``rank``: the first n % world ranks
    take one extra unit, so sizes differ by at most one."""
    if n < 0 or world < 1 or not 0 <= rank < world:
        raise ValueError(f"bad shard request n={n} rank={rank} world={world}")
    base, extra = divmod(n, world)
    start = rank * base + min(rank, extra)
    return start, start + base + (1 if rank < extra else 0)


def sharded_reduce_sum(x_local: torch.Tensor, op: Callable[[torch.Tensor], torch.Tensor]
                       ) -> torch.Tensor:
    """Global sum: the local fp32 partial of this rank's chunk, combined by one
    all_reduce(SUM) of a single float (the only exchange step)."""
    part = op(x_local).reshape(1).to(torch.float32)
    if dist.is_initialized() and dist.get_world_size() > 1:
        dist.all_reduce(part, op=dist.ReduceOp.SUM)
    return part.reshape(())


def assemble_rows(local: torch.Tensor, counts: list[int]) -> torch.Tensor:
    """All-gather row blocks of (possibly) unequal sizes into the full tensor along
    dim 0, in rank order."""
    world = dist.get_world_size()
    if world == 1:
        return local
    cap = max(counts)
    pad = torch.zeros((cap - local.shape[0],) + tuple(local.shape[1:]), dtype=local.dtype,
                      device=local.device)
    mine = torch.cat([local, pad]) if pad.shape[0] else local.contiguous()
    out = torch.empty((cap * world,) + tuple(local.shape[1:]), dtype=local.dtype,
                      device=local.device)
    dist.all_gather_into_tensor(out, mine)
    return torch.cat([out[i * cap: i * cap + c] for i, c in enumerate(counts)])


def row_counts(n: int, world: int) -> list[int]:
    return [b - a for a, b in (shard_range(n, r, world) for r in range(world))]

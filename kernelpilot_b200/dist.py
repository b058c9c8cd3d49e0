"""Data-parallel layer: one process per GPU, each op sharded along its natural axis.

The reference has no multi-GPU code. Here every headline workload partitions into
independent units, and the only exchange steps are the ones the math needs:

    reduce_sum        contiguous chunks; the per-GPU sums are exchanged inside the
                      finishing kernel over NVLink peer memory (PeerSum), or by an
                      all_reduce(SUM) of the fp32 partial (sharded_reduce_sum)
    softmax           row blocks; no collective (all_gather only to assemble)
    matmul            M-blocks of A (B replicated); all_gather of C only to assemble
    attention(_causal) (B*H) slices; all_gather of O only to assemble

Ops are passed in as callables so the same host logic runs the CUDA kernels on GPUs
(NCCL) and the PyTorch CPU baseline in multi-process tests (gloo).
"""

from __future__ import annotations

import ctypes
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


# the axis each op is split along, and what a rank holds
PARTITION: dict[str, str] = {
    "reduce_sum": "contiguous element chunks (sizes differ by at most one)",
    "vector_add": "contiguous element chunks of a and b",
    "softmax": "row blocks",
    "layernorm": "row blocks (w and b replicated)",
    "matmul": "M-blocks: row blocks of A and C (B replicated)",
    "attention": "(batch, head) slices of q, k, v and o",
    "attention_causal": "(batch, head) slices of q, k, v and o",
}


def _units(kernel: str, shape: tuple) -> int:
    """Independent units of an op's shape along its partition axis."""
    if kernel in ("attention", "attention_causal"):
        return shape[0] * shape[1]
    return shape[0]


def local_shape(kernel: str, shape: tuple, rank: int, world: int) -> tuple:
    """The shape this rank's shard of a global ``shape`` has, as the op sees it."""
    if kernel not in PARTITION:
        raise KeyError(f"no partition for {kernel!r}")
    if world == 1:
        return tuple(shape)
    a, b = shard_range(_units(kernel, shape), rank, world)
    if kernel in ("attention", "attention_causal"):
        return (1, b - a) + tuple(shape[2:])
    return (b - a,) + tuple(shape[1:])


def shard_inputs(kernel: str, inputs: tuple, rank: int, world: int) -> tuple:
    """This rank's part of the global inputs, as contiguous tensors (copies when
    world > 1, so the global tensors can be freed)."""
    if world == 1:
        return tuple(inputs)
    if kernel in ("attention", "attention_causal"):
        B, H, S, D = inputs[0].shape
        a, b = shard_range(B * H, rank, world)
        return tuple(t.reshape(B * H, S, D)[a:b].reshape(1, b - a, S, D).clone()
                     for t in inputs)
    a, b = shard_range(_units(kernel, tuple(inputs[0].shape)), rank, world)
    if kernel in ("reduce_sum", "vector_add"):
        return tuple(t.reshape(-1)[a:b].clone() for t in inputs)
    if kernel in ("softmax", "matmul", "layernorm"):
        return (inputs[0][a:b].clone(),) + tuple(inputs[1:])
    raise KeyError(f"no partition for {kernel!r}")


def sharded_reduce_sum(x_local: torch.Tensor, op: Callable[[torch.Tensor], torch.Tensor]
                       ) -> torch.Tensor:
    """Global sum: the local fp32 partial of this rank's chunk, combined by one
    all_reduce(SUM) of a single float (the only exchange step)."""
    part = op(x_local).reshape(1).to(torch.float32)
    if dist.is_initialized() and dist.get_world_size() > 1:
        dist.all_reduce(part, op=dist.ReduceOp.SUM)
    return part.reshape(())


class PeerSum:
    """Global sum of a vector sharded over this node's GPUs, with the exchange step
    inside the finishing kernel over NVLink peer memory (``kpb_peer_sum_*``): each
    call reduces the local shard and the one-CTA finishing kernel stores its sum into
    every rank's exchange buffer, waits (bounded) for the others and adds them in rank
    order, so every rank gets the same bits and no collective is launched.

    Construction is collective (every rank of the process group must construct it, in
    the same order as its other collectives): the ranks export their exchange buffers
    as CUDA IPC handles, agree that all exports worked (else every rank raises and the
    caller can fall back to ``sharded_reduce_sum``) and all-gather the handles. Calls
    must then be made by every rank, the same number of times, in the same order, on
    one stream per rank. The call number lives in device memory, so a call captured in
    a CUDA graph may be replayed (by every rank, equally often).

    If a rank misses a call, the others' bounded waits give up: they return NaN and
    their exchange is marked out of step for good (later calls return NaN at once).
    ``healthy()`` (collective, synchronising) finds that out; after it has returned
    False every call raises, and the caller can fall back to ``sharded_reduce_sum``.
    """

    def __init__(self, group=None):
        from . import ext

        self._lib = lib = ext.capi()
        self._group = group
        self._broken = False
        world = dist.get_world_size(group) if dist.is_initialized() else 1
        rank = dist.get_rank(group) if dist.is_initialized() else 0
        self._world = world
        nb = lib.kpb_peer_sum_handle_bytes()
        handle = ctypes.create_string_buffer(nb)
        self._ps = ctypes.c_void_p()
        rc = lib.kpb_peer_sum_create(rank, world, handle, ctypes.byref(self._ps))
        msg = lib.kpb_last_error().decode() if rc else ""
        dev = (torch.device("cuda", torch.cuda.current_device()) if torch.cuda.is_available()
               else torch.device("cpu"))
        if world > 1:
            ok = torch.tensor([1 if rc == 0 else 0], device=dev)
            dist.all_reduce(ok, op=dist.ReduceOp.MIN, group=group)
            if int(ok.item()) == 0:
                self._release()
                raise RuntimeError(f"peer sum unavailable on some rank ({msg or 'another rank'})")
            mine = torch.frombuffer(bytearray(handle.raw), dtype=torch.uint8).to(dev)
            every = torch.empty(world * nb, dtype=torch.uint8, device=dev)
            dist.all_gather_into_tensor(every, mine, group=group)
            raw = bytes(every.cpu().tolist())
        else:
            if rc:
                raise RuntimeError(f"peer sum unavailable: {msg}")
            raw = handle.raw
        rc = lib.kpb_peer_sum_connect(self._ps, raw)
        msg = lib.kpb_last_error().decode() if rc else ""
        if world > 1:
            # every rank must take the same path: fail together if any rank could not
            # map its peers
            ok = torch.tensor([1 if rc == 0 else 0], device=dev)
            dist.all_reduce(ok, op=dist.ReduceOp.MIN, group=group)
            rc = 0 if int(ok.item()) == 1 else (rc or 1)
        if rc:
            self._release()
            raise RuntimeError(f"peer sum connect failed on some rank ({msg or 'another rank'})")
        self._ws = torch.empty(0, dtype=torch.uint8, device=dev)

    def __call__(self, x_local: torch.Tensor) -> torch.Tensor:
        from . import ext

        if self._broken:
            raise RuntimeError("peer sum is out of step (a rank missed a call); "
                               "use sharded_reduce_sum")
        if self._ps is None:
            raise RuntimeError("peer sum is closed")
        x = x_local.reshape(-1)
        if not x.is_contiguous():
            x = x.contiguous()
        n = x.numel()
        need = self._lib.kpb_peer_sum_workspace_bytes(n)
        if self._ws.numel() < need:
            self._ws = torch.empty(need, dtype=torch.uint8, device=x.device)
        out = torch.empty((), dtype=torch.float32, device=x.device)
        ext.capi_check(self._lib.kpb_peer_sum_run(
            self._ps, ext.DTYPE_CODES[x.dtype], x.data_ptr(), out.data_ptr(), n,
            self._ws.data_ptr(), self._ws.numel(), ext.current_stream_ptr(x.device)))
        return out

    def healthy(self) -> bool:
        """True while every rank's exchange is in step. Collective at world > 1 (every
        rank must call it, at the same point of its call sequence); synchronises the
        device. Once False, later calls raise."""
        from . import ext

        if self._ps is None:
            return False
        flag = ctypes.c_int(0)
        ext.capi_check(self._lib.kpb_peer_sum_status(self._ps, ctypes.byref(flag)))
        bad = torch.tensor([flag.value], device=self._ws.device, dtype=torch.int32)
        if self._world > 1:
            dist.all_reduce(bad, op=dist.ReduceOp.MAX, group=self._group)
        if int(bad.item()):
            self._broken = True
        return not self._broken

    def close(self) -> None:
        """Release the exchange buffer and the peers' mappings. Collective at world > 1:
        each rank waits for its own work to finish, then for every other rank to get
        here, so no peer still stores into a buffer that is being freed."""
        if getattr(self, "_ps", None) is None:
            return
        if self._world > 1 and dist.is_initialized():
            torch.cuda.synchronize()
            dist.barrier(group=self._group)
        self._release()

    def _release(self) -> None:
        if getattr(self, "_ps", None) is not None and self._ps.value:
            self._lib.kpb_peer_sum_destroy(self._ps)
        self._ps = None


_GATHER_ALIGN = 256  # bytes per rank slot of a gathered block


def assemble_rows(local: torch.Tensor, counts: list[int]) -> torch.Tensor:
    """All-gather row blocks of (possibly) unequal sizes into the full tensor along
    dim 0, in rank order. Blocks of equal size whose bytes are a multiple of
    ``_GATHER_ALIGN`` are gathered straight into the result. Any other blocks go
    through one flat buffer whose per-rank slot is the largest block rounded up to
    ``_GATHER_ALIGN`` bytes, and are compacted afterwards: NCCL moves misaligned
    per-rank chunks at a small fraction of its aligned rate."""
    world = dist.get_world_size()
    if world == 1:
        return local
    local = local.contiguous()
    inner = tuple(local.shape[1:])
    row = 1
    for d in inner:
        row *= d
    esize = local.element_size()
    if all(c == counts[0] for c in counts) and (counts[0] * row * esize) % _GATHER_ALIGN == 0:
        out = torch.empty((counts[0] * world,) + inner, dtype=local.dtype, device=local.device)
        dist.all_gather_into_tensor(out, local)
        return out
    align = max(1, _GATHER_ALIGN // esize)
    slot = -(-max(counts) * row // align) * align
    mine = torch.zeros(slot, dtype=local.dtype, device=local.device)
    mine[: local.numel()].copy_(local.reshape(-1))
    flat = torch.empty(slot * world, dtype=local.dtype, device=local.device)
    dist.all_gather_into_tensor(flat, mine)
    return torch.cat([flat[i * slot: i * slot + c * row] for i, c in enumerate(counts)]
                     ).reshape((sum(counts),) + inner)


def row_counts(n: int, world: int) -> list[int]:
    return [b - a for a, b in (shard_range(n, r, world) for r in range(world))]

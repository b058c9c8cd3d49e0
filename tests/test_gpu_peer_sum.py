"""The full sum over GPUs with the exchange inside the finishing kernel (dist.PeerSum
over kpb_peer_sum_*): on one GPU it equals kpb_reduce_sum bit for bit, eagerly and
replayed from a CUDA graph; on two GPUs (one process each, NCCL only to hand the IPC
handles around) every rank gets the same bits, equal to the rank-ordered fp32 sum of
the ranks' own reductions, on several calls in a row (both exchange rows) and on graph
replays where one rank arrives late (a call number frozen into the graph would let the
early rank read the late rank's previous word); and a rank that skips a call makes the
other rank's bounded wait give up with NaN and the timeout bit instead of hanging,
after which the exchange reports itself out of step and answers NaN without waiting."""

import os
import socket

import pytest
import torch
import torch.multiprocessing as mp

from kernelpilot_b200 import dist as kdist
from kernelpilot_b200 import ext
from kernelpilot_b200.specs import get_spec

pytestmark = pytest.mark.gpu


def _reduce(x):
    out = torch.empty((), device=x.device)
    ext.capi_check(ext.capi().kpb_reduce_sum(2, ext.DTYPE_CODES[x.dtype], x.data_ptr(),
                                             out.data_ptr(), x.numel(),
                                             ext.current_stream_ptr(x.device)))
    return out


def test_one_gpu_matches_the_allocating_reduction_bit_for_bit():
    peer = kdist.PeerSum()
    try:
        spec = get_spec("reduce_sum")
        for seed, n, dtype in [(0, 2**24 + 3, torch.float32), (1, 1_000_001, torch.bfloat16),
                               (2, 7, torch.float16), (3, 2**24 + 3, torch.float32)]:
            x = spec.make_inputs((n,), dtype, torch.device("cuda"), seed)[0]
            got, want = peer(x), _reduce(x)
            torch.cuda.synchronize()
            assert torch.equal(got, want), (n, str(dtype), float(got), float(want))
        empty = peer(torch.empty(0, device="cuda"))
        torch.cuda.synchronize()
        assert float(empty) == 0.0
    finally:
        peer.close()


def test_one_gpu_graph_replays_follow_the_input():
    spec = get_spec("reduce_sum")
    n = 2**22 + 5
    x = torch.empty(n, device="cuda")
    peer = kdist.PeerSum()
    try:
        x.copy_(spec.make_inputs((n,), torch.float32, torch.device("cuda"), 0)[0])
        peer(x)  # sizes the workspace before capture
        torch.cuda.synchronize()
        g = torch.cuda.CUDAGraph()
        with torch.cuda.graph(g):
            out = peer(x)
        for seed in (1, 2, 3):
            x.copy_(spec.make_inputs((n,), torch.float32, torch.device("cuda"), seed)[0])
            g.replay()
            want = _reduce(x)
            torch.cuda.synchronize()
            assert torch.equal(out, want), (seed, float(out), float(want))
        assert peer.healthy()
        del g
    finally:
        peer.close()


def _free_port() -> int:
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _two_rank_worker(rank: int, world: int, port: int, results) -> None:
    import datetime

    import torch.distributed as dist

    os.environ["NCCL_NVLS_ENABLE"] = "0"
    torch.cuda.set_device(rank)
    dist.init_process_group("nccl", init_method=f"tcp://127.0.0.1:{port}", rank=rank,
                            world_size=world, timeout=datetime.timedelta(seconds=60),
                            device_id=torch.device("cuda", rank))
    try:
        spec = get_spec("reduce_sum")
        peer = kdist.PeerSum()
        for call in range(3):
            x = spec.make_inputs((3_000_017 + rank,), torch.float32, torch.device("cuda"),
                                 10 * call + rank)[0]
            got = peer(x)
            mine = _reduce(x)
            both = [torch.empty((), device="cuda") for _ in range(world)]
            dist.all_gather(both, mine)
            want = both[0] + both[1]  # fp32, rank order
            seen = [torch.empty((), device="cuda") for _ in range(world)]
            dist.all_gather(seen, got)
            torch.cuda.synchronize()
            results[(rank, call)] = (got.item(), want.item(), seen[0].item(), seen[1].item())
        # graph replays with rank 0 arriving ~50 ms late: rank 1 must wait for rank 0's
        # word of this replay, not take the one left by the previous replay
        n = 1_000_003
        x = torch.empty(n, device="cuda")
        x.copy_(spec.make_inputs((n,), torch.float32, torch.device("cuda"), 50 + rank)[0])
        peer(x)
        torch.cuda.synchronize()
        dist.barrier()
        g = torch.cuda.CUDAGraph()
        with torch.cuda.graph(g):
            gout = peer(x)
        for rep in range(3):
            x.copy_(spec.make_inputs((n,), torch.float32, torch.device("cuda"),
                                     60 + 10 * rep + rank)[0])
            torch.cuda.synchronize()
            dist.barrier()
            if rank == 0:
                torch.cuda._sleep(100_000_000)
            g.replay()
            mine = _reduce(x)
            both = [torch.empty((), device="cuda") for _ in range(world)]
            dist.all_gather(both, mine)
            want = both[0] + both[1]
            torch.cuda.synchronize()
            results[(rank, "graph", rep)] = (gout.item(), want.item())
        del g
        assert peer.healthy()
        # rank 1 skips the next call: rank 0's wait must give up, not hang
        dist.barrier()
        ext.capi().kpb_device_errors(None)  # clear the word
        if rank == 0:
            x = spec.make_inputs((1000,), torch.float32, torch.device("cuda"), 99)[0]
            got = peer(x)
            torch.cuda.synchronize()
            word = ext.ctypes.c_uint(0)
            ext.capi_check(ext.capi().kpb_device_errors(ext.ctypes.byref(word)))
            results[(rank, "timeout")] = (got.item(), word.value)
            # out of step now: the next call answers NaN without waiting again
            import time

            t0 = time.perf_counter()
            again = peer(x)
            torch.cuda.synchronize()
            results[(rank, "after")] = (again.item(), time.perf_counter() - t0)
        torch.cuda.synchronize()
        dist.barrier()
        results[(rank, "healthy")] = peer.healthy()
        try:
            peer(torch.ones(4, device="cuda"))
            results[(rank, "raises")] = False
        except RuntimeError:
            results[(rank, "raises")] = True
        peer.close()
    finally:
        dist.destroy_process_group()


@pytest.mark.skipif(torch.cuda.device_count() < 2, reason="needs two GPUs")
def test_two_gpus_agree_bit_for_bit_and_time_out_cleanly():
    results = mp.get_context("spawn").Manager().dict()
    mp.spawn(_two_rank_worker, args=(2, _free_port(), results), nprocs=2, join=True)
    for call in range(3):
        for rank in range(2):
            got, want, s0, s1 = results[(rank, call)]
            assert got == want, (rank, call, got, want)
            assert s0 == s1  # the same bits on both ranks
    for rep in range(3):
        for rank in range(2):
            got, want = results[(rank, "graph", rep)]
            assert got == want, (rank, rep, got, want)
    got, word = results[(0, "timeout")]
    assert got != got  # NaN
    assert word & 1  # the timeout bit of the device error word
    again, seconds = results[(0, "after")]
    assert again != again and seconds < 1.0
    assert results[(0, "healthy")] is False and results[(1, "healthy")] is False
    assert results[(0, "raises")] and results[(1, "raises")]

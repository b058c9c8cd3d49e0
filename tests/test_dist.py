"""Host logic of the data-parallel layer with world_size 2 gloo ranks on CPU: shard
ranges cover every unit once, the reduction partials combine into the global sum,
and row blocks of unequal size assemble in rank order."""

import os
import socket

import pytest
import torch
import torch.distributed as dist
import torch.multiprocessing as mp

from kernelpilot_b200 import dist as kdist


@pytest.mark.parametrize("n,world", [(0, 1), (1, 2), (7, 2), (10, 3), (2**28 + 1, 8)])
def test_shard_ranges_partition(n, world):
    spans = [kdist.shard_range(n, r, world) for r in range(world)]
    assert spans[0][0] == 0 and spans[-1][1] == n
    for (a0, b0), (a1, _b1) in zip(spans, spans[1:], strict=False):
        assert b0 == a1
    sizes = [b - a for a, b in spans]
    assert max(sizes) - min(sizes) <= 1


def test_shard_range_rejects_bad_ranks():
    with pytest.raises(ValueError):
        kdist.shard_range(10, 2, 2)


def _free_port() -> int:
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _worker(rank, world, port, q):
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port), RANK=str(rank),
                      WORLD_SIZE=str(world), LOCAL_RANK=str(rank))
    try:
        kdist.init(backend="gloo", timeout_s=30)
        g = torch.Generator().manual_seed(0)
        x = torch.rand(1001, generator=g) * 2 - 1
        a, b = kdist.shard_range(x.numel(), rank, world)
        total = kdist.sharded_reduce_sum(x[a:b], lambda t: t.sum(dtype=torch.float32))
        rows = torch.arange(7 * 3, dtype=torch.float32).reshape(7, 3)
        ra, rb = kdist.shard_range(7, rank, world)
        full = kdist.assemble_rows(torch.softmax(rows[ra:rb], -1),
                                   kdist.row_counts(7, world))
        ok = bool(torch.allclose(full, torch.softmax(rows, -1)))
        # equal blocks both sides of the slot alignment, and a 2-byte type unequal
        for n_rows, width, dt in [(8, 3, torch.float32), (8, 32, torch.float32),
                                  (9, 5, torch.bfloat16)]:
            whole = torch.arange(n_rows * width, dtype=torch.float32).reshape(n_rows, width)
            whole = whole.to(dt)
            ra, rb = kdist.shard_range(n_rows, rank, world)
            got = kdist.assemble_rows(whole[ra:rb], kdist.row_counts(n_rows, world))
            ok = ok and got.dtype == dt and torch.equal(got, whole)
        q.put((rank, float(total), float(x.double().sum()), ok))
        dist.destroy_process_group()
    except Exception as e:  # reported to the parent, which fails the test
        q.put((rank, "error", repr(e), False))


def test_two_gloo_ranks_combine_partials_and_assemble_rows():
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=_worker, args=(r, 2, port, q)) for r in range(2)]
    for p in procs:
        p.start()
    results = [q.get(timeout=120) for _ in procs]
    for p in procs:
        p.join(timeout=60)
    for rank, total, want, assembled in results:
        assert total != "error", want
        assert abs(total - want) < 1e-3, (rank, total, want)
        assert assembled


def _fallback_worker(rank, world, port, q):
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port), RANK=str(rank),
                      WORLD_SIZE=str(world), LOCAL_RANK=str(rank))
    try:
        kdist.init(backend="gloo", timeout_s=30)
        # no rank can export an exchange buffer here (no GPU): every rank must learn it
        # in the same collective and raise, so all can fall back to the all_reduce
        try:
            kdist.PeerSum()
            outcome = "constructed"
        except RuntimeError as e:
            outcome = str(e)
        x = torch.full((10,), float(rank + 1))
        total = kdist.sharded_reduce_sum(x, lambda t: t.sum(dtype=torch.float32))
        dist.barrier()
        q.put((rank, outcome, float(total)))
        dist.destroy_process_group()
    except Exception as e:
        q.put((rank, "error", repr(e)))


def test_peer_sum_unavailable_on_every_rank_falls_back_together():
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=_fallback_worker, args=(r, 2, port, q)) for r in range(2)]
    for p in procs:
        p.start()
    results = [q.get(timeout=120) for _ in procs]
    for p in procs:
        p.join(timeout=60)
    for rank, outcome, total in results:
        assert outcome.startswith("peer sum unavailable"), (rank, outcome, total)
        assert total == 30.0  # 10 * 1 + 10 * 2 on both ranks, through the fallback


@pytest.mark.parametrize("kernel,shape", [
    ("reduce_sum", (1001,)), ("vector_add", (17,)), ("softmax", (7, 5)), ("layernorm", (9, 4)),
    ("matmul", (10, 3, 4)), ("attention", (2, 3, 8, 4)), ("attention_causal", (1, 5, 8, 4))])
@pytest.mark.parametrize("world", [1, 2, 3, 8])
def test_shards_reassemble_the_global_inputs(kernel, shape, world):
    from kernelpilot_b200.specs import get_spec

    spec = get_spec(kernel)
    full = spec.make_inputs(shape, torch.float32, torch.device("cpu"), 0)
    parts = [kdist.shard_inputs(kernel, full, r, world) for r in range(world)]
    for r, p in enumerate(parts):
        # matmul's spec shape is (M, N, K): A is (M, K), B is (K, N)
        seen = (p[0].shape[0], p[1].shape[1], p[0].shape[1]) if kernel == "matmul" \
            else tuple(p[0].shape)
        assert seen == kdist.local_shape(kernel, shape, r, world)
        assert all(t.is_contiguous() for t in p)
    if kernel in ("attention", "attention_causal"):
        B, H, S, D = shape
        for i in range(3):
            got = torch.cat([p[i].reshape(-1, S, D) for p in parts]).reshape(shape)
            assert torch.equal(got, full[i])
    elif kernel in ("reduce_sum", "vector_add"):
        for i in range(len(full)):
            assert torch.equal(torch.cat([p[i] for p in parts]), full[i])
    else:
        assert torch.equal(torch.cat([p[0] for p in parts]), full[0])
        for i in range(1, len(full)):  # replicated operands
            assert all(torch.equal(p[i], full[i]) for p in parts)
    # the shards' work adds up to the job's (up to the reduction's 4-byte result each)
    if kernel != "reduce_sum":
        total = sum(spec.flops(kdist.local_shape(kernel, shape, r, world)) for r in range(world))
        assert total == pytest.approx(spec.flops(shape)) or kernel == "attention_causal"


def _sharded_op_worker(rank, world, port, q):
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port), RANK=str(rank),
                      WORLD_SIZE=str(world), LOCAL_RANK=str(rank))
    try:
        from kernelpilot_b200.specs import get_spec

        kdist.init(backend="gloo", timeout_s=30)
        ok = []
        # unequal blocks (padded gather) and equal ones (gathered in place)
        for kernel, shape in [("softmax", (9, 33)), ("matmul", (9, 5, 7)),
                              ("attention", (1, 3, 16, 8)), ("layernorm", (5, 12)),
                              ("softmax", (8, 33)), ("attention", (2, 2, 16, 8))]:
            spec = get_spec(kernel)
            full = spec.make_inputs(shape, torch.float32, torch.device("cpu"), 0)
            local = kdist.shard_inputs(kernel, full, rank, world)
            out = spec.baseline(*local)
            if kernel == "attention":
                B, H, S, D = shape
                counts = kdist.row_counts(B * H, world)
                got = kdist.assemble_rows(out.reshape(-1, S, D).contiguous(), counts)
                got = got.reshape(shape)
            else:
                got = kdist.assemble_rows(out.contiguous(), kdist.row_counts(shape[0], world))
            ok.append(bool(torch.allclose(got, spec.baseline(*full), atol=1e-5, rtol=1e-5)))
        q.put((rank, ok))
        dist.destroy_process_group()
    except Exception as e:
        q.put((rank, repr(e)))


def test_two_gloo_ranks_split_each_op_and_reassemble_its_output():
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=_sharded_op_worker, args=(r, 2, port, q)) for r in range(2)]
    for p in procs:
        p.start()
    results = [q.get(timeout=120) for _ in procs]
    for p in procs:
        p.join(timeout=60)
    for rank, ok in results:
        assert ok == [True] * 6, (rank, ok)

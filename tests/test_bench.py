"""Host-side pieces of bench.py (no GPU): launch counts claimed in the JSON line and the
algorithmic work each headline workload is measured against."""
import dataclasses

import pytest

import bench
from kernelpilot_b200.specs import CONFIGS


@pytest.mark.parametrize("key,expected", [
    ("reduce_f32_2p28p1", 2),             # persistent level + one-CTA finish
    ("softmax_f32_4096x4097", 1),
    ("softmax_bf16_65536x32768", 1),
    ("softmax_bf16_4096x131072", 1),
    ("gemm_bf16_8192", 1),
    ("gemm_bf16_4097x4097x4096", 2),      # B's 8194-byte rows take a pitch copy first
    ("attn_bf16_b8h32s4096d128", 1),
    ("attn_causal_bf16_b8h32s4096d128", 2),  # main grid + the few-key-rows grid
    ("vadd_f32_2p26", 1),
    ("layernorm_f32_8192x8192", 1),
    ("layernorm_bf16_8192x8192", 1),
])
def test_launches_per_call(key, expected):
    assert bench.launches_per_call(CONFIGS[key]) == expected


def test_launches_per_call_short_causal_is_one_grid():
    w = CONFIGS["attn_causal_bf16_b8h32s4096d128"]
    short = dataclasses.replace(w, shape=(w.shape[0], w.shape[1], 256, w.shape[3]))
    assert bench.launches_per_call(short) == 1


def test_launches_per_call_gemm_pads_each_unaligned_operand():
    w = CONFIGS["gemm_bf16_8192"]
    assert bench.launches_per_call(dataclasses.replace(w, shape=(512, 512, 4100))) == 2
    assert bench.launches_per_call(dataclasses.replace(w, shape=(512, 4100, 4100))) == 3


def test_work_per_call_is_the_spec_formula():
    # the figures the roofline fractions are computed from (kernelpilot/specs.py formulas)
    assert bench.work_per_call(CONFIGS["softmax_f32_4096x4097"]) == 2 * 4096 * 4097 * 4
    assert bench.work_per_call(CONFIGS["reduce_f32_2p28p1"]) == 4 * (2**28 + 1) + 4
    assert bench.work_per_call(CONFIGS["gemm_bf16_8192"]) == pytest.approx(2 * 8192**3)
    assert bench.work_per_call(CONFIGS["attn_bf16_b8h32s4096d128"]) == pytest.approx(
        4 * 8 * 32 * 4096 * 4096 * 128)
    assert bench.work_per_call(CONFIGS["vadd_f32_2p26"]) == 3 * 4 * 2**26
    assert bench.work_per_call(CONFIGS["layernorm_bf16_8192x8192"]) == (
        2 * 8192 * 8192 + 2 * 8192) * 2
    # causal: the useful FLOPs (half the scores plus the diagonal)
    assert bench.work_per_call(CONFIGS["attn_causal_bf16_b8h32s4096d128"]) == pytest.approx(
        4 * 8 * 32 * 4096 * 4097 / 2 * 128)


@pytest.mark.parametrize("world", [1, 2, 8])
def test_both_arms_print_the_same_config(world):
    for key, w in CONFIGS.items():
        cfg = bench.job_config(w, world)
        assert cfg == bench.job_config(w, world)
        assert cfg["workload"] == key and cfg["parallelism"] == f"dp{world}"
        # a rank's shard is one of the listed shapes
        assert list(bench.local_workload(w, world - 1, world).shape) in cfg["per_rank"]


def test_partitioned_reduction_shards_are_near_equal():
    w = CONFIGS["reduce_f32_2p28p1"]
    sizes = [bench.local_workload(w, r, 8).shape[0] for r in range(8)]
    assert sum(sizes) == 2**28 + 1 and max(sizes) - min(sizes) == 1


def test_reference_arm_reports_unavailable_without_the_package(tmp_path, monkeypatch, capsys):
    import json

    from kernelpilot_b200 import harness

    monkeypatch.setenv("KP_REF_HARNESS", str(tmp_path))
    harness.reference.cache_clear()
    try:
        args = type("A", (), {"workload": "reduce_f32_2p28p1", "steps": 1, "warmup": 3})()
        assert bench.run_reference(args, bench.kdist.Rank(0, 1, 0)) == 0
        line = json.loads(capsys.readouterr().out.strip().splitlines()[-1])
        assert line["impl"] == "reference" and "not installed" in line["unavailable"]
    finally:
        monkeypatch.delenv("KP_REF_HARNESS")
        harness.reference.cache_clear()


@pytest.mark.parametrize("key,shape", [
    ("softmax_f32_4096x4097", (70, 300)), ("gemm_bf16_8192", (80, 48, 64)),
    ("attn_bf16_b8h32s4096d128", (1, 2, 64, 32)), ("vadd_f32_2p26", (5000,)),
    ("layernorm_f32_8192x8192", (70, 200)), ("reduce_f32_2p28p1", (10001,))])
def test_spot_check_passes_a_correct_output_and_catches_a_wrong_one(key, shape):
    import dataclasses

    import torch

    w = dataclasses.replace(CONFIGS[key], shape=shape)
    inputs = w.make_inputs(shape, w.dtype, torch.device("cpu"), 0)
    out = w.spec.baseline(*inputs)
    res = bench.spot_check(w, inputs, out)
    assert res["ok"], res
    bad = out.clone()
    bad.reshape(-1)[0] += 1.0
    assert not bench.spot_check(w, inputs, bad)["ok"]


def test_cpu_baseline_names_its_cores_and_model():
    # the reference's CPU path on a small vector: the record carries what it ran on
    import bench
    w = bench.CONFIGS["reduce_f32_2p28p1"]
    rec = bench.time_cpu(w, reps=1, budget_s=1.0)
    assert rec["cores"] >= 1 and rec["kind"] in ("reference", "port")
    assert isinstance(rec["cpu_model"], str) and rec["cpu_model"]
    assert rec["value"] > 0 and rec["unit"] == "TB/s"


def _flush_worker(rank, world, port, q):
    import os
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port), RANK=str(rank),
                      WORLD_SIZE=str(world), LOCAL_RANK=str(rank))
    try:
        import torch
        import torch.distributed as dist

        import bench
        from kernelpilot_b200 import dist as kdist
        kdist.init(backend="gloo", timeout_s=30)
        bench.L2_BYTES = 1000  # shards of 1996 and 2004 bytes straddle 2 x L2
        x = torch.zeros(499 if rank == 0 else 501)
        q.put((rank, bench.decide_flush((x,), world)))
        dist.destroy_process_group()
    except Exception as e:  # reported to the parent, which fails the test
        q.put((rank, repr(e)))


def test_flush_decision_is_the_same_on_every_rank():
    # a rank-local decision could send one rank into the post-flush collective alone
    import socket

    import torch.multiprocessing as mp
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        port = s.getsockname()[1]
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    procs = [ctx.Process(target=_flush_worker, args=(r, 2, port, q)) for r in range(2)]
    for p in procs:
        p.start()
    got = dict(q.get(timeout=120) for _ in procs)
    for p in procs:
        p.join(timeout=60)
    assert got[0] is False and got[1] is False, got  # the larger shard decides


def test_clock_summary_keeps_the_samples_of_the_timed_window():
    import datetime

    import bench

    def line(t, mhz, power_cap="Not Active"):
        stamp = datetime.datetime.fromtimestamp(t).strftime("%Y/%m/%d %H:%M:%S.%f")[:-3]
        return (f"{stamp}, 0, {mhz}, 1965, 700.0, 0x0, Not Active, Not Active, Not Active, "
                f"{power_cap}")

    t0 = 1_800_000_000.0
    c = bench.ClockSampler(0)
    c.out = "\n".join([line(t0 - 0.2, 1200), line(t0 + 0.05, 1965),
                       line(t0 + 0.10, 1900, "Active"), line(t0 + 0.6, 1200)])
    c.load(t0, t0 + 0.2)
    got = c.summary()
    assert got["samples"] == 2 and got["samples_total"] == 4
    assert got["sm_mhz_min"] == 1900 and got["sm_max_mhz"] == 1965
    assert got["reasons"] == ["sw_power_cap"]
    # a window shorter than the sampling period keeps the nearest sample
    c.load(t0 + 0.55, t0 + 0.56)
    assert c.summary()["samples"] == 1 and c.summary()["sm_mhz"] == 1200
    # no window: every sample
    c.window = None
    assert c.summary()["samples"] == 4

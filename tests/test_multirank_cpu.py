"""World-size-2 gloo tests (CPU) of the multi-rank plumbing bench.py uses on
N GPUs: barrier and the max-over-ranks reduction of the timed region."""

import os
import sys

import pytest
import torch.multiprocessing as mp

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))


def _worker(rank, world, port, q):
    import torch.distributed as dist
    sys.path.insert(0, ROOT)
    import bench
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
    dist.init_process_group("gloo", rank=rank, world_size=world)
    try:
        bench.barrier(dist)
        got = bench.max_over_ranks(dist, 10.0 + rank)  # rank 1 is the slow one
        q.put((rank, got))
    finally:
        dist.destroy_process_group()


def test_max_over_ranks_gloo_world2():
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = 29500 + (os.getpid() % 1000)
    procs = [ctx.Process(target=_worker, args=(r, 2, port, q)) for r in range(2)]
    for p in procs:
        p.start()
    for p in procs:
        p.join(timeout=120)
        assert p.exitcode == 0
    res = dict(q.get(timeout=10) for _ in range(2))
    assert res == {0: 11.0, 1: 11.0}


def test_single_process_reduction_is_identity():
    sys.path.insert(0, ROOT)
    import bench
    assert bench.max_over_ranks(None, 3.5) == 3.5


def test_weak_scaling_value_definition():
    sys.path.insert(0, ROOT)
    import bench
    flops = sum(bench.direct_flops(128, C, C, H) for _, C, H in bench.LAYERS)
    assert flops == pytest.approx(4 * 2 * 128 * 9 * (64 * 64 * 56 * 56))


def test_roofline_picks_the_largest_share_and_reports_traffic():
    sys.path.insert(0, ROOT)
    import bench
    peaks = {"hbm_gbs": 6500.0, "bf16_tflops": 1600.0, "source": "measured"}
    stages = []
    for layer, _, _ in bench.LAYERS:
        stages += [
            {"layer": layer, "kernel": "input_transform_kernel", "ms": 0.040, "bytes": 1.0e8,
             "flops": 0.0},
            {"layer": layer, "kernel": "gemm_tc_kernel", "ms": 0.030, "bytes": 1.5e8,
             "flops": 1.0e10},
            {"layer": layer, "kernel": "output_transform_kernel", "ms": 0.020, "bytes": 1.0e8,
             "flops": 0.0},
        ]
    rl = bench.roofline_from_stages(stages, peaks, batch=128)
    assert rl["kernel"] == "input_transform_kernel" and rl["bound"] == "hbm"
    assert rl["achieved"] == pytest.approx(1.0e8 / 0.040e-3 / 1e9)
    assert rl["frac"] == pytest.approx(rl["achieved"] / 6500.0)
    assert sum(rl["shares"].values()) == pytest.approx(1.0)
    # ncu DRAM bytes per launch, averaged over the layers and scaled by batch.
    t128 = rl["traffic"]
    assert t128 > 0
    assert bench.ncu_traffic("input_transform_kernel", 64) == pytest.approx(t128 / 2)
    assert bench.ncu_traffic("no_such_kernel", 128) is None

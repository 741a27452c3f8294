"""Multi-process host logic of bench.py on CPU: two gloo ranks.

The forward shards by batch with no collective on the data path; the only
cross-rank steps are the barriers and the max-over-ranks reduction of the
event-timed durations.  These tests run that logic on two CPU processes.
"""

import os
import socket
import sys

import pytest
import torch
import torch.distributed as dist
import torch.multiprocessing as mp

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))


def _free_port():
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _worker(rank, ws, port, out):
    sys.path.insert(0, ROOT)
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port), RANK=str(rank), WORLD_SIZE=str(ws),
                      LOCAL_RANK=str(rank))
    import datetime
    import bench
    dist.init_process_group("gloo", rank=rank, world_size=ws, timeout=datetime.timedelta(seconds=60))
    try:
        got_ws, got_rank, got_local = bench.dist_env()
        # the durations differ per rank; every rank must see the largest
        mx = bench.max_over_ranks(10.0 + 5.0 * rank, torch.device("cpu"))
        # each rank's first input set is its own shard
        src, tgt, _ = bench.make_inputs(2, bench.shard_seed(rank, 0))
        digest = torch.stack([src.sum(), tgt.double().sum().float()])
        gathered = [torch.zeros(2) for _ in range(ws)]
        dist.all_gather(gathered, digest)
        dist.barrier()
        out[rank] = (got_ws, got_rank, got_local, mx, [g.tolist() for g in gathered])
    finally:
        dist.destroy_process_group()


def test_two_gloo_ranks_max_and_distinct_shards():
    ws = 2
    port = _free_port()
    with mp.Manager() as mgr:
        out = mgr.dict()
        mp.start_processes(_worker, args=(ws, port, out), nprocs=ws, join=True, start_method="spawn")
        res = dict(out)
    assert sorted(res) == [0, 1]
    for rank, (got_ws, got_rank, got_local, mx, gathered) in res.items():
        assert (got_ws, got_rank, got_local) == (ws, rank, rank)
        assert mx == 15.0
        assert gathered[0] != gathered[1]  # the two ranks drew different images


def test_max_over_ranks_without_a_group():
    sys.path.insert(0, ROOT)
    import bench
    assert not dist.is_initialized()
    assert bench.max_over_ranks(3.5, torch.device("cpu")) == 3.5


@pytest.mark.parametrize("rank", [1])
def test_reference_arm_other_ranks_do_no_work(rank, capsys):
    sys.path.insert(0, ROOT)
    import bench
    ns = type("A", (), dict(steps=1, warmup=0))()
    bench.run_reference(ns, 2, rank)
    assert capsys.readouterr().out == ""


def _dp_worker(rank, ws, port, out):
    sys.path.insert(0, ROOT)
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
    import datetime
    from spikingtransformer_b200.dp import BucketedGradReducer
    dist.init_process_group("gloo", rank=rank, world_size=ws, timeout=datetime.timedelta(seconds=60))
    try:
        results = []
        for mode in ("ddp", "buckets_fp32", "buckets_bf16"):
            torch.manual_seed(0)  # same initial weights on every rank
            model = torch.nn.Sequential(torch.nn.Linear(12, 16), torch.nn.Tanh(), torch.nn.Linear(16, 16),
                                        torch.nn.Tanh(), torch.nn.Linear(16, 3))
            unused = torch.nn.Parameter(torch.zeros(5))  # never receives a gradient
            params = list(model.parameters()) + [unused]
            net, reducer = model, None
            if mode == "ddp":
                net = torch.nn.parallel.DistributedDataParallel(model)
            else:
                # buckets of about 50 elements: several per backward
                reducer = BucketedGradReducer(params, bucket_elems=50,
                                              comm_dtype=torch.float32 if mode == "buckets_fp32" else torch.bfloat16)
                assert len(reducer.buckets) >= 3
            # plain SGD keeps the update linear in the gradient, so the bf16
            # rounding of the buckets shows at its own size
            opt = torch.optim.SGD(model.parameters(), lr=0.1)
            for step in range(3):
                g = torch.Generator().manual_seed(100 * rank + step)  # each rank its own batch
                x, y = torch.randn(8, 12, generator=g), torch.randn(8, 3, generator=g)
                if reducer is not None:
                    reducer.begin()
                else:
                    opt.zero_grad(set_to_none=True)
                torch.nn.functional.mse_loss(net(x), y).backward()
                if reducer is not None:
                    reducer.finish()
                opt.step()
            if reducer is not None:
                # the gradients are still the views the optimizer read
                assert all(p.grad.data_ptr() >= reducer.flat.data_ptr() for p in model.parameters())
                assert float(unused.grad.abs().sum()) == 0.0
                reducer.remove()
            results.append(torch.cat([p.detach().reshape(-1) for p in model.parameters()]).tolist())
        out[rank] = results
    finally:
        dist.destroy_process_group()


def test_bucketed_gradient_reducer_matches_ddp():
    """The training bench's multi-GPU step (gradients as views into one flat
    buffer, buckets all-reduced as the backward completes them, divided by the
    world size) updates the weights as DistributedDataParallel does: to fp32
    rounding with fp32 buckets, to bf16 rounding with the bf16 buckets the
    benchmark sends; and identically on every rank, including a parameter that
    receives no gradient."""
    ws = 2
    port = _free_port()
    with mp.Manager() as mgr:
        out = mgr.dict()
        mp.start_processes(_dp_worker, args=(ws, port, out), nprocs=ws, join=True, start_method="spawn")
        res = dict(out)
    ddp0, f32_0, bf16_0 = (torch.tensor(v) for v in res[0])
    ddp1, f32_1, bf16_1 = (torch.tensor(v) for v in res[1])
    assert torch.equal(f32_0, f32_1) and torch.equal(bf16_0, bf16_1) and torch.equal(ddp0, ddp1)
    assert torch.allclose(f32_0, ddp0, rtol=1e-5, atol=1e-6)
    assert torch.allclose(bf16_0, ddp0, rtol=0, atol=1e-3)
    assert not torch.equal(bf16_0, f32_0)


def test_clock_sampler_keeps_only_the_timed_window():
    """bench.ClockSampler: samples taken before begin() or after end() (the
    warm-up, the sampler's start-up) are left out of the summary; the median
    SM clock, the maximum and the throttle reasons come from the window only."""
    sys.path.insert(0, ROOT)
    import bench
    clk = bench.ClockSampler(0)
    row = lambda mhz, cap: [str(mhz), "1965", "500.0", "0x0", "Not Active", "Not Active", "Not Active", cap]  # noqa
    clk.samples = [(0.0, row(1965, "Not Active")),     # before the window
                   (1.0, row(1600, "Active")),
                   (1.1, row(1650, "Active")),
                   (1.2, row(1700, "Not Active")),
                   (5.0, row(900, "Not Active"))]       # after it
    clk.t0, clk.t1 = 0.5, 2.0
    s = clk.summary()
    assert s["samples"] == 3
    assert s["sm_mhz"] == 1650.0 and s["sm_max_mhz"] == 1965.0
    assert s["reasons"] == ["sw_power_cap"]
    clk.t0, clk.t1 = 3.0, 4.0  # a window with no sample in it
    assert clk.summary()["reasons"] == ["unavailable"]

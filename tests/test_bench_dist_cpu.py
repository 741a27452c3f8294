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

"""The benchmark's multi-rank logic on CPU with two gloo ranks: every rank prefills its own
requests (weak scaling, no collective on the data path) and the reported times are the
maximum over ranks."""
import os
import socket
import sys
from pathlib import Path

import pytest
import torch
import torch.distributed as dist
import torch.multiprocessing as mp

ROOT = Path(__file__).resolve().parents[1]


def _free_port():
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _rank_main(rank, world, port, out):
    sys.path.insert(0, str(ROOT))
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
    dist.init_process_group("gloo", rank=rank, world_size=world)
    try:
        import bench
        prefill, decode = bench.make_inputs(1000, 4, 16, rank)
        # rank-dependent fake per-call times (ms); rank 1 is the slow replica
        rec = {"p": [10.0 + rank, 11.0 + rank, 12.0 + rank], "d": [1.0, 1.5 + rank, 2.0],
               "p_wall": [20.0, 21.0 + 3 * rank, 22.0], "d_wall": [3.0, 3.0, 3.0]}
        times = bench.reduce_step_times(rec, world, "cpu")
        out[rank] = (prefill, decode, times)
    finally:
        dist.destroy_process_group()


def test_two_rank_sharding_and_max_times():
    world = 2
    port = _free_port()
    with mp.Manager() as mgr:
        out = mgr.dict()
        mp.spawn(_rank_main, args=(world, port, out), nprocs=world, join=True)
        res = dict(out)
    (p0, d0, t0), (p1, d1, t1) = res[0], res[1]
    # each replica gets its own requests of the same shape
    assert [len(r) for r in p0] == [len(r) for r in p1] == [16] * 4
    assert p0 != p1 and d0 != d1
    # every rank reports the maximum over ranks of its medians (rank 1 is slower):
    # prefill 12 vs 11, decode 2.0 vs 1.5, step 14.0 vs 12.5, end to end 25 vs 24
    assert t0 == t1
    step_ms, e2e_ms, prefill_ms, decode_ms = t0
    assert prefill_ms == pytest.approx(12.0) and decode_ms == pytest.approx(2.0)
    assert step_ms == pytest.approx(14.0) and e2e_ms == pytest.approx(25.0)

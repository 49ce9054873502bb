"""Multi-GPU sharding of the bench, run as two gloo ranks on the CPU: each rank owns a disjoint set
of streams and its own language draw, and the step time reported is the max over ranks."""
import os
import socket
import sys
import types

import pytest
import torch.distributed as dist
import torch.multiprocessing as mp

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))


def _free_port():
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _rank(rank, world, port, out):
    import datetime
    sys.path.insert(0, ROOT)
    import bench
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
    dist.init_process_group("gloo", rank=rank, world_size=world, timeout=datetime.timedelta(seconds=60))
    try:
        a = types.SimpleNamespace(streams=256)
        seeds = bench.stream_seeds(a, rank)
        langs = bench.languages(a, rank)
        got = [None] * world
        dist.all_gather_object(got, (seeds, langs))
        t = bench.max_over_ranks(dist, 1.5 + rank, "cpu")
        if rank == 0:
            with open(out, "w") as f:
                f.write(repr((got, t)))
    finally:
        dist.destroy_process_group()


def test_streams_shard_disjointly_and_time_is_max_over_ranks(tmp_path):
    out = str(tmp_path / "r.txt")
    mp.start_processes(_rank, args=(2, _free_port(), out), nprocs=2, join=True, start_method="spawn")
    import ast
    got, t = ast.literal_eval(open(out).read())
    (s0, l0), (s1, l1) = got
    assert len(s0) == len(s1) == 256 and not set(s0) & set(s1)
    assert l0 != l1 and len(l0) == 256
    assert t == pytest.approx(2.5)

"""One process per GPU over NCCL: each rank runs the engine on its contiguous
shard of a batch on its own GPU (rosenna_b200.ranks.use_model_shard with the
default runner), the shards are gathered over NCCL, and the joined batch must
match the fp64 oracle within the limits of oracle/parity.py (max abs 1e-5; max
rel 1e-4 where |ref| >= 0.1).  Needs two GPUs;
NVLS is off in the children."""
import datetime
import multiprocessing as mp
import os

import numpy as np
import pytest

from oracle import parity
from rosenna_b200 import ranks
from tests.test_ranks import free_port, oracle_runner

pytestmark = pytest.mark.gpu

CASES = [("small_mlp", 100003), ("wide_mlp", 4099), ("lstm", 1001), ("cnn", 257)]


def _nccl_rank(rank, world, port, model_dirs, q):
    import torch
    import torch.distributed as dist

    from rosenna_b200 import api, workloads

    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port), RANK=str(rank), LOCAL_RANK=str(rank),
                      WORLD_SIZE=str(world), NCCL_NVLS_ENABLE="0")
    r, local, w = ranks.env()
    torch.cuda.set_device(local)
    dist.init_process_group("nccl", timeout=datetime.timedelta(seconds=60), device_id=torch.device("cuda", local))
    try:
        api.set_devices([local])
        for name, n in CASES:
            api.initialize(model_dirs[name])
            a, b, local_out = ranks.use_model_shard(workloads.make_inputs(name, n), r, w)
            full = ranks.gather_shards(local_out, n)
            if r == 0:
                q.put((name, n, full))
            api.finalize()
        dist.barrier()
    finally:
        dist.destroy_process_group()


def test_two_ranks_shard_over_nccl(tmp_path):
    import torch

    if torch.cuda.device_count() < 2:
        pytest.skip("needs two GPUs")
    from rosenna_b200 import workloads

    model_dirs = {}
    for name, _ in CASES:
        workloads.write_model(name, str(tmp_path / name))
        model_dirs[name] = str(tmp_path / name)
    world, port = 2, free_port()
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    procs = [ctx.Process(target=_nccl_rank, args=(r, world, port, model_dirs, q)) for r in range(world)]
    for p in procs:
        p.start()
    got = [q.get(timeout=300) for _ in CASES]
    for p in procs:
        p.join(timeout=120)
        assert p.exitcode == 0
    for name, n, full in got:
        want = oracle_runner(model_dirs[name], np.float64, 0)(workloads.make_inputs(name, n), n)
        for x, y in zip(full, want):
            assert x.shape == y.shape
            r = parity.compare(x.astype(np.float64), y)
            assert r["ok"], (name, n, parity.describe(r))

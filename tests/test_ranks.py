"""The one-process-per-GPU front end (rosenna_b200.ranks) on the host.

Shard arithmetic, and two gloo ranks that each evaluate their contiguous
shard, gather the outputs and take the max over ranks of a timing.  On the CPU
the shard runner is the oracle (the host logic is what is tested here; the
engine on each GPU is covered by the parity tests and test_gpu_ranks.py); the
joined batch must equal one oracle run over the whole batch exactly."""
import datetime
import multiprocessing as mp
import os
import socket

import numpy as np
import pytest

from rosenna_b200 import ranks

CASES = [("small_mlp", 7), ("small_mlp", 1), ("small_mlp", 0), ("lstm", 5)]


@pytest.mark.parametrize("world", [1, 2, 3, 8])
@pytest.mark.parametrize("n", [0, 1, 2, 7, 1000, 1001])
def test_shards_tile_the_batch(n, world):
    bounds = [ranks.shard_bounds(n, r, world) for r in range(world)]
    assert bounds[0][0] == 0 and bounds[-1][1] == n
    for (a, b), (c, _) in zip(bounds, bounds[1:]):
        assert b == c
    sizes = [b - a for a, b in bounds]
    assert max(sizes) - min(sizes) <= 1
    assert sizes == sorted(sizes, reverse=True)  # the first n % world ranks take the extra sample


def test_bad_shard_requests():
    for args in [(5, 2, 2), (5, -1, 2), (5, 0, 0), (-1, 0, 1)]:
        with pytest.raises(ValueError):
            ranks.shard_bounds(*args)
    with pytest.raises(ValueError):
        ranks.shard_rows([np.zeros((2, 4)), np.zeros((3, 5))], 0, 2)


def test_env_defaults(monkeypatch):
    for k in ("RANK", "LOCAL_RANK", "WORLD_SIZE"):
        monkeypatch.delenv(k, raising=False)
    assert ranks.env() == (0, 0, 1)
    monkeypatch.setenv("RANK", "3")
    monkeypatch.setenv("LOCAL_RANK", "1")
    monkeypatch.setenv("WORLD_SIZE", "4")
    assert ranks.env() == (3, 1, 4)


def oracle_runner(model_dir, dtype=np.float32, threads=1):
    """use_model over (rows, k) arrays by the oracle (batch-first models)."""
    from oracle.oracle import OracleModel

    m = OracleModel(model_dir)

    def run(xs, k):
        outs = m.run_batched(k, xs, threads=threads)
        return [o.reshape(int(np.prod(s)), k).astype(dtype) for o, s in zip(outs, m.output_shapes)]

    return run


def free_port():
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _gloo_rank(rank, world, port, model_dirs, q):
    import torch.distributed as dist

    from rosenna_b200 import workloads

    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port), RANK=str(rank), LOCAL_RANK=str(rank),
                      WORLD_SIZE=str(world))
    dist.init_process_group("gloo", timeout=datetime.timedelta(seconds=60))
    try:
        r, _, w = ranks.env()
        for name, n in CASES:
            ins = workloads.make_inputs(name, n)  # the same seeded batch on every rank
            a, b, local = ranks.use_model_shard(ins, r, w, run=oracle_runner(model_dirs[name]))
            full = ranks.gather_shards(local, n)
            q.put((r, name, n, a, b, full))
        q.put((r, "max", ranks.max_over_ranks(0.25 + r)))
        q.put((r, "all", ranks.values_over_ranks(0.5 * r)))
    finally:
        dist.destroy_process_group()


def test_two_gloo_ranks_shard_gather_and_time(tmp_path):
    from rosenna_b200 import workloads

    model_dirs = {}
    for name in {c[0] for c in CASES}:
        d = tmp_path / name
        workloads.write_model(name, str(d))
        model_dirs[name] = str(d)
    world, port = 2, free_port()
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    procs = [ctx.Process(target=_gloo_rank, args=(r, world, port, model_dirs, q)) for r in range(world)]
    for p in procs:
        p.start()
    got = [q.get(timeout=240) for _ in range(world * (len(CASES) + 2))]
    for p in procs:
        p.join(timeout=60)
        assert p.exitcode == 0
    for rank in range(world):
        assert [g[2] for g in got if g[0] == rank and g[1] == "max"] == [0.25 + world - 1]
        assert [g[2] for g in got if g[0] == rank and g[1] == "all"] == [[0.5 * r for r in range(world)]]
    for name, n in CASES:
        want = oracle_runner(model_dirs[name])(workloads.make_inputs(name, n), n)
        rows = {g[0]: g for g in got if g[1] == name and g[2] == n}
        assert sorted(rows) == list(range(world))
        assert [rows[r][3:5] for r in range(world)] == [ranks.shard_bounds(n, r, world) for r in range(world)]
        for r in range(world):
            full = rows[r][5]
            assert len(full) == len(want)
            for x, y in zip(full, want):
                assert x.shape == y.shape
                np.testing.assert_array_equal(x, y)

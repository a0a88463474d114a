"""Parity at each workload's full batch (small MLP 1,048,576; wide MLP
4,194,304; LSTM 262,144; CNN 65,536; 2-layer LSTM 1,048,576 samples).

The engine evaluates the whole batch; the fp64 oracle evaluates a fixed subset
of about 4,096 sample indices (oracle/parity.py check_indices: the first and last
128-sample tile, the final sample, both sides of every power-of-two boundary
where calls are split into chunks, the shard boundaries of 2..8 GPUs, and seeded
uniform indices), so the persistent tile loops, 64-bit offsets, chunk splits
and the last partial tile at these sizes are all checked.  Limits: max abs
<= 1e-5 over every checked element and max rel <= 1e-4 where |ref| >= 0.1;
both maxima are printed.  The host-array entry point is checked bit for bit
against the device entry point on the same batch.
"""
import numpy as np
import pytest
import torch

from oracle import parity
from oracle.oracle import OracleModel
from rosenna_b200 import api, workloads

pytestmark = pytest.mark.gpu


@pytest.fixture(autouse=True)
def _device():
    assert torch.cuda.is_available(), "gpu tests need a CUDA device"
    api.set_devices([0])
    yield
    api.finalize()


def oracle_subset(model_dir, ins, idx):
    """The oracle on the samples `idx` of device inputs `ins` ((rows, n) each)."""
    t = torch.from_numpy(idx).to(ins[0].device)
    sub = [x.index_select(1, t).double().cpu().numpy() for x in ins]
    return OracleModel(model_dir).run_batched(len(idx), sub)[0].reshape(-1, len(idx))


@pytest.mark.parametrize("name", list(workloads.WORKLOADS))
def test_full_batch_parity(name, tmp_path):
    w = workloads.WORKLOADS[name]
    n = w.batch
    d = str(tmp_path)
    workloads.write_model(name, d)
    api.initialize(d)
    ins = workloads.make_inputs_torch(name, n, device="cuda", seed_offset=17)
    outs = [torch.full((r, n), float("nan"), dtype=torch.float32, device="cuda") for r in w.output_rows]
    api.use_model_device(n, [x.data_ptr() for x in ins], [o.data_ptr() for o in outs],
                         torch.cuda.current_stream().cuda_stream)
    torch.cuda.synchronize()
    assert api.last_launch_count() > 0
    assert bool(torch.isfinite(outs[0]).all()), f"{name}: non-finite outputs at n={n}"
    idx = parity.check_indices(n, 4096, seed=w.key)
    ref = oracle_subset(d, ins, idx)
    got = outs[0].index_select(1, torch.from_numpy(idx).cuda()).double().cpu().numpy()
    r = parity.compare(got, ref)
    print(f"{name} n={n}, {len(idx)} samples checked: {parity.describe(r)}")
    assert r["ok"], f"{name} n={n}: {parity.describe(r)}"


@pytest.mark.parametrize("name", ["small_mlp", "wide_mlp", "lstm", "cnn"])
def test_full_batch_host_path_matches_device_path(name, tmp_path):
    """rosenna_use_model_f32 (host arrays, chunked over four streams) at the
    full batch gives the device entry point's outputs bit for bit."""
    w = workloads.WORKLOADS[name]
    n = w.batch
    d = str(tmp_path)
    workloads.write_model(name, d)
    api.initialize(d)
    ins = workloads.make_inputs_torch(name, n, device="cuda", seed_offset=23)
    outs = [torch.empty((r, n), dtype=torch.float32, device="cuda") for r in w.output_rows]
    api.use_model_device(n, [x.data_ptr() for x in ins], [o.data_ptr() for o in outs],
                         torch.cuda.current_stream().cuda_stream)
    torch.cuda.synchronize()
    host = api.use_model_rows([x.cpu().numpy() for x in ins])
    for h, o in zip(host, outs):
        assert np.array_equal(h, o.cpu().numpy()), name

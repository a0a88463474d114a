"""The streamed-input tensor-core MLP kernel (mlp_stream_tc_kernel: a first
layer of more than 64 inputs and at most 64 outputs whose inputs and weights
are streamed by TMA, 32-deep partials added in fp32 registers, later layers at
most 64 wide with resident weights, two tiles per CTA) on chain shapes around
its limits: first layers of 65 to 1000 inputs (K-chunks of 32 with a ragged
last one), widths 16 to 64, one and several later layers, every activation, a
CUDA-core last layer of 8 or 16 padded columns and none, batches with partial
tiles and an odd tile left over for one of the two tile groups.  Batches whose
pitch is a multiple of 4 samples take the tensor-map path; the others fall back
to the dual-tile kernel (both compared).  Compared with the fp64 oracle within
the limits of oracle/parity.py (max abs 1e-5; max rel 1e-4 where
|ref| >= 0.1)."""
import numpy as np
import pytest
import torch
from torch import nn

from oracle.oracle import OracleModel
from rosenna_b200 import api, writer
from tests.test_gpu_parity import assert_close

pytestmark = pytest.mark.gpu

ACTS = {"relu": nn.ReLU, "tanh": nn.Tanh, "sigmoid": nn.Sigmoid, "none": None}

CASES = {  # widths, activation per layer
    "cnn_head": ([784, 64, 10], ["relu", "none"]),
    "k65_tail8": ([65, 64, 5], ["tanh", "none"]),
    "k100_deep": ([100, 48, 64, 32, 12], ["sigmoid", "sigmoid", "sigmoid", "none"]),
    "k1000_no_tail": ([1000, 32, 40], ["relu", "relu"]),
    "k300_one_layer": ([300, 16], ["tanh"]),
}


def build(case, d):
    widths, acts = CASES[case]
    torch.manual_seed(sum(widths) + 5 * len(widths))
    mods = []
    for i, (k, m) in enumerate(zip(widths[:-1], widths[1:])):
        lin = nn.Linear(k, m)
        mods.append(lin)
        if ACTS[acts[i]] is not None:
            mods.append(ACTS[acts[i]]())
    writer.write_model_files(writer.export_sequential(mods, [1, widths[0]]), d)
    return widths


@pytest.fixture(autouse=True)
def _device(monkeypatch):
    assert torch.cuda.is_available(), "gpu tests need a CUDA device"
    monkeypatch.setenv("ROSENNA_MLP_PATH", "tc")
    api.set_devices([0])
    yield
    api.finalize()


@pytest.mark.parametrize("case", sorted(CASES))
def test_stream_chain_shapes(case, tmp_path):
    d = str(tmp_path)
    widths = build(case, d)
    api.initialize(d)
    names = [k for k, _ in api.step_info()]
    assert "mlp_stream_tc_kernel" in names, (names, api.plan_description())
    oracle = OracleModel(d)
    rng = np.random.default_rng(len(case) * 13)
    # 1000, 4096, 50000: pitch a multiple of 4 (tensor-map path); 129, 4097: the fallback
    for n in (129, 1000, 4096, 4097, 50000):
        x = rng.uniform(-1.5, 1.5, size=(widths[0], n)).astype(np.float32)
        out = api.use_model_rows([x])[0]
        ref = oracle.run_batched(n, [x])[0]
        assert_close(out, ref.reshape(out.shape), f"{case} n={n}")


def test_stream_device_path_full_tiles(tmp_path):
    """Device arrays (16-byte aligned, pitch = batch) at a batch of whole tiles."""
    d = str(tmp_path)
    widths = build("cnn_head", d)
    api.initialize(d)
    n = 65536
    rng = np.random.default_rng(7)
    x = rng.uniform(-1.0, 1.0, size=(widths[0], n)).astype(np.float32)
    xd = torch.from_numpy(x).cuda()
    yd = torch.empty(widths[-1], n, device="cuda")
    api.use_model_device(n, [xd.data_ptr()], [yd.data_ptr()])
    torch.cuda.synchronize()
    idx = np.concatenate([np.arange(0, 300), np.arange(n - 300, n), rng.integers(0, n, 2000)])
    ref = OracleModel(d).run_batched(len(idx), [x[:, idx]])[0]
    assert_close(yd.cpu().numpy()[:, idx], ref.reshape(widths[-1], len(idx)), "cnn_head device n=65536")


def test_stream_off_switch(tmp_path, monkeypatch):
    """ROSENNA_TC_STREAM=0 keeps an eligible chain on the dual-tile kernel."""
    monkeypatch.setenv("ROSENNA_TC_STREAM", "0")
    build("cnn_head", str(tmp_path))
    api.initialize(str(tmp_path))
    assert "mlp_stream_tc_kernel" not in [k for k, _ in api.step_info()]

"""The resident-weight tensor-core MLP kernel (mlp_narrow_tc_kernel: every
layer at most 64 wide with at most 64 inputs, weights resident in shared
memory, the A operand in TMEM, two tiles per CTA) on chain shapes around its
limits: one and many layers, widths 16/48/64 (and N between multiples of 16),
inputs from 1 to 64, each activation, a CUDA-core last layer of 8 or 16
padded columns and none, batches with partial 128-sample tiles and an odd
tile left over for one of the two tile groups.  Compared with the fp64 oracle
within the limits of oracle/parity.py (max abs 1e-5; max rel 1e-4 where
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
    "small_mlp": ([10, 64, 64, 64, 5], ["tanh", "tanh", "tanh", "none"]),
    "relu_tail16": ([33, 48, 64, 12], ["relu", "relu", "none"]),
    "sigmoid_no_tail": ([20, 64, 32, 40], ["sigmoid", "sigmoid", "sigmoid"]),
    "linear_no_tail": ([64, 64, 17], ["none", "none"]),
    "one_layer": ([5, 16], ["relu"]),
    "deep": ([8] + [32] * 7 + [3], ["tanh"] * 7 + ["none"]),
    "one_input": ([1, 50, 7], ["tanh", "sigmoid"]),
}


def build(case, d):
    widths, acts = CASES[case]
    torch.manual_seed(sum(widths) + 3 * len(widths))
    mods = []
    for i, (k, m) in enumerate(zip(widths[:-1], widths[1:])):
        mods.append(nn.Linear(k, m))
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
def test_narrow_chain_shapes(case, tmp_path):
    d = str(tmp_path)
    widths = build(case, d)
    api.initialize(d)
    names = [k for k, _ in api.step_info()]
    assert "mlp_narrow_tc_kernel" in names, (names, api.plan_description())
    oracle = OracleModel(d)
    rng = np.random.default_rng(len(case) * 11)
    # 50001 samples: 391 tiles, an odd tile left for one group on some CTAs
    for n in (1, 129, 1000, 4097, 50001):
        x = rng.uniform(-1.5, 1.5, size=(widths[0], n)).astype(np.float32)
        out = api.use_model_rows([x])[0]
        ref = oracle.run_batched(n, [x])[0]
        assert_close(out, ref.reshape(out.shape), f"{case} n={n}")


def test_narrow_off_switch(tmp_path, monkeypatch):
    """ROSENNA_TC_NARROW=0 keeps an eligible chain on the dual-tile kernel."""
    monkeypatch.setenv("ROSENNA_TC_NARROW", "0")
    build("small_mlp", str(tmp_path))
    api.initialize(str(tmp_path))
    assert "mlp_narrow_tc_kernel" not in [k for k, _ in api.step_info()]

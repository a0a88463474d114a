"""Tensor-core MLP kernels on many chain shapes: widths around the 16/32/128
boundaries of their tiling (N multiple of 16 per half, K chunks of 32, two
column halves of 128), depths up to the 8-layer limit, every activation, the
CUDA-core tail on and off, batches that leave partial 128-sample tiles (and,
for chains no wider than 128, an odd tile left over for one column group).
Chains no wider than 128 run both on the kernel that gives each column group
a tile of its own (the default) and on the one that splits a tile's columns.
Compared with the fp64 oracle within the limits of oracle/parity.py
(max abs 1e-5; max rel 1e-4 where |ref| >= 0.1)."""
import os

import numpy as np
import pytest
import torch
from torch import nn

from oracle.oracle import OracleModel
from rosenna_b200 import api, writer
from tests.test_gpu_parity import assert_close

pytestmark = pytest.mark.gpu

ACTS = {"relu": nn.ReLU, "tanh": nn.Tanh, "sigmoid": nn.Sigmoid, "none": None}

CASES = {
    "wide_relu": ([10, 256, 256, 8], ["relu", "relu", "none"]),
    "odd_tanh": ([33, 129, 200, 5], ["tanh", "tanh", "none"]),
    "sigmoid_no_tail": ([100, 128, 128, 128, 17], ["sigmoid", "sigmoid", "sigmoid", "none"]),
    "mixed": ([7, 64, 256, 64, 256, 1], ["relu", "tanh", "sigmoid", "relu", "tanh"]),
    "eight_layers": ([256] * 8 + [16], ["relu"] * 7 + ["none"]),
    "long_input": ([300, 144, 96, 12], ["tanh", "relu", "sigmoid"]),
    "two_cols_in_half_1": ([5, 130, 3], ["relu", "none"]),
    "all_narrow": ([16, 16, 16, 16], ["tanh", "tanh", "none"]),
    "ragged": ([20, 50, 70, 9], ["sigmoid", "relu", "none"]),
    "narrow_deep": ([40] + [96] * 7 + [12], ["relu"] * 7 + ["none"]),
    "narrow_long_input": ([300, 96, 64, 3], ["tanh", "sigmoid", "none"]),
}


def build(case, d):
    widths, acts = CASES[case]
    torch.manual_seed(sum(widths) + len(widths))
    mods = []
    for i, (k, m) in enumerate(zip(widths[:-1], widths[1:])):
        mods.append(nn.Linear(k, m))
        if ACTS[acts[i]] is not None:
            mods.append(ACTS[acts[i]]())
    g = writer.export_sequential(mods, [1, widths[0]])
    writer.write_model_files(g, d)
    return widths


@pytest.fixture(autouse=True)
def _device():
    assert torch.cuda.is_available(), "gpu tests need a CUDA device"
    api.set_devices([0])
    yield


def narrow(case):
    return max(CASES[case][0][1:]) <= 128


@pytest.mark.parametrize("tail", ["1", "0"])
@pytest.mark.parametrize("case,dual", [(c, d) for c in sorted(CASES) for d in (("1", "0") if narrow(c) else ("1",))])
def test_tc_chain_shapes(case, tail, dual, tmp_path, monkeypatch):
    monkeypatch.setenv("ROSENNA_MLP_PATH", "tc")
    monkeypatch.setenv("ROSENNA_TC_TAIL", tail)
    monkeypatch.setenv("ROSENNA_TC_DUAL", dual)
    monkeypatch.setenv("ROSENNA_TC_NARROW", "0")  # the resident-weight kernel: test_gpu_narrow.py
    d = str(tmp_path)
    widths = build(case, d)
    api.initialize(d)
    assert "mlp_tc" in api.plan_description(), api.plan_description()
    oracle = OracleModel(d)
    rng = np.random.default_rng(len(case) * 7 + int(tail))
    # 50001 samples: 391 tiles, more than one pair of tiles for some CTAs
    for n in (1, 129, 1000, 4097) + ((50001,) if narrow(case) and dual == "1" else ()):
        x = rng.uniform(-1.5, 1.5, size=(widths[0], n)).astype(np.float32)
        out = api.use_model_rows([x])[0]
        ref = oracle.run_batched(n, [x])[0]
        assert_close(out, ref.reshape(out.shape), f"{case} tail={tail} dual={dual} n={n}")

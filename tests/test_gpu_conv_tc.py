"""The tensor-core convolution (conv_tc_kernel: implicit GEMM on tcgen05,
3xTF32, fused with ReLU and the 2x2 pool) against the fp64 oracle, within the
limits of oracle/parity.py (max abs 1e-5; max rel 1e-4 where |ref| >= 0.1).

Covers the shapes the kernel takes: a single input channel (K-steps of 8
patch positions; with at most 8 output channels two pooled windows per block)
and 2..8 input channels (K-steps of one position's 8 channels), 1..16 output
channels, padding 0..2, max and average pooling, batches with partial tiles,
and the
CNN workload and golden CNNs with every eligible conv forced onto it.  (Images
are square: the plan rejects non-square pooled outputs, whose columns the
reference writes with MODULO(., rows).)"""
import numpy as np
import pytest
import torch
import torch.nn as nn

from oracle.oracle import OracleModel
from rosenna_b200 import api, workloads, writer
from tests import goldens
from tests.test_gpu_parity import assert_close

pytestmark = pytest.mark.gpu


@pytest.fixture(autouse=True)
def _device(monkeypatch):
    assert torch.cuda.is_available(), "gpu tests need a CUDA device"
    monkeypatch.setenv("ROSENNA_CONV_PATH", "tc")
    api.set_devices([0])
    yield
    api.finalize()


SHAPES = [  # (C, OC, H, W, pad, pool)
    (8, 16, 14, 14, 1, "avg"), (8, 16, 14, 14, 1, "max"), (3, 5, 10, 10, 1, "max"), (1, 8, 12, 12, 1, "max"),
    (8, 9, 8, 8, 0, "avg"), (5, 16, 6, 6, 2, "avg"), (4, 6, 12, 12, 1, "max"), (8, 1, 16, 16, 1, "avg"),
    (1, 8, 28, 28, 1, "max"), (1, 3, 10, 10, 2, "avg"), (1, 12, 6, 6, 1, "max"), (1, 16, 14, 14, 0, "avg"),
]


@pytest.mark.parametrize("C,OC,H,W,pad,pool", SHAPES)
def test_conv_tc_shapes(C, OC, H, W, pad, pool, tmp_path):
    torch.manual_seed(C * 100 + OC * 10 + H + pad)
    conv = nn.Conv2d(C, OC, 3, padding=pad)
    nn.init.uniform_(conv.weight, -0.5, 0.5)
    mods = [conv, nn.ReLU(), (nn.MaxPool2d if pool == "max" else nn.AvgPool2d)(2, 2)]
    g = writer.export_sequential(mods, [1, C, H, W])
    writer.write_model_files(g, str(tmp_path))
    api.initialize(str(tmp_path))
    assert "conv_tc" in api.plan_description(), api.plan_description()
    for n in (1, 129, 1000):
        ins = [np.random.default_rng(n + C).uniform(-1, 1, size=(C * H * W, n)).astype(np.float32)]
        out = api.use_model_rows(ins)[0]
        assert api.last_launch_count() > 0
        ref = OracleModel(str(tmp_path)).run_batched(n, ins)[0]
        assert_close(out, ref.reshape(out.shape), f"C={C} OC={OC} {H}x{W} pad={pad} {pool} n={n}")


def test_cnn_workload_on_conv_tc(tmp_path):
    workloads.write_model("cnn", str(tmp_path))
    api.initialize(str(tmp_path))
    desc = api.plan_description()
    assert desc.count("conv_tc") == 2, desc  # conv1 (one channel) and conv2
    for n in (1, 37, 1000, 4099):
        ins = workloads.make_inputs("cnn", n, seed_offset=31 + n)
        out = api.use_model_rows(ins)[0]
        ref = OracleModel(str(tmp_path)).run_batched(n, ins)[0]
        assert_close(out, ref.reshape(out.shape), f"cnn conv_tc n={n}")


@pytest.mark.parametrize("case", ["cnn_small", "add_conv"])
def test_golden_convs_on_conv_tc(case):
    api.initialize(goldens.case_dir(case))
    assert "conv_tc" in api.plan_description()
    out = api.use_model(goldens.inputs(case), n=1)[0]
    assert_close(out, goldens.golden(case), f"{case} conv_tc")

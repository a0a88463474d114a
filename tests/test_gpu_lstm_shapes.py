"""The CUDA-core LSTM kernel on many layer shapes: the instantiation with the
hidden size 32 and 128-sample tiles fixed at compile time (two CTAs per SM),
the runtime-shaped one at two CTAs per SM (other hidden sizes, hidden sizes
below their padding) and at one CTA per SM (a wide input that leaves room for
one tile), with every output the reference emits (h_n through a head, the
whole sequence Y, c_n), zero or given initial state, one to seventeen time
steps, two stacked layers, and batches that leave partial tiles.  Compared
with the fp64 oracle within the limits of oracle/parity.py
(max abs 1e-5; max rel 1e-4 where |ref| >= 0.1)."""
import numpy as np
import pytest
import torch
from torch import nn

from oracle.oracle import OracleModel
from rosenna_b200 import api, writer
from tests.test_gpu_parity import assert_close

pytestmark = pytest.mark.gpu

# name: (input size, hidden sizes of the stacked layers, time steps, output, initial state given)
CASES = {
    "h32_i8_hn": (8, [32], 7, "hn_head", False),
    "h32_i1_y": (1, [32], 5, "y", True),
    "h32_i20_cn": (20, [32], 9, "cn", True),
    "h32_t1_y": (8, [32], 1, "y", True),
    "h32_t17_hn": (3, [32], 17, "hn_head", True),
    "h32_i100_hn": (100, [32], 3, "hn_head", True),
    "h30_i8_y": (8, [30], 4, "y", True),
    "h16_i8_y": (8, [16], 6, "y", True),
    "h5_i3_cn": (3, [5], 8, "cn", True),
    "h48_i8_cn": (8, [48], 5, "cn", True),
    "h32x2_hn": (8, [32, 32], 6, "hn_head", True),
}


def build(case, d):
    I, hs, T, mode, state = CASES[case]
    torch.manual_seed(len(case) * 31 + I)
    lstms, k = [], I
    for h in hs:
        lstms.append(nn.LSTM(k, h, 1, batch_first=True))
        k = h
    head = [nn.Linear(hs[-1], 3), nn.Tanh()] if mode == "hn_head" else []
    g = writer.export_lstm(lstms, head, batch=1, seq_len=T, mode=mode, with_state=state)
    writer.write_model_files(g, d)


@pytest.fixture(autouse=True)
def _device():
    assert torch.cuda.is_available(), "gpu tests need a CUDA device"
    api.set_devices([0])
    yield
    api.finalize()


@pytest.mark.parametrize("case", sorted(CASES))
def test_ffma_lstm_shapes(case, tmp_path, monkeypatch):
    monkeypatch.setenv("ROSENNA_LSTM_PATH", "ffma")
    d = str(tmp_path)
    build(case, d)
    api.initialize(d)
    plan = api.plan_description()
    assert "lstm b" in plan and "lstm_tc" not in plan, plan
    oracle = OracleModel(d)
    rows = [int(np.prod(s)) // s[b] for s, b in api.input_specs()]
    rng = np.random.default_rng(len(case))
    for n in (1, 129, 1000, 4097):
        # the sequence input first, then h0/c0 pairs (smaller values, as a state)
        ins = [rng.uniform(-1.5, 1.5, size=(r, n)).astype(np.float32) if i == 0
               else rng.uniform(-0.5, 0.5, size=(r, n)).astype(np.float32) for i, r in enumerate(rows)]
        out = api.use_model_rows(ins)[0]
        ref = oracle.run_batched(n, ins)[0]
        assert_close(out, ref.reshape(out.shape), f"{case} n={n}")


@pytest.mark.parametrize("case", sorted(c for c, v in CASES.items() if v[0] <= 32 and max(v[1]) <= 32))
def test_dual_tile_lstm_shapes(case, tmp_path, monkeypatch):
    """The dual-tile tensor-core kernel (I <= 32, H <= 32: each column group a
    tile of its own), the default for these shapes."""
    monkeypatch.delenv("ROSENNA_LSTM_PATH", raising=False)
    d = str(tmp_path)
    build(case, d)
    api.initialize(d)
    plan = api.plan_description()
    assert "lstm_tc_dual" in plan, plan
    oracle = OracleModel(d)
    rows = [int(np.prod(s)) // s[b] for s, b in api.input_specs()]
    rng = np.random.default_rng(len(case) + 1)
    for n in (1, 129, 1000, 4097):
        ins = [rng.uniform(-1.5, 1.5, size=(r, n)).astype(np.float32) if i == 0
               else rng.uniform(-0.5, 0.5, size=(r, n)).astype(np.float32) for i, r in enumerate(rows)]
        out = api.use_model_rows(ins)[0]
        ref = oracle.run_batched(n, ins)[0]
        assert_close(out, ref.reshape(out.shape), f"{case} n={n}")


# the fused two-layer tensor-core kernel: hidden size 64 in both layers,
# layer-1 input width <= 32
FUSED = {
    "x2_i12_t7_hn": (12, 7, "hn_head", True),
    "x2_i1_t3_y": (1, 3, "y", True),
    "x2_i32_t2_cn": (32, 2, "cn", True),
    "x2_i5_t1_hn": (5, 1, "hn_head", False),
    "x2_i20_t9_y": (20, 9, "y", False),
}


@pytest.mark.parametrize("case", sorted(FUSED))
def test_fused_two_layer_lstm_shapes(case, tmp_path):
    I, T, mode, state = FUSED[case]
    torch.manual_seed(len(case) * 7 + I)
    lstms = [nn.LSTM(I, 64, 1, batch_first=True), nn.LSTM(64, 64, 1, batch_first=True)]
    head = [nn.Linear(64, 3), nn.Tanh()] if mode == "hn_head" else []
    g = writer.export_lstm(lstms, head, batch=1, seq_len=T, mode=mode, with_state=state)
    d = str(tmp_path)
    writer.write_model_files(g, d)
    api.initialize(d)
    plan = api.plan_description()
    assert "lstm2_tc" in plan, plan
    oracle = OracleModel(d)
    rows = [int(np.prod(s)) // s[b] for s, b in api.input_specs()]
    rng = np.random.default_rng(len(case))
    for n in (1, 129, 1000, 4097):
        ins = [rng.uniform(-1.5, 1.5, size=(r, n)).astype(np.float32) if i == 0
               else rng.uniform(-0.5, 0.5, size=(r, n)).astype(np.float32) for i, r in enumerate(rows)]
        out = api.use_model_rows(ins)[0]
        ref = oracle.run_batched(n, ins)[0]
        assert_close(out, ref.reshape(out.shape), f"{case} n={n}")

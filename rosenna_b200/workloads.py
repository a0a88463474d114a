"""The five benchmark workloads: seeded synthetic models and inputs.

Each workload is a small physics-style network of the kinds roseNNa runs
(MLP, LSTM, CNN), exported to roseNNa's model files through
rosenna_b200.writer at export batch 1, with seeded weights and seeded synthetic
inputs (no dataset is involved).  Weights use torch.manual_seed(1000 + k), inputs
numpy.random.default_rng(2000 + k) (or a torch generator seeded the same way for
device-side generation of large batches); values are generated in fp64 and
rounded to fp32, and the same fp32 values feed the engine and the fp64 oracle.

Inputs are returned in the batched reference layout: (rows, n) arrays, row r
holding per-sample element r (Fortran order of the shape without its batch
dimension) for all n samples, when the batch is the input's first dimension;
the 2-layer LSTM's (2, N, 64) initial states, whose batch is the middle
dimension, are (64, n, 2) C-order arrays (the Fortran order of (2, n, 64)).
"""
from __future__ import annotations

import math
import os
from dataclasses import dataclass
from typing import Callable, Dict, List

import numpy as np
import torch
import torch.nn as nn

from . import writer


@dataclass
class Workload:
    key: int
    name: str
    description: str
    batch: int                      # full batch of the workload
    flops_per_sample: int           # 2 x MACs of the Gemm / gate / conv contractions
    io_bytes_per_sample: int        # fp32 input + output bytes
    input_rows: List[int]
    output_rows: List[int]
    build: Callable[[], tuple]      # -> (graph, torch module for fp64 reference or None)
    inputs: Callable[[int, object], List[np.ndarray]]


def _xavier_mlp(dims, act):
    mods = []
    for i in range(len(dims) - 1):
        lin = nn.Linear(dims[i], dims[i + 1])
        nn.init.xavier_uniform_(lin.weight, gain=1.0)
        nn.init.zeros_(lin.bias)
        mods.append(lin)
        if i + 2 < len(dims):
            mods.append(act())
    return mods


def _kaiming_mlp(dims):
    mods = []
    for i in range(len(dims) - 1):
        lin = nn.Linear(dims[i], dims[i + 1])
        nn.init.kaiming_uniform_(lin.weight, nonlinearity="relu")
        nn.init.uniform_(lin.bias, -0.05, 0.05)
        mods.append(lin)
        if i + 2 < len(dims):
            mods.append(nn.ReLU())
    return mods


def _rng(k, seed_offset=0):
    return np.random.default_rng(2000 + k + seed_offset)


def _f32(a):
    return np.ascontiguousarray(np.asarray(a, dtype=np.float64).astype(np.float32))


# ---- 1: small MLP ----------------------------------------------------------------
def _small_mlp():
    torch.manual_seed(1001)
    mods = _xavier_mlp([10, 64, 64, 64, 5], nn.Tanh)
    return writer.export_sequential(mods, [1, 10]), nn.Sequential(*mods)


def _small_mlp_inputs(n, rng):
    return [_f32(rng.uniform(-1.0, 1.0, size=(10, n)))]


# ---- 2: wide MLP -------------------------------------------------------------------
# 16 -> 256, four hidden 256 -> 256 layers, 256 -> 8 (six Linear layers, ReLU between)
def _wide_mlp():
    torch.manual_seed(1002)
    mods = _kaiming_mlp([16, 256, 256, 256, 256, 256, 8])
    return writer.export_sequential(mods, [1, 16]), nn.Sequential(*mods)


def _wide_mlp_inputs(n, rng):
    return [_f32(rng.standard_normal(size=(16, n)))]


# ---- 3: LSTM + head ----------------------------------------------------------------
class _LstmHead(nn.Module):
    def __init__(self, lstms, head):
        super().__init__()
        self.lstms = nn.ModuleList(lstms)
        self.head = nn.Sequential(*head)

    def forward(self, x, *state):
        for i, l in enumerate(self.lstms):
            if state:
                x, (hn, cn) = l(x, (state[2 * i], state[2 * i + 1]))
            else:
                x, (hn, cn) = l(x)
        return self.head(hn.view(-1, hn.size(2)))


def _lstm():
    torch.manual_seed(1003)
    lstm = nn.LSTM(8, 32, 1, batch_first=True)
    head = [nn.Linear(32, 4)]
    g = writer.export_lstm([lstm], head, batch=1, seq_len=50, mode="hn_head", with_state=False)
    return g, _LstmHead([lstm], head)


def _lstm_inputs(n, rng):
    # x (n, 50, 8) ~ N(0, 0.5^2); rows t + 50*i
    return [_f32(0.5 * rng.standard_normal(size=(50 * 8, n)))]


# ---- 4: CNN ----------------------------------------------------------------------------
def _cnn():
    torch.manual_seed(1004)
    c1, c2 = nn.Conv2d(1, 8, 3, padding=1), nn.Conv2d(8, 16, 3, padding=1)
    f1, f2 = nn.Linear(784, 64), nn.Linear(64, 10)
    for m in (c1, c2, f1, f2):
        nn.init.kaiming_uniform_(m.weight, nonlinearity="relu")
    mods = [c1, nn.ReLU(), nn.MaxPool2d(2, 2), c2, nn.ReLU(), nn.AvgPool2d(2, 2), nn.Flatten(), f1, nn.ReLU(), f2]
    return writer.export_sequential(mods, [1, 1, 28, 28]), nn.Sequential(*mods)


def _cnn_inputs(n, rng):
    return [_f32(rng.standard_normal(size=(784, n)))]


# ---- 5: a 2-layer stacked LSTM + MLP head ----------------------------------------
class _StackedHead(nn.Module):
    def __init__(self, lstm, head):
        super().__init__()
        self.lstm = lstm
        self.head = nn.Sequential(*head)

    def forward(self, x, h0, c0):
        _, (hn, _) = self.lstm(x, (h0, c0))
        return self.head(hn[-1])


def _lstm2():
    torch.manual_seed(1005)
    lstm = nn.LSTM(12, 64, 2, batch_first=True)
    head = [nn.Linear(64, 64), nn.ReLU(), nn.Linear(64, 3)]
    g = writer.export_stacked_lstm(lstm, head, batch=1, seq_len=100)
    return g, _StackedHead(lstm, head)


def _lstm2_inputs(n, rng):
    T, F = 100, 12
    t = np.arange(T, dtype=np.float64)
    x = np.zeros((T, F, n), dtype=np.float64)  # -> rows t + T*f
    for k in range(1, 5):
        phi = rng.uniform(0.0, 2.0 * math.pi, size=(F, n))
        x += (1.0 / k) * np.sin(2.0 * math.pi * k * t[:, None, None] / T + phi[None, :, :])
    x += 0.05 * rng.standard_normal(size=(T, F, n))
    rows = x.transpose(1, 0, 2).reshape(F * T, n)  # row f*T + t, i.e. t + T*f
    # h0, c0: (2, n, 64) in Fortran order = (64, n, 2) C order
    h = [_f32(0.1 * rng.standard_normal(size=(64, n, 2))) for _ in range(2)]
    return [_f32(rows), h[0], h[1]]


WORKLOADS: Dict[str, Workload] = {
    "small_mlp": Workload(1, "small_mlp", "MLP 10-64-64-64-5, tanh, fp32", 1_048_576, 2 * 9_152, 4 * (10 + 5),
                          [10], [5], _small_mlp, _small_mlp_inputs),
    "wide_mlp": Workload(2, "wide_mlp", "MLP 16-256-256-256-256-256-8, ReLU, fp32", 4_194_304, 2 * 268_288,
                         4 * (16 + 8), [16], [8], _wide_mlp, _wide_mlp_inputs),
    "lstm": Workload(3, "lstm", "LSTM I=8 H=32 T=50 + Linear(32,4), fp32", 262_144, 2 * (50 * 128 * 40 + 128),
                     4 * (400 + 4), [400], [4], _lstm, _lstm_inputs),
    "cnn": Workload(4, "cnn", "CNN 1x28x28: conv8+relu+max2, conv16+relu+avg2, 784-64-10, fp32", 65_536,
                    2 * 333_056, 4 * (784 + 10), [784], [10], _cnn, _cnn_inputs),
    "lstm2": Workload(5, "lstm2", "LSTM I=12 H=64 2 layers T=100 + MLP 64-64-3, fp32", 1_048_576,
                      2 * (100 * 256 * 76 + 100 * 256 * 128 + 64 * 64 + 64 * 3), 4 * (1200 + 4 * 64 + 3),
                      [1200, 128, 128], [3], _lstm2, _lstm2_inputs),
}


def write_model(name: str, out_dir: str):
    """Writes the workload's model files; returns the torch module (fp32 weights)."""
    g, module = WORKLOADS[name].build()
    writer.write_model_files(g, out_dir)
    return module


def make_inputs(name: str, n: int, seed_offset: int = 0) -> List[np.ndarray]:
    w = WORKLOADS[name]
    return w.inputs(n, _rng(w.key, seed_offset))


def torch_reference(name: str, module, inputs: List[np.ndarray]) -> List[np.ndarray]:
    """fp64 PyTorch evaluation of the workload on (rows, n) inputs; returns (rows, n) outputs."""
    w = WORKLOADS[name]
    m = module.double().eval()
    n = inputs[0].shape[1]
    with torch.no_grad():
        if name in ("small_mlp", "wide_mlp"):
            y = m(torch.from_numpy(inputs[0].T.astype(np.float64)))
            return [y.numpy().T.copy()]
        if name == "cnn":
            x = inputs[0].astype(np.float64).reshape(28, 28, 1, n)  # rows c + 1*(h + 28*w): (w, h, c, n)
            x = torch.from_numpy(x).permute(3, 2, 1, 0).contiguous()  # (n, c, h, w)
            return [m(x).numpy().T.copy()]
        T, I = (50, 8) if name == "lstm" else (100, 12)
        x = inputs[0].astype(np.float64).reshape(I, T, n)  # rows t + T*i
        x = torch.from_numpy(x).permute(2, 1, 0).contiguous()  # (n, T, I)
        if name == "lstm":
            y = m(x)
        else:  # (64, n, 2) C order -> (2, n, 64)
            st = [torch.from_numpy(np.asarray(a, dtype=np.float64).reshape(64, n, 2).transpose(2, 1, 0).copy())
                  for a in inputs[1:]]
            y = m(x, *st)
        return [y.numpy().T.copy()]


def make_inputs_torch(name: str, n: int, device="cuda", seed_offset: int = 0) -> List[torch.Tensor]:
    """The workload's synthetic inputs generated on `device` ((rows, n) fp32),
    from a torch generator seeded with 2000 + k (+ offset): for batches too large
    to generate on the host quickly.  Same distributions as make_inputs."""
    w = WORKLOADS[name]
    g = torch.Generator(device=device)
    g.manual_seed(2000 + w.key + seed_offset)
    f64 = dict(dtype=torch.float64, device=device, generator=g)
    if name == "small_mlp":
        return [(torch.rand((10, n), **f64) * 2.0 - 1.0).float()]
    if name == "wide_mlp":
        return [torch.randn((16, n), **f64).float()]
    if name == "lstm":
        return [(0.5 * torch.randn((400, n), **f64)).float()]
    if name == "cnn":
        return [torch.randn((784, n), **f64).float()]
    T, F = 100, 12
    t = torch.arange(T, dtype=torch.float64, device=device).view(1, T, 1)
    x = torch.zeros((F, T, n), dtype=torch.float64, device=device)  # rows t + T*f
    for k in range(1, 5):
        phi = torch.rand((F, 1, n), **f64) * (2.0 * math.pi)
        x += (1.0 / k) * torch.sin(2.0 * math.pi * k * t / T + phi)
    x += 0.05 * torch.randn((F, T, n), **f64)
    states = [(0.1 * torch.randn((64, n, 2), **f64)).float() for _ in range(2)]  # (2, n, 64) Fortran order
    return [x.reshape(F * T, n).float()] + states

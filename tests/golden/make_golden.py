"""Generates the golden fixtures under tests/golden/<case>/.

roseNNa commits no golden vectors: each goldenFiles/<case>/<case>.py builds a
PyTorch model with unseeded default init, runs it on torch.ones / torch.rand
inputs, writes the golden output (<case>.txt: shape line, then the values in C
order) and exports the model to ONNX (goldenFiles/*/*.py; test/run.sh:1-23).
This script restates those sixteen case definitions (minus mnist, which needs
onnxruntime) with seeded weights and inputs, and for each case writes

  onnxModel.txt, onnxWeights.txt, variables.fpp   the model files, through
                                                  rosenna_b200.writer (the
                                                  restated modelParserONNX.py)
  inputs.txt      per input: a shape line, then its values in C order
  golden.txt      PyTorch's fp64 output in the reference format (shape line,
                  values in C order), the same convention test/testChecker.py reads

Run from the repository root:  python tests/golden/make_golden.py
"""
import os
import sys

import numpy as np
import torch
import torch.nn as nn

HERE = os.path.dirname(os.path.abspath(__file__))
sys.path.insert(0, os.path.dirname(os.path.dirname(HERE)))

from rosenna_b200 import writer  # noqa: E402
from rosenna_b200.writer import View  # noqa: E402


def _line(vals):
    return " ".join(str(float(v)) for v in vals)


def _write_case(name, graph, inputs, golden):
    d = os.path.join(HERE, name)
    writer.write_model_files(graph, d)
    with open(os.path.join(d, "inputs.txt"), "w") as f:
        for x in inputs:
            x = np.asarray(x, dtype=np.float64)
            f.write(" ".join(str(s) for s in x.shape) + "\n")
            f.write(_line(x.reshape(-1)) + "\n")
    g = np.asarray(golden, dtype=np.float64)
    with open(os.path.join(d, "golden.txt"), "w") as f:
        f.write(" ".join(str(s) for s in g.shape) + "\n")
        f.write(_line(g.reshape(-1)) + "\n")


def _f32(t):
    """Round to fp32, the precision of the exported weights and inputs."""
    return t.float()


def mlp_case(name, seed, layers, in_dim, inp_kind="ones", batch=1):
    torch.manual_seed(seed)
    mods = layers()
    x = torch.ones(batch, in_dim) if inp_kind == "ones" else torch.rand(batch, in_dim)
    x = _f32(x)
    g = writer.export_sequential(mods, [batch, in_dim])
    net = nn.Sequential(*mods).double()
    with torch.no_grad():
        y = net(x.double())
    _write_case(name, g, [x.numpy()], y.numpy())


class _LstmHead(nn.Module):
    def __init__(self, lstm, head, mode):
        super().__init__()
        self.lstm, self.head, self.mode = lstm, nn.Sequential(*head), mode

    def forward(self, x, h, c):
        y, (hn, cn) = self.lstm(x, (h, c))
        if self.mode == "cn":
            return cn
        if self.mode == "y":
            return y
        if self.mode == "hn_head":
            return self.head(hn.view(-1, hn.size(2)))
        return self.head(y.reshape(-1, y.size(2)))


def lstm_case(name, seed, I, H, T, head_fn, mode, batch=1):
    torch.manual_seed(seed)
    lstm = nn.LSTM(I, H, 1, batch_first=True)
    head = head_fn() if head_fn else []
    x = torch.ones(batch, T, I)
    h0 = torch.ones(1, batch, H)
    c0 = torch.ones(1, batch, H)
    g = writer.export_lstm([lstm], head, batch, T, mode=mode, with_state=True)
    net = _LstmHead(lstm, head, mode).double()
    with torch.no_grad():
        y = net(x.double(), h0.double(), c0.double())
    _write_case(name, g, [x.numpy(), h0.numpy(), c0.numpy()], y.numpy())


def conv_case(name, seed, mods_fn, shape):
    torch.manual_seed(seed)
    mods = mods_fn()
    x = _f32(torch.rand(*shape))
    g = writer.export_sequential(mods, list(shape))
    net = nn.Sequential(*mods).double()
    with torch.no_grad():
        y = net(x.double())
    _write_case(name, g, [x.numpy()], y.numpy())


def _head():
    return [nn.Linear(2, 2), nn.ReLU(), nn.Linear(2, 3), nn.Sigmoid(), nn.Linear(3, 3), nn.ReLU(),
            nn.Linear(3, 1), nn.Sigmoid()]


def main():
    # MLPs: goldenFiles/gemm_small, gemm_big, batchnet, droplet
    mlp_case("gemm_small", 101, lambda: [nn.Linear(2, 2), nn.ReLU(), nn.Linear(2, 3), nn.ReLU()], 2)
    mlp_case("gemm_big", 102, lambda: [nn.Linear(2, 20), nn.ReLU(), nn.Linear(20, 30), nn.Sigmoid(),
                                       nn.Linear(30, 30), nn.ReLU(), nn.Linear(30, 40), nn.Tanh(),
                                       nn.Linear(40, 1), nn.Sigmoid()], 2)
    mlp_case("batchnet", 103, lambda: [nn.Linear(2, 8), nn.ReLU(), nn.Linear(8, 16), nn.ReLU(),
                                       nn.Linear(16, 32), nn.ReLU(), nn.Linear(32, 16), nn.ReLU(),
                                       nn.Linear(16, 8), nn.ReLU(), nn.Linear(8, 68)], 2)
    mlp_case("droplet", 104, lambda: [nn.Linear(4, 5), nn.Linear(5, 3)], 4)
    # LSTMs: goldenFiles/lstm_cell, lstm_output, lstm_gemm, lstm_gemm_hid
    lstm_case("lstm_cell", 105, 5, 2, 2, None, "cn")
    lstm_case("lstm_output", 106, 10, 20, 25, None, "y")
    lstm_case("lstm_gemm", 107, 5, 2, 2, _head, "y_head")
    lstm_case("lstm_gemm_hid", 108, 5, 2, 2, _head, "hn_head")
    # Convolutions and pooling: goldenFiles/conv_*, maxpool_*, avgpool_basic
    conv_case("conv_basic", 109, lambda: [nn.Conv2d(2, 3, 3)], (2, 2, 7, 7))
    conv_case("conv_padding", 110, lambda: [nn.Conv2d(2, 3, 3, padding=[2, 3])], (1, 2, 6, 6))
    conv_case("conv_strides", 111, lambda: [nn.Conv2d(2, 3, 3, stride=2)], (1, 2, 7, 7))
    conv_case("conv_padding-stride", 112, lambda: [nn.Conv2d(2, 3, 3, padding=[2, 3], stride=2)], (1, 2, 6, 6))
    conv_case("maxpool_basic", 113, lambda: [nn.MaxPool2d(3)], (1, 2, 6, 6))
    conv_case("maxpool_padding", 114, lambda: [nn.MaxPool2d(3, padding=[1, 1])], (1, 2, 6, 6))
    conv_case("maxpool_strides", 115, lambda: [nn.MaxPool2d(3, stride=1)], (1, 2, 6, 6))
    conv_case("avgpool_basic", 116, lambda: [nn.AvgPool2d(3)], (1, 2, 6, 6))
    # A small CNN in the shape of the conv/pool/view/Linear stack (two conv blocks + head)
    conv_case("cnn_small", 117, lambda: [nn.Conv2d(1, 4, 3, padding=1), nn.ReLU(), nn.MaxPool2d(2, 2),
                                         nn.Conv2d(4, 6, 3, padding=1), nn.ReLU(), nn.AvgPool2d(2, 2),
                                         View(1, -1), nn.Linear(6 * 3 * 3, 16), nn.ReLU(), nn.Linear(16, 5)],
              (1, 1, 12, 12))


if __name__ == "__main__":
    main()

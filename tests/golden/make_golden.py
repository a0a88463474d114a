"""Generates the golden fixtures under tests/golden/<case>/.

roseNNa commits no golden vectors: each goldenFiles/<case>/<case>.py builds a
PyTorch model with unseeded default init, runs it on torch.ones / torch.rand
inputs, writes the golden output (<case>.txt: shape line, then the values in C
order) and exports the model to ONNX (goldenFiles/*/*.py; test/run.sh:1-23).
This script restates those case definitions with seeded weights and inputs,
and for each case writes

  onnxModel.txt, onnxWeights.txt, variables.fpp   the model files, through
                                                  rosenna_b200.writer (the
                                                  restated modelParserONNX.py)
  inputs.txt      per input: a shape line, then its values in C order
  golden.txt      PyTorch's fp64 output in the reference format (shape line,
                  values in C order), the same convention test/testChecker.py reads

mnist (goldenFiles/mnist) is the one case with a stored model: mnist.onnx,
scored there by onnxruntime, which is not installed here.  Its model files
come from that file through rosenna_b200.onnx_file (the restated parser); its
input is the one goldenFiles/mnist/mnist.py feeds, read from that file as
text; its golden output is an independent fp64 evaluation of the ONNX graph
in PyTorch (`eval_graph`).  It is regenerated only where the reference tree
is present.  add_matmul and add_conv are seeded graphs of the same op forms
(stored-constant Reshape, MatMul, broadcast Add after an activation or a
pool), scored the same way.

Run from the repository root:  python tests/golden/make_golden.py
"""
import os
import sys

import numpy as np
import torch
import torch.nn as nn

HERE = os.path.dirname(os.path.abspath(__file__))
sys.path.insert(0, os.path.dirname(os.path.dirname(HERE)))

from rosenna_b200 import onnx_file, writer  # noqa: E402
from rosenna_b200.writer import Graph, Node, View  # noqa: E402

# the roseNNa checkout (its goldenFiles/mnist holds the one stored model);
# ROSENNA_REFERENCE_DIR names it, the mnist case is skipped without it
REFERENCE_DIR = os.environ.get("ROSENNA_REFERENCE_DIR", "")
REFERENCE_MNIST = os.path.join(REFERENCE_DIR, "goldenFiles", "mnist") if REFERENCE_DIR else ""


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


def stacked_lstm_case(name, seed, I, H, T, layers, head_fn, batch=1):
    """A batch-first nn.LSTM with num_layers >= 2, given (h0, c0) of shape
    (layers, N, H), with a head on the last layer's h_n: the graph
    torch.onnx.export gives it (Slice of the states per layer, Concat of h_n,
    Gather of the last layer), which the reference parser passes through
    unwritten (modelParserONNX.py:519-523) and this build's front end writes."""
    torch.manual_seed(seed)
    lstm = nn.LSTM(I, H, layers, batch_first=True)
    head = head_fn()
    x = torch.ones(batch, T, I)
    h0 = torch.ones(layers, batch, H) * 0.5
    c0 = torch.ones(layers, batch, H) * -0.25
    g = writer.export_stacked_lstm(lstm, head, batch, T)
    net = nn.Sequential(*head).double()
    with torch.no_grad():
        _, (hn, _) = lstm.double()(x.double(), (h0.double(), c0.double()))
        y = net(hn[-1])
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


def eval_graph(g, feeds):
    """ONNX semantics in torch fp64 for the ops of the stored-model cases."""
    import torch.nn.functional as F

    env = {k: torch.tensor(np.asarray(v, dtype=np.float64)) for k, v in g.initializers.items()}
    env.update({k: torch.tensor(np.asarray(v)) for k, v in g.constants.items()})
    env.update({k: torch.tensor(np.asarray(v, dtype=np.float64)) for k, v in feeds.items()})
    for nd in g.nodes:
        a = nd.attrs
        x = [env.get(i) for i in nd.inputs]
        op = nd.op_type
        if op == "Constant":
            continue
        if op in ("Conv", "MaxPool", "AveragePool"):
            k = list(a["kernel_shape"])
            st = list(a.get("strides", [1, 1]))
            auto = str(a.get("auto_pad", "NOTSET"))
            if auto in ("SAME_UPPER", "SAME_LOWER"):
                pads = []
                for i in range(2):
                    size = x[0].shape[2 + i]
                    total = max(0, (-(-size // st[i]) - 1) * st[i] + k[i] - size)
                    lo = total // 2 if auto == "SAME_UPPER" else total - total // 2
                    pads.append((lo, total - lo))
                pt, pl, pb, pr = pads[0][0], pads[1][0], pads[0][1], pads[1][1]
            else:
                pt, pl, pb, pr = list(a.get("pads", [0, 0, 0, 0]))
            fill = float("-inf") if op == "MaxPool" else 0.0
            xp = F.pad(x[0], (pl, pr, pt, pb), value=fill)
            if op == "Conv":
                y = F.conv2d(xp, x[1], x[2] if len(x) > 2 else None, stride=st)
            elif op == "MaxPool":
                y = F.max_pool2d(xp, k, st)
            else:
                y = F.avg_pool2d(xp, k, st)
        elif op == "Add":
            y = x[0] + x[1]
        elif op == "MatMul":
            y = torch.matmul(x[0], x[1])
        elif op == "Relu":
            y = torch.relu(x[0])
        elif op == "Tanh":
            y = torch.tanh(x[0])
        elif op == "Sigmoid":
            y = torch.sigmoid(x[0])
        elif op == "Reshape":
            tgt = [int(v) for v in x[1].reshape(-1).tolist()]
            tgt = [x[0].shape[i] if d == 0 else d for i, d in enumerate(tgt)]
            y = x[0].reshape(tgt)
        else:
            raise ValueError(f"eval_graph: op {op}")
        env[nd.outputs[0]] = y
    return [env[name].numpy() for name, _ in g.outputs]


def stored_model_case(name, g, inputs):
    feeds = {nm: x for (nm, _), x in zip([i for i in g.inputs if i[0] not in g.initializers], inputs)}
    (y,) = eval_graph(g, feeds)
    _write_case(name, g, inputs, y)


def mnist_case():
    import re

    if not REFERENCE_MNIST or not os.path.isdir(REFERENCE_MNIST):
        print("mnist: reference tree absent, committed fixture kept")
        return
    g = onnx_file.load_graph(os.path.join(REFERENCE_MNIST, "mnist.onnx"))
    with open(os.path.join(REFERENCE_MNIST, "mnist.py")) as f:
        body = re.search(r"inp = np\.array\(\[(.*?)\]\)", f.read(), re.S).group(1)
    x = np.array([float(v) for v in body.split(",")], dtype=np.float32).reshape(1, 1, 28, 28)
    stored_model_case("mnist", g, [x])


def add_matmul_case(seed=118):
    """x(1,6) . Reshape(W(2,3,4) -> (6,4)) + b(4) -> Relu -> + c(1,4) -> Tanh."""
    rng = np.random.default_rng(seed)
    f32 = lambda *s: rng.uniform(-1, 1, size=s).astype(np.float32)  # noqa: E731
    init = {"W": f32(2, 3, 4), "shape": np.array([6, 4], np.int64), "b": f32(4), "c": f32(1, 4)}
    nodes = [Node("Reshape", ["W", "shape"], ["Wr"]), Node("MatMul", ["x", "Wr"], ["mm"]),
             Node("Add", ["mm", "b"], ["ab"]), Node("Relu", ["ab"], ["r"]), Node("Add", ["r", "c"], ["ac"]),
             Node("Tanh", ["ac"], ["y"])]
    vi = {"Wr": [6, 4], "mm": [1, 4], "ab": [1, 4], "r": [1, 4], "ac": [1, 4]}
    g = Graph(nodes=nodes, inputs=[("x", [1, 6])], outputs=[("y", [1, 4])], initializers=init, value_info=vi)
    stored_model_case("add_matmul", g, [f32(1, 6)])


def add_conv_case(seed=119):
    """Conv (no bias, SAME_UPPER) + Add(3,1,1) -> Relu -> MaxPool 2 -> Add(3,1,1) -> Sigmoid -> Reshape(1,27)."""
    rng = np.random.default_rng(seed)
    f32 = lambda *s: rng.uniform(-1, 1, size=s).astype(np.float32)  # noqa: E731
    init = {"K": f32(3, 2, 3, 3), "b1": f32(3, 1, 1), "b2": f32(3, 1, 1), "shape": np.array([1, 27], np.int64)}
    nodes = [Node("Conv", ["x", "K"], ["cv"], {"kernel_shape": [3, 3], "strides": [1, 1], "auto_pad": "SAME_UPPER",
                                              "group": 1, "dilations": [1, 1]}),
             Node("Add", ["cv", "b1"], ["a1"]), Node("Relu", ["a1"], ["r1"]),
             Node("MaxPool", ["r1"], ["p1"], {"kernel_shape": [2, 2], "strides": [2, 2], "pads": [0, 0, 0, 0]}),
             Node("Add", ["p1", "b2"], ["a2"]), Node("Sigmoid", ["a2"], ["s2"]),
             Node("Reshape", ["s2", "shape"], ["y"])]
    vi = {"cv": [1, 3, 6, 6], "a1": [1, 3, 6, 6], "r1": [1, 3, 6, 6], "p1": [1, 3, 3, 3], "a2": [1, 3, 3, 3],
          "s2": [1, 3, 3, 3], "y": [1, 27]}
    g = Graph(nodes=nodes, inputs=[("x", [1, 2, 6, 6])], outputs=[("y", [1, 27])], initializers=init, value_info=vi)
    stored_model_case("add_conv", g, [f32(1, 2, 6, 6)])


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
    # a stacked nn.LSTM(num_layers=2) exported as one graph (Slice / Concat / Gather)
    stacked_lstm_case("lstm_stacked", 120, 5, 6, 4, 2, lambda: [nn.Linear(6, 3), nn.Tanh()])
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
    # Stored-model op forms: goldenFiles/mnist and two seeded graphs like it
    mnist_case()
    add_matmul_case()
    add_conv_case()


if __name__ == "__main__":
    main()

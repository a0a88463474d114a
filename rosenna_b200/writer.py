"""Model-file writer: emits roseNNa's onnxModel.txt, onnxWeights.txt and variables.fpp.

roseNNa's front end is fLibrary/modelParserONNX.py, which walks an ONNX graph and
writes these three files (modelParserONNX.py:151-541).  This module restates that
walk over an in-memory graph (:class:`Graph`), so the files can be produced
without the `onnx` package, plus exporters that build the graph torch.onnx.export
would produce (opset 10, two exports: folded structure + unfolded weights) for the
module kinds roseNNa supports: Linear/ReLU/Tanh/Sigmoid chains, batch-first
single-layer LSTMs with a head, and Conv/MaxPool/AvgPool/view stacks.

The files keep the reference format exactly:
  onnxModel.txt    node count, then per node its op name and the dims lines that
                   fLibrary/reader.f90:38-290 reads;
  onnxWeights.txt  one tensor per line, values in Fortran column-major order
                   printed with Python ``str(float)`` (modelParserONNX.py:72-86);
  variables.fpp    ``#:set architecture/inputs/trueInputs/outShape/outputs``
                   (modelParserONNX.py:531-541).
"""
from __future__ import annotations

import os
from dataclasses import dataclass, field
from typing import Dict, List, Optional, Sequence, Tuple

import numpy as np


@dataclass
class Node:
    op_type: str
    inputs: List[str]
    outputs: List[str]
    attrs: Dict[str, object] = field(default_factory=dict)  # attribute name -> int | list[int] | str


@dataclass
class Graph:
    nodes: List[Node]
    inputs: List[Tuple[str, List[int]]]          # graph inputs that are not initializers
    outputs: List[Tuple[str, List[int]]]
    initializers: Dict[str, np.ndarray]          # folded export (dims source)
    value_info: Dict[str, List[int]]             # inferred intermediate shapes
    constants: Dict[str, np.ndarray] = field(default_factory=dict)
    true_weights: Optional[List[np.ndarray]] = None  # unfolded export initializers, in order


def _values_line(arr) -> str:
    """stranspose + stringer (modelParserONNX.py:72-86): the pairwise axis swaps
    there reverse all axes before a C-order flatten, i.e. a Fortran-order flatten."""
    a = np.asarray(arr)
    vals = a.flatten(order="F").tolist()
    return " ".join(str(float(v)) for v in vals)


def _reshape_parser(reshape: List[int], true_shape: List[int]) -> List[int]:
    """reshapeParser, modelParserONNX.py:88-103: resolve one -1 entry."""
    reshape = list(reshape)
    for i, d in enumerate(reshape):
        if d == -1:
            res = int(np.prod(reshape)) * -1
            reshape[i] = int(int(np.prod(true_shape)) / res)
            break
    return reshape


def _auto_pads(kernel: int, mode: str) -> List[int]:
    """SAME_UPPER / SAME_LOWER pads from the first kernel dim, as
    modelParserONNX.py:348-358 and :411-421 compute them."""
    total = kernel - 1
    pad = int(total / 2)
    if total % 2 != 0:
        return [pad, pad, pad + 1, pad + 1] if mode == "SAME_UPPER" else [pad + 1, pad + 1, pad, pad]
    return [pad] * 4


def _four_d_transform(true_shape: List[int], adder_shape: List[int]) -> List[int]:
    """fourDTransform, modelParserONNX.py:110-119: each adder dim is placed at
    the position of its FIRST equal dim in the input shape (counted from the
    right of a rank-4 shape); dims without an equal are dropped."""
    new = [1, 1, 1, 1]
    for dim in adder_shape:
        if dim in true_shape:
            new[true_shape.index(dim) - len(true_shape)] = dim
    return new


def _spread_info(true: List[int], fourd: List[int]) -> List[int]:
    """spreadInfo, modelParserONNX.py:125-131: (1-based dim, copies) pairs where
    the shapes differ."""
    ret: List[int] = []
    for i, d in enumerate(fourd):
        if true[i] != d:
            ret += [i + 1, true[i]]
    return ret


def write_model_files(g: Graph, out_dir: str) -> None:
    """Restates the node walk of modelParserONNX.py:151-541 for the supported ops."""
    os.makedirs(out_dir, exist_ok=True)
    external = g.true_weights is not None
    true_weights = list(g.true_weights or [])
    true_index = 0

    io_map: Dict[str, str] = {name: name for name, _ in g.inputs}
    input_shapes = {name: list(s) for name, s in g.inputs}
    inter = dict(g.value_info)
    init_dims = {k: list(v.shape) for k, v in g.initializers.items()}
    out = {name: [d if d != 0 else 1 for d in s] for name, s in g.outputs}
    outputs: Dict[str, str] = {}
    out_shape: List[list] = []
    arch: List[tuple] = []
    inputs: List[list] = []
    extra = "0"

    def find_weights(name):
        if name in g.initializers:
            return g.initializers[name]
        return g.constants[name]

    def next_weights(name):
        nonlocal true_index
        if external:
            w = true_weights[true_index]
            true_index += 1
            return w
        return find_weights(name)

    f_lines: List[str] = [str(len(g.nodes))]
    w_lines: List[str] = []
    for node in g.nodes:
        layer = node.op_type
        for x in node.outputs:
            if x in out:
                out_shape.append([x, out[x]])
        if layer == "Transpose":  # :160-172
            f_lines.append(layer)
            src = node.inputs[0]
            rank = len(inter.get(src, input_shapes.get(src, [])))
            perm = node.attrs.get("perm", list(range(rank - 1, -1, -1)))
            arch.append(("Transpose", [io_map[src]], [[p + 1 for p in perm]]))
            io_map[node.outputs[0]] = io_map[src]
        elif layer == "LSTM":  # :174-243
            f_lines.append(layer)
            has_state = len(node.inputs) > 6 and node.inputs[5] in io_map and node.inputs[6] in io_map
            if has_state:
                arch.append(("LSTM", [io_map[node.inputs[0]], io_map[node.inputs[5]], io_map[node.inputs[6]]],
                             ["output" + extra], [0]))
                f_lines.append("0")
            else:
                arch.append(("LSTM", [io_map[node.inputs[0]], "output" + str(int(extra) + 1),
                                      "output" + str(int(extra) + 2)], ["output" + extra], [1]))
                f_lines.append("1")
            inputs.append(["output" + extra, len(inter[node.outputs[0]])])
            for inp in node.inputs[1:3]:
                f_lines.append(" ".join(str(d) for d in init_dims[inp]) + " ")
                w_lines.append(_values_line(next_weights(inp)))
            if not external:
                split = np.split(find_weights(node.inputs[3]), 2, axis=1)
            for x in range(2):
                f_lines.append(str(int(init_dims[node.inputs[3]][1] / 2)))
                w_lines.append(_values_line(true_weights[true_index] if external else split[x]))
                if external:
                    true_index += 1
            if not has_state:
                in_shape = inter[node.inputs[0]]
                batch = in_shape[1] if in_shape[1] != 0 else 1
                hidden = int(node.attrs["hidden_size"])
                shape = (1, batch, hidden)
                for _ in range(2):
                    f_lines.append(" ".join(str(s) for s in shape) + " ")
                    w_lines.append(_values_line(np.zeros(shape)))
                io_map[node.outputs[0]] = "output" + extra
                extra = str(int(extra) + 1)
                inputs.append(["output" + extra, len(inter[node.outputs[1]])])
                io_map[node.outputs[1]] = "output" + extra
                extra = str(int(extra) + 1)
                inputs.append(["output" + extra, len(inter[node.outputs[2]])])
                io_map[node.outputs[2]] = "output" + extra
                extra = str(int(extra) + 1)
            else:
                io_map[node.outputs[0]] = "output" + extra
                extra = str(int(extra) + 1)
                io_map[node.outputs[1]] = io_map[node.inputs[-2]]
                io_map[node.outputs[2]] = io_map[node.inputs[-1]]
        elif layer in ("Gemm",):  # :245-281
            f_lines.append(layer)
            trans_b = int(node.attrs.get("transB", 0))
            arch.append(("Gemm", [io_map[node.inputs[0]], trans_b], None))
            if len(node.inputs) < 3:
                numzs = 0
                for inp in node.inputs[1:]:
                    numzs = init_dims[inp][0]
                    f_lines.append(" ".join(str(d) for d in init_dims[inp]) + " ")
                    w_lines.append(_values_line(next_weights(inp)))
                f_lines.append(str(numzs))
                w_lines.append(_values_line(np.zeros(numzs)))
            else:
                for inp in node.inputs[1:3]:
                    f_lines.append(" ".join(str(d) for d in init_dims[inp]) + " ")
                    w_lines.append(_values_line(next_weights(inp)))
            io_map[node.outputs[0]] = io_map[node.inputs[0]]
        elif layer == "Squeeze":  # :284-308 (opset < 13: axes attribute; the walk appends two entries)
            f_lines.append(layer)
            src = node.inputs[0]
            axes = list(node.attrs.get("axes", []))
            entry = ("Squeeze", (io_map[src], len(inter[src])), ["output" + extra], [axes])
            if "axes" in node.attrs:
                arch.append(entry)
            arch.append(("Squeeze", (io_map[src], len(inter[src])), ["output" + extra],
                         [[x for x in range(len(inter[src])) if x == 1]]))
            inputs.append(["output" + extra, len(inter[node.outputs[0]])])
            io_map[node.outputs[0]] = "output" + extra
            extra = str(int(extra) + 1)
        elif layer == "Reshape":  # :312-331
            f_lines.append(layer)
            src = node.inputs[0]
            # the reference takes the variable form when the source has an
            # inferred intermediate shape, else the stored-constant form over
            # an initializer; a graph input without either is taken as a
            # variable here (the reference stops with a KeyError)
            if src in inter or (src in input_shapes and src not in init_dims):
                src_shape = inter.get(src, input_shapes.get(src))
                new_shape = _reshape_parser([int(v) for v in np.asarray(find_weights(node.inputs[-1])).tolist()], src_shape)
                arch.append(("Reshape", (io_map[src], len(src_shape)), ["output" + extra], [new_shape], [0]))
                f_lines.append("0")
            else:
                new_shape = _reshape_parser([int(v) for v in np.asarray(find_weights(node.inputs[-1])).tolist()], init_dims[src])
                arch.append(("Reshape", (io_map.get(src, src), len(init_dims[src])), ["output" + extra], [new_shape], [1]))
                f_lines.append(str(len(init_dims[src])))
                f_lines.append(" ".join(str(d) for d in init_dims[src]) + " ")
                w_lines.append(_values_line(find_weights(src)))
            inputs.append(["output" + extra, len(inter[node.outputs[0]])])
            io_map[node.outputs[0]] = "output" + extra
            extra = str(int(extra) + 1)
        elif layer == "Flatten":
            # modelParserONNX.py:519-523 writes nothing for Flatten and passes its
            # input through, so a Gemm after it would get the 4-D array; here it is
            # written as the variable-form Reshape entry that x.view(N, -1) gives
            # (:312-331), to the 2-D shape ONNX defines for Flatten(axis)
            f_lines.append("Reshape")
            src = node.inputs[0]
            src_shape = list(inter.get(src, input_shapes.get(src, [])))
            axis = int(node.attrs.get("axis", 1))
            axis = axis + len(src_shape) if axis < 0 else axis
            new_shape = [int(np.prod(src_shape[:axis])), int(np.prod(src_shape[axis:]))]
            arch.append(("Reshape", (io_map[src], len(src_shape)), ["output" + extra], [new_shape], [0]))
            f_lines.append("0")
            inputs.append(["output" + extra, 2])
            io_map[node.outputs[0]] = "output" + extra
            extra = str(int(extra) + 1)
        elif layer in ("Slice", "Gather", "Concat"):
            # modelParserONNX.py:519-523 passes these through unwritten; a stacked
            # LSTM export needs them (per-layer slices of its (L, N, H) initial
            # states, h_n = Concat of the layers' h_n, the head on h_n[-1]).  They
            # are written as architecture entries only (no weights):
            #   ('Slice', [x], [out], [axes, starts, ends])
            #   ('Gather', [x], [out], [axis, index])
            #   ('Concat', [x0, x1, ..], [out], [axis])
            src = node.inputs[0]
            if layer == "Slice":
                if len(node.inputs) >= 3:  # opset >= 10: starts, ends, axes as constant inputs
                    starts = [int(v) for v in np.asarray(find_weights(node.inputs[1])).reshape(-1)]
                    ends = [int(v) for v in np.asarray(find_weights(node.inputs[2])).reshape(-1)]
                    axes = ([int(v) for v in np.asarray(find_weights(node.inputs[3])).reshape(-1)]
                            if len(node.inputs) > 3 and node.inputs[3] else list(range(len(starts))))
                else:
                    starts, ends = list(node.attrs["starts"]), list(node.attrs["ends"])
                    axes = list(node.attrs.get("axes", range(len(starts))))
                ends = [min(e, 2 ** 31 - 1) for e in ends]
                arch.append(("Slice", [io_map[src]], ["output" + extra], [axes, starts, ends]))
            elif layer == "Gather":
                index = int(np.asarray(find_weights(node.inputs[1])).reshape(-1)[0])
                arch.append(("Gather", [io_map[src]], ["output" + extra], [int(node.attrs.get("axis", 0)), index]))
            else:
                arch.append(("Concat", [io_map[x] for x in node.inputs], ["output" + extra], [int(node.attrs["axis"])]))
            inputs.append(["output" + extra, len(inter[node.outputs[0]])])
            io_map[node.outputs[0]] = "output" + extra
            extra = str(int(extra) + 1)
        elif layer == "Conv":  # :333-390
            f_lines.append(layer)
            attributes = dict(node.attrs)
            pads = list(attributes.get("pads", [0, 0, 0, 0]))
            if "auto_pad" in attributes:  # :338-358: any auto_pad value, NOTSET included, replaces pads
                pads = _auto_pads(int(list(attributes["kernel_shape"])[0]), str(attributes["auto_pad"]))
            arch.append(("Conv", [io_map[node.inputs[0]]],
                         [list(attributes.get("dilations", [1, 1])), list(attributes["kernel_shape"]), pads,
                          list(attributes.get("strides", [1, 1]))]))
            if len(node.inputs) < 3:
                numzs = 0
                for inp in node.inputs[1:]:
                    numzs = init_dims[inp][0]
                    f_lines.append(" ".join(str(d) for d in init_dims[inp]) + " ")
                    w_lines.append(_values_line(next_weights(inp)))
                f_lines.append(str(numzs))
                w_lines.append(_values_line(np.zeros(numzs)))
            else:
                for inp in node.inputs[1:3]:
                    f_lines.append(" ".join(str(d) for d in init_dims[inp]) + " ")
                    w_lines.append(_values_line(next_weights(inp)))
            io_map[node.outputs[0]] = io_map[node.inputs[0]]
        elif layer == "MaxPool":  # :392-425
            f_lines.append(layer)
            pads = list(node.attrs.get("pads", [0, 0, 0, 0]))
            auto = str(node.attrs.get("auto_pad", "NOTSET"))
            if auto != "NOTSET":  # :400-421
                pads = _auto_pads(int(list(node.attrs["kernel_shape"])[0]), auto)
            arch.append(("MaxPool", [io_map[node.inputs[0]]],
                         [int(node.attrs.get("ceil_mode", 0)), pads, list(node.attrs["strides"])]))
            # :423: the window size written is the first int of the node's SECOND
            # attribute (kernel_shape in torch's sorted order; strides in files
            # that list kernel_shape, strides, ...)
            second = list(node.attrs.values())[1]
            f_lines.append(str(list(second)[0] if isinstance(second, (list, tuple)) else int(second)))
            io_map[node.outputs[0]] = io_map[node.inputs[0]]
        elif layer == "AveragePool":  # :427-439
            f_lines.append(layer)
            arch.append(("AveragePool", [io_map[node.inputs[0]]],
                         [int(node.attrs.get("ceil_mode", 0)), list(node.attrs.get("pads", [0, 0, 0, 0])),
                          list(node.attrs.get("strides", [1, 1]))]))
            f_lines.append(str(list(node.attrs["kernel_shape"])[0]))
            io_map[node.outputs[0]] = io_map[node.inputs[0]]
        elif layer == "Add":  # :441-457
            f_lines.append(layer)
            src = node.inputs[0]
            src_shape = list(inter.get(src, input_shapes.get(src, [])))  # (the reference reads value_info only)
            adder = np.asarray(find_weights(node.inputs[-1]))
            fourd = _four_d_transform(src_shape, list(adder.shape))
            true = [1] * (4 - len(src_shape)) + src_shape
            arch.append(("Add", [io_map[src]], [true, _spread_info(true, fourd), len(src_shape)]))
            f_lines.append("".join(str(d) + " " for d in fourd))
            w_lines.append(_values_line(next_weights(node.inputs[1])))
            io_map[node.outputs[0]] = io_map[src]
        elif layer == "MatMul":  # :459-488
            f_lines.append(layer)
            if node.inputs[0] in io_map and node.inputs[1] in io_map:
                rank = len(inter.get(node.inputs[0], input_shapes.get(node.inputs[0], [])))
                arch.append(("MatMul", [io_map[node.inputs[0]], io_map[node.inputs[1]]], [rank]))
            else:  # a weight operand that is no graph value: written as a bias-free Gemm (transB = 1)
                f_lines[-1] = "Gemm"
                arch.append(("Gemm", [io_map[node.inputs[0]], 1], None))
                numzs = 0
                for inp in node.inputs[1:]:
                    numzs = init_dims[inp][0]
                    f_lines.append(" ".join(str(d) for d in init_dims[inp]) + " ")
                    w_lines.append(_values_line(next_weights(inp)))
                f_lines.append(str(numzs))
                w_lines.append(_values_line(np.zeros(numzs)))
            io_map[node.outputs[0]] = io_map[node.inputs[0]]
        elif layer in ("Relu", "Sigmoid", "Tanh"):  # :495-514
            f_lines.append(layer)
            src = node.inputs[0]
            arch.append((layer, [io_map[src]], [len(inter.get(src, input_shapes.get(src, [])))]))
            io_map[node.outputs[0]] = io_map[src]
        elif layer == "Pad":  # :490-493
            f_lines.append(layer)
            io_map[node.outputs[0]] = io_map[node.inputs[0]]
        elif layer == "Constant":  # :515-518
            f_lines.append(layer)
            continue
        else:  # :519-523: unsupported ops write nothing and pass their input through
            io_map[node.outputs[0]] = io_map[node.inputs[0]]
            continue
    for x in list(io_map.keys()):
        if x in out:
            outputs[x] = io_map[x]
    true_inputs = [[name, [d if d != 0 else 1 for d in shape]] for name, shape in g.inputs if name not in g.initializers]

    with open(os.path.join(out_dir, "onnxModel.txt"), "w") as f:
        f.write("\n".join(f_lines) + "\n")
    with open(os.path.join(out_dir, "onnxWeights.txt"), "w") as f:
        f.write("\n".join(w_lines) + ("\n" if w_lines else ""))
    with open(os.path.join(out_dir, "variables.fpp"), "w") as f:
        f.write(f"#:set architecture = {arch}\n")
        f.write(f"#:set inputs = {inputs}\n")
        f.write(f"#:set trueInputs = {true_inputs}\n")
        f.write(f"#:set outShape = {out_shape}\n")
        f.write(f"#:set outputs = {outputs}\n")


# --------------------------------------------------------------------------
# Exporters: the graphs torch.onnx.export (opset 10) produces for the module
# kinds roseNNa's golden cases use (goldenFiles/*/*.py).
# --------------------------------------------------------------------------

def _np32(t) -> np.ndarray:
    return t.detach().cpu().to(dtype=__import__("torch").float32).numpy().copy()


class _Builder:
    def __init__(self):
        self.nodes: List[Node] = []
        self.inits: Dict[str, np.ndarray] = {}
        self.true_weights: List[np.ndarray] = []
        self.vi: Dict[str, List[int]] = {}
        self.consts: Dict[str, np.ndarray] = {}
        self.n = 0

    def name(self, base):
        self.n += 1
        return f"{base}_{self.n}"

    def add(self, op, inputs, out_shapes, attrs=None):
        outs = [self.name(op.lower()) for _ in out_shapes]
        self.nodes.append(Node(op, list(inputs), outs, dict(attrs or {})))
        for o, s in zip(outs, out_shapes):
            self.vi[o] = list(s)
        return outs

    def weight(self, arr, folded=None):
        nm = self.name("w")
        self.inits[nm] = folded if folded is not None else arr
        self.true_weights.append(arr)
        return nm

    def const(self, arr):
        outs = self.add("Constant", [], [list(np.shape(arr))])
        self.consts[outs[0]] = np.asarray(arr)
        return outs[0]


def _emit_module(b: _Builder, mod, x: str, shape: List[int]) -> Tuple[str, List[int]]:
    """Appends the nodes torch emits for one module; returns (output name, shape)."""
    import torch.nn as nn

    if isinstance(mod, nn.Linear):
        w = b.weight(_np32(mod.weight))
        ins = [x, w]
        if mod.bias is not None:
            ins.append(b.weight(_np32(mod.bias)))
        out_shape = shape[:-1] + [mod.out_features]
        (y,) = b.add("Gemm", ins, [out_shape], {"alpha": 1.0, "beta": 1.0, "transB": 1})
        return y, out_shape
    if isinstance(mod, (nn.ReLU, nn.Tanh, nn.Sigmoid)):
        op = {nn.ReLU: "Relu", nn.Tanh: "Tanh", nn.Sigmoid: "Sigmoid"}[type(mod)]
        (y,) = b.add(op, [x], [shape])
        return y, shape
    if isinstance(mod, nn.Conv2d):
        kh, kw = mod.kernel_size
        ph, pw = mod.padding
        sh, sw = mod.stride
        n, c, h, w_ = shape
        oh, ow = (h + 2 * ph - kh) // sh + 1, (w_ + 2 * pw - kw) // sw + 1
        wn = b.weight(_np32(mod.weight))
        ins = [x, wn]
        if mod.bias is not None:
            ins.append(b.weight(_np32(mod.bias)))
        out_shape = [n, mod.out_channels, oh, ow]
        (y,) = b.add("Conv", ins, [out_shape], {"dilations": [1, 1], "group": 1, "kernel_shape": [kh, kw],
                                                "pads": [ph, pw, ph, pw], "strides": [sh, sw]})
        return y, out_shape
    if isinstance(mod, (nn.MaxPool2d, nn.AvgPool2d)):
        k = mod.kernel_size if isinstance(mod.kernel_size, int) else mod.kernel_size[0]
        s = mod.stride if isinstance(mod.stride, int) else mod.stride[0]
        p = mod.padding if isinstance(mod.padding, int) else mod.padding[0]
        n, c, h, w_ = shape
        out_shape = [n, c, (h + 2 * p - k) // s + 1, (w_ + 2 * p - k) // s + 1]
        op = "MaxPool" if isinstance(mod, nn.MaxPool2d) else "AveragePool"
        attrs = {"ceil_mode": 0, "kernel_shape": [k, k], "pads": [p, p, p, p], "strides": [s, s]}
        (y,) = b.add(op, [x], [out_shape], attrs)
        return y, out_shape
    if isinstance(mod, nn.Flatten):
        a = mod.start_dim if mod.start_dim >= 0 else mod.start_dim + len(shape)
        if mod.end_dim not in (-1, len(shape) - 1):
            raise TypeError("only Flatten up to the last dimension exports as ONNX Flatten")
        out_shape = [int(np.prod(shape[:a])), int(np.prod(shape[a:]))]
        (y,) = b.add("Flatten", [x], [out_shape], {"axis": a})
        return y, out_shape
    if isinstance(mod, View):
        target = list(mod.shape)
        tgt = _reshape_parser(target, shape)
        c = b.const(np.asarray(target, dtype=np.int64))
        (y,) = b.add("Reshape", [x, c], [tgt])
        return y, tgt
    raise TypeError(f"module {type(mod).__name__} has no roseNNa export here")


class View(__import__("torch").nn.Module):
    """``x.view(x.size(0), *shape[1:])`` as a module, so a stack can hold it
    (exported as Reshape with target ``shape``, whose first entry is the export
    batch)."""

    def __init__(self, *shape):
        super().__init__()
        self.shape = shape

    def forward(self, x):
        return x.reshape(x.shape[0], *self.shape[1:])


def export_sequential(modules: Sequence, input_shape: Sequence[int]) -> Graph:
    """Graph of a feed-forward stack (Linear/act/Conv/pool/Flatten/View) with one input."""
    b = _Builder()
    x, shape = "input", list(input_shape)
    for m in modules:
        x, shape = _emit_module(b, m, x, shape)
    # the last node's output is the graph output
    last = b.nodes[-1]
    b.vi.pop(last.outputs[0], None)
    last.outputs[0] = "output"
    b.vi["output"] = shape
    return Graph(nodes=b.nodes, inputs=[("input", list(input_shape))], outputs=[("output", shape)],
                 initializers=b.inits, value_info=b.vi, constants=b.consts, true_weights=b.true_weights)


def export_lstm(lstms: Sequence, head: Sequence, batch: int, seq_len: int, mode: str = "hn_head",
                with_state: bool = True) -> Graph:
    """Graph of batch-first single-layer LSTMs chained one after the other, then a head.

    mode: 'hn_head'  head on the last LSTM's h_n.view(-1, H)  (goldenFiles/lstm_gemm_hid)
          'y'        the last LSTM's batch-first output Y    (goldenFiles/lstm_output)
          'y_head'   head on Y.view(-1, H)                     (goldenFiles/lstm_gemm)
          'cn'       the last LSTM's c_n                       (goldenFiles/lstm_cell)
    with_state: h0/c0 are graph inputs (one pair per LSTM, `hidden_state`/`cell_state`
    for the first, `hidden_state{k}`/`cell_state{k}` after); otherwise they are zero.
    """
    b = _Builder()
    I = lstms[0].input_size
    g_inputs = [("input", [batch, seq_len, I])]
    x, shape = "input", [batch, seq_len, I]
    yh = yc = None
    for li, lstm in enumerate(lstms):
        H = lstm.hidden_size
        (t0,) = b.add("Transpose", [x], [[seq_len, batch, shape[2]]], {"perm": [1, 0, 2]})
        w_ih, w_hh = _np32(lstm.weight_ih_l0), _np32(lstm.weight_hh_l0)
        b_ih, b_hh = _np32(lstm.bias_ih_l0), _np32(lstm.bias_hh_l0)
        # folded structure: W (1,4H,I), R (1,4H,H), B (1,8H); unfolded weights in torch order
        W = b.weight(w_ih, folded=w_ih.reshape(1, 4 * H, -1))
        R = b.weight(w_hh, folded=w_hh.reshape(1, 4 * H, H))
        B = b.name("w")
        b.inits[B] = np.concatenate([b_ih, b_hh]).reshape(1, 8 * H)
        b.true_weights += [b_ih, b_hh]
        ins = [t0, W, R, B]
        if with_state:
            hn, cn = ("hidden_state", "cell_state") if li == 0 else (f"hidden_state{li}", f"cell_state{li}")
            g_inputs += [(hn, [1, batch, H]), (cn, [1, batch, H])]
            ins += ["", hn, cn]
        y, yh, yc = b.add("LSTM", ins, [[seq_len, 1, batch, H], [1, batch, H], [1, batch, H]], {"hidden_size": H})
        if li + 1 < len(lstms) or mode in ("y", "y_head"):
            (s0,) = b.add("Squeeze", [y], [[seq_len, batch, H]], {"axes": [1]})
            (x,) = b.add("Transpose", [s0], [[batch, seq_len, H]], {"perm": [1, 0, 2]})
            shape = [batch, seq_len, H]
    H = lstms[-1].hidden_size
    if mode == "cn":
        out_name, out_shape = yc, [1, batch, H]
    elif mode == "y":
        out_name, out_shape = x, shape
    else:
        if mode == "hn_head":
            src, sshape = yh, [1, batch, H]
        else:
            src, sshape = x, shape
        c = b.const(np.asarray([-1, H], dtype=np.int64))
        tgt = _reshape_parser([-1, H], sshape)
        (x2,) = b.add("Reshape", [src, c], [tgt])
        shp = tgt
        for m in head:
            x2, shp = _emit_module(b, m, x2, shp)
        out_name, out_shape = x2, shp
    # rename the graph output
    for n in b.nodes:
        n.outputs = ["output" if o == out_name else o for o in n.outputs]
        n.inputs = ["output" if i == out_name else i for i in n.inputs]
    b.vi["output"] = b.vi.pop(out_name, out_shape)
    return Graph(nodes=b.nodes, inputs=g_inputs, outputs=[("output", out_shape)], initializers=b.inits,
                 value_info=b.vi, constants=b.consts, true_weights=b.true_weights)


def export_stacked_lstm(lstm, head: Sequence, batch: int, seq_len: int) -> Graph:
    """Graph of one batch-first nn.LSTM with num_layers >= 2, given (h0, c0) of
    shape (num_layers, N, H), with a head on the last layer's h_n (hn[-1]), as
    torch.onnx.export emits it (opset 10): the input Transpose; per layer a
    Slice of h0 and c0 along axis 0, the LSTM node, and a Squeeze of its output
    sequence as the next layer's input; h_n = Concat of the layers' h_n along
    axis 0; Gather(h_n, -1, axis 0) into the head."""
    b = _Builder()
    L, H, I = lstm.num_layers, lstm.hidden_size, lstm.input_size
    if L < 2 or not lstm.batch_first or lstm.bidirectional:
        raise TypeError("export_stacked_lstm takes a batch-first, one-direction nn.LSTM with num_layers >= 2")
    g_inputs = [("input", [batch, seq_len, I]), ("hidden_state", [L, batch, H]), ("cell_state", [L, batch, H])]
    (x,) = b.add("Transpose", ["input"], [[seq_len, batch, I]], {"perm": [1, 0, 2]})
    hns = []
    for k in range(L):
        starts, ends, axes = (b.const(np.asarray([v], dtype=np.int64)) for v in (k, k + 1, 0))
        (h_k,) = b.add("Slice", ["hidden_state", starts, ends, axes], [[1, batch, H]])
        starts, ends, axes = (b.const(np.asarray([v], dtype=np.int64)) for v in (k, k + 1, 0))
        (c_k,) = b.add("Slice", ["cell_state", starts, ends, axes], [[1, batch, H]])
        w_ih, w_hh = _np32(getattr(lstm, f"weight_ih_l{k}")), _np32(getattr(lstm, f"weight_hh_l{k}"))
        b_ih, b_hh = _np32(getattr(lstm, f"bias_ih_l{k}")), _np32(getattr(lstm, f"bias_hh_l{k}"))
        W = b.weight(w_ih, folded=w_ih.reshape(1, 4 * H, -1))
        R = b.weight(w_hh, folded=w_hh.reshape(1, 4 * H, H))
        B = b.name("w")
        b.inits[B] = np.concatenate([b_ih, b_hh]).reshape(1, 8 * H)
        b.true_weights += [b_ih, b_hh]
        y, yh, _ = b.add("LSTM", [x, W, R, B, "", h_k, c_k], [[seq_len, 1, batch, H], [1, batch, H], [1, batch, H]],
                         {"hidden_size": H})
        hns.append(yh)
        if k + 1 < L:
            (x,) = b.add("Squeeze", [y], [[seq_len, batch, H]], {"axes": [1]})
    (hn,) = b.add("Concat", hns, [[L, batch, H]], {"axis": 0})
    idx = b.const(np.asarray(-1, dtype=np.int64))
    (last,) = b.add("Gather", [hn, idx], [[batch, H]], {"axis": 0})
    out, shp = last, [batch, H]
    for m in head:
        out, shp = _emit_module(b, m, out, shp)
    for n in b.nodes:
        n.outputs = ["output" if o == out else o for o in n.outputs]
        n.inputs = ["output" if i == out else i for i in n.inputs]
    b.vi["output"] = b.vi.pop(out, shp)
    return Graph(nodes=b.nodes, inputs=g_inputs, outputs=[("output", shp)], initializers=b.inits, value_info=b.vi,
                 constants=b.consts, true_weights=b.true_weights)

"""ONNX front end without the `onnx` package: .onnx file -> roseNNa model files.

roseNNa's fLibrary/modelParserONNX.py loads a model with `onnx.load`, runs
`onnx.shape_inference.infer_shapes` and walks the graph (modelParserONNX.py:
25-69).  This module decodes the ONNX protobuf wire format directly (the
field numbers of onnx.proto's ModelProto, GraphProto, NodeProto,
AttributeProto, TensorProto and ValueInfoProto are the file format, so they
are the same here), infers intermediate shapes for the ops roseNNa handles
when the file carries none, and hands the graph to
:func:`rosenna_b200.writer.write_model_files`, which restates the parser's
node walk.  The command line mirrors the parser's:

    python -m rosenna_b200.onnx_file -f model.onnx [-w weights.onnx] [-i inferred.onnx] [-o dir]

`-w` is the unfolded export whose initializers supply the weight values in
order (modelParserONNX.py:27-33), `-i` a file whose value_info holds the
inferred shapes (:35-40).
"""
from __future__ import annotations

import argparse
import math
import struct
from collections import OrderedDict
from typing import Dict, List, Optional, Tuple

import numpy as np

from .writer import Graph, Node, write_model_files

# --------------------------------------------------------------------------
# protobuf wire format
# --------------------------------------------------------------------------


def _varint(b: bytes, i: int) -> Tuple[int, int]:
    r = sh = 0
    while True:
        if i >= len(b):
            raise ValueError("truncated varint")
        c = b[i]
        i += 1
        r |= (c & 0x7F) << sh
        sh += 7
        if c < 0x80:
            return r, i


def _fields(b: bytes) -> List[Tuple[int, int, object]]:
    """(field number, wire type, value) of every field of one message."""
    out = []
    i = 0
    n = len(b)
    while i < n:
        key, i = _varint(b, i)
        f, w = key >> 3, key & 7
        if w == 0:
            v, i = _varint(b, i)
        elif w == 1:
            v = b[i:i + 8]
            i += 8
        elif w == 5:
            v = b[i:i + 4]
            i += 4
        elif w == 2:
            ln, i = _varint(b, i)
            v = b[i:i + ln]
            i += ln
        else:
            raise ValueError(f"unsupported wire type {w}")
        if i > n:
            raise ValueError("truncated field")
        out.append((f, w, v))
    return out


def _signed(v: int) -> int:
    return v - (1 << 64) if v >= (1 << 63) else v


def _packed_varints(v, w) -> List[int]:
    if w == 0:
        return [_signed(v)]
    out, i = [], 0
    while i < len(v):
        x, i = _varint(v, i)
        out.append(_signed(x))
    return out


def _packed_fixed(v, w, fmt: str, size: int) -> List[float]:
    if w in (1, 5):
        return list(struct.unpack("<" + fmt, v))
    return list(struct.unpack("<%d%s" % (len(v) // size, fmt), v))


# TensorProto.DataType values used by models roseNNa reads
_DT = {1: np.float32, 6: np.int32, 7: np.int64, 11: np.float64, 9: np.bool_, 2: np.uint8, 3: np.int8}


def _tensor(b: bytes) -> Tuple[str, np.ndarray]:
    """TensorProto -> (name, array)."""
    dims: List[int] = []
    dt = 1
    name = ""
    raw = None
    fl: List[float] = []
    i64: List[int] = []
    i32: List[int] = []
    f64: List[float] = []
    for f, w, v in _fields(b):
        if f == 1:
            dims += _packed_varints(v, w)
        elif f == 2:
            dt = v
        elif f == 4:
            fl += _packed_fixed(v, w, "f", 4)
        elif f == 5:
            i32 += _packed_varints(v, w)
        elif f == 7:
            i64 += _packed_varints(v, w)
        elif f == 8:
            name = v.decode()
        elif f == 9:
            raw = bytes(v)
        elif f == 10:
            f64 += _packed_fixed(v, w, "d", 8)
        elif f == 14 and v == 1:
            raise ValueError(f"tensor {name}: external data is not supported")
    if dt not in _DT:
        raise ValueError(f"tensor {name}: data type {dt} is not supported")
    npdt = _DT[dt]
    if raw is not None:
        arr = np.frombuffer(raw, dtype=np.dtype(npdt).newbyteorder("<")).astype(npdt)
    elif dt == 1:
        arr = np.asarray(fl, dtype=np.float32)
    elif dt == 11:
        arr = np.asarray(f64, dtype=np.float64)
    elif dt == 7:
        arr = np.asarray(i64, dtype=np.int64)
    else:
        arr = np.asarray(i32, dtype=np.int64).astype(npdt)
    count = int(np.prod(dims)) if dims else 1
    if arr.size != count:
        raise ValueError(f"tensor {name}: {arr.size} values for dims {dims}")
    return name, arr.reshape(dims)


# AttributeProto.AttributeType
_A_FLOAT, _A_INT, _A_STRING, _A_TENSOR, _A_FLOATS, _A_INTS, _A_STRINGS = 1, 2, 3, 4, 6, 7, 8


def _attribute(b: bytes) -> Tuple[str, object]:
    name = ""
    typ = None
    vals: Dict[int, list] = {}
    for f, w, v in _fields(b):
        if f == 1:
            name = v.decode()
        elif f == 20:
            typ = v
        else:
            vals.setdefault(f, []).append((w, v))
    if typ is None:  # files older than the type field: the field that is present decides
        for f, t in ((2, _A_FLOAT), (3, _A_INT), (4, _A_STRING), (5, _A_TENSOR), (7, _A_FLOATS), (8, _A_INTS), (9, _A_STRINGS)):
            if f in vals:
                typ = t
                break
    if typ == _A_INT:
        w, v = vals.get(3, [(0, 0)])[0]
        return name, _signed(v)
    if typ == _A_FLOAT:
        w, v = vals.get(2, [(5, b"\0\0\0\0")])[0]
        return name, struct.unpack("<f", v)[0]
    if typ == _A_STRING:
        w, v = vals.get(4, [(2, b"")])[0]
        return name, bytes(v).decode("ascii")
    if typ == _A_INTS:
        out: List[int] = []
        for w, v in vals.get(8, []):
            out += _packed_varints(v, w)
        return name, out
    if typ == _A_FLOATS:
        out_f: List[float] = []
        for w, v in vals.get(7, []):
            out_f += _packed_fixed(v, w, "f", 4)
        return name, out_f
    if typ == _A_STRINGS:
        return name, [bytes(v).decode("ascii") for w, v in vals.get(9, [])]
    if typ == _A_TENSOR:
        return name, _tensor(vals[5][0][1])[1]
    raise ValueError(f"attribute {name}: type {typ} is not supported")


def _value_info(b: bytes) -> Tuple[str, List[int]]:
    """ValueInfoProto -> (name, dims); unknown or symbolic dims read as 0, as
    `dim.dim_value` does."""
    name = ""
    dims: List[int] = []
    for f, w, v in _fields(b):
        if f == 1:
            name = v.decode()
        elif f == 2:  # TypeProto
            for f2, w2, v2 in _fields(v):
                if f2 != 1:  # tensor_type
                    continue
                for f3, w3, v3 in _fields(v2):
                    if f3 != 2:  # shape
                        continue
                    for f4, w4, v4 in _fields(v3):
                        if f4 != 1:  # dim
                            continue
                        dv = 0
                        for f5, w5, v5 in _fields(v4):
                            if f5 == 1:
                                dv = _signed(v5)
                        dims.append(dv)
    return name, dims


class OnnxModel:
    """The parts of a ModelProto that the parser reads."""

    def __init__(self, data: bytes):
        graph = None
        for f, w, v in _fields(data):
            if f == 7:
                graph = v
        if graph is None:
            raise ValueError("no graph in the model file")
        self.nodes: List[Node] = []
        self.inputs: List[Tuple[str, List[int]]] = []
        self.outputs: List[Tuple[str, List[int]]] = []
        self.value_info: "OrderedDict[str, List[int]]" = OrderedDict()
        self.initializers: "OrderedDict[str, np.ndarray]" = OrderedDict()
        for f, w, v in _fields(graph):
            if f == 1:
                ins: List[str] = []
                outs: List[str] = []
                op = ""
                attrs: "OrderedDict[str, object]" = OrderedDict()
                for f2, w2, v2 in _fields(v):
                    if f2 == 1:
                        ins.append(v2.decode())
                    elif f2 == 2:
                        outs.append(v2.decode())
                    elif f2 == 4:
                        op = v2.decode()
                    elif f2 == 5:
                        k, a = _attribute(v2)
                        attrs[k] = a
                self.nodes.append(Node(op, ins, outs, dict(attrs)))
            elif f == 5:
                k, a = _tensor(v)
                self.initializers[k] = a
            elif f == 11:
                self.inputs.append(_value_info(v))
            elif f == 12:
                self.outputs.append(_value_info(v))
            elif f == 13:
                k, d = _value_info(v)
                self.value_info[k] = d

    @classmethod
    def load(cls, path: str) -> "OnnxModel":
        with open(path, "rb") as fh:
            return cls(fh.read())


# --------------------------------------------------------------------------
# shape inference for the ops the parser handles (stands in for
# onnx.shape_inference.infer_shapes when a file carries no value_info)
# --------------------------------------------------------------------------


def _conv_out(size: int, k: int, pb: int, pe: int, s: int, d: int = 1, ceil: bool = False) -> int:
    span = size + pb + pe - d * (k - 1) - 1
    return (math.ceil(span / s) if ceil else span // s) + 1


def _spatial_pads(attrs: dict, in_sp: List[int], ks: List[int], strides: List[int], dil: List[int]) -> List[int]:
    auto = str(attrs.get("auto_pad", "NOTSET"))
    nd = len(in_sp)
    if auto in ("SAME_UPPER", "SAME_LOWER"):
        pb, pe = [], []
        for i in range(nd):
            out = -(-in_sp[i] // strides[i])
            total = max(0, (out - 1) * strides[i] + dil[i] * (ks[i] - 1) + 1 - in_sp[i])
            lo = total // 2 if auto == "SAME_UPPER" else total - total // 2
            pb.append(lo)
            pe.append(total - lo)
        return pb + pe
    if auto == "VALID":
        return [0] * (2 * nd)
    return list(attrs.get("pads", [0] * (2 * nd)))


def _broadcast(a: List[int], b: List[int]) -> List[int]:
    n = max(len(a), len(b))
    a = [1] * (n - len(a)) + list(a)
    b = [1] * (n - len(b)) + list(b)
    return [max(x, y) if 1 in (x, y) else x for x, y in zip(a, b)]


def infer_shapes(m: OnnxModel, constants: Dict[str, np.ndarray]) -> Dict[str, List[int]]:
    """Shapes of every node output that can be inferred from the graph inputs,
    the initializers and the node attributes."""
    shapes: Dict[str, List[int]] = {k: list(v) for k, v in m.inputs}
    for k, v in m.initializers.items():
        shapes[k] = list(v.shape)
    for k, v in m.value_info.items():
        shapes.setdefault(k, list(v))

    def value(name):
        if name in m.initializers:
            return m.initializers[name]
        return constants.get(name)

    for nd in m.nodes:
        op, a = nd.op_type, nd.attrs
        ins = [shapes.get(x) for x in nd.inputs]
        outs: List[Optional[List[int]]] = []
        try:
            if op == "Constant":
                outs = [list(np.shape(a["value"]))]
            elif op in ("Relu", "Tanh", "Sigmoid", "Identity", "Dropout"):
                outs = [list(ins[0])]
            elif op == "Add" or op == "Mul" or op == "Sub":
                outs = [_broadcast(ins[0], ins[1])]
            elif op == "Gemm":
                x, w = ins[0], ins[1]
                rows = x[1] if a.get("transA", 0) else x[0]
                cols = w[0] if a.get("transB", 0) else w[1]
                outs = [[rows, cols]]
            elif op == "MatMul":
                x, w = list(ins[0]), list(ins[1])
                lead = _broadcast(x[:-2], w[:-2]) if len(x) > 2 or len(w) > 2 else []
                outs = [lead + [x[-2], w[-1]] if len(x) >= 2 else [w[-1]]]
            elif op == "Conv":
                x, w = ins[0], ins[1]
                sp = len(x) - 2
                ks = list(a.get("kernel_shape", w[2:]))
                st = list(a.get("strides", [1] * sp))
                dl = list(a.get("dilations", [1] * sp))
                pads = _spatial_pads(a, x[2:], ks, st, dl)
                outs = [[x[0], w[0]] + [_conv_out(x[2 + i], ks[i], pads[i], pads[sp + i], st[i], dl[i]) for i in range(sp)]]
            elif op in ("MaxPool", "AveragePool"):
                x = ins[0]
                sp = len(x) - 2
                ks = list(a["kernel_shape"])
                st = list(a.get("strides", [1] * sp))
                pads = _spatial_pads(a, x[2:], ks, st, [1] * sp)
                ceil = bool(a.get("ceil_mode", 0))
                outs = [[x[0], x[1]] + [_conv_out(x[2 + i], ks[i], pads[i], pads[sp + i], st[i], 1, ceil) for i in range(sp)]]
            elif op == "Reshape":
                x = ins[0]
                tgt = [int(v) for v in np.asarray(value(nd.inputs[1])).reshape(-1).tolist()]
                tgt = [x[i] if d == 0 else d for i, d in enumerate(tgt)]
                if -1 in tgt:
                    known = int(np.prod([d for d in tgt if d != -1]))
                    tgt[tgt.index(-1)] = int(np.prod(x)) // known
                outs = [tgt]
            elif op == "Flatten":
                x = ins[0]
                ax = int(a.get("axis", 1))
                ax = ax + len(x) if ax < 0 else ax
                outs = [[int(np.prod(x[:ax])), int(np.prod(x[ax:]))]]
            elif op == "Transpose":
                x = ins[0]
                perm = list(a.get("perm", list(range(len(x) - 1, -1, -1))))
                outs = [[x[p] for p in perm]]
            elif op in ("Squeeze", "Unsqueeze"):
                x = ins[0]
                if "axes" in a:
                    axes = list(a["axes"])
                elif len(nd.inputs) > 1:
                    axes = [int(v) for v in np.asarray(value(nd.inputs[1])).reshape(-1).tolist()]
                else:
                    axes = [i for i, d in enumerate(x) if d == 1]
                if op == "Squeeze":
                    axes = [ax + len(x) if ax < 0 else ax for ax in axes]
                    outs = [[d for i, d in enumerate(x) if i not in axes]]
                else:
                    r = len(x) + len(axes)
                    axes = sorted(ax + r if ax < 0 else ax for ax in axes)
                    o = list(x)
                    for ax in axes:
                        o.insert(ax, 1)
                    outs = [o]
            elif op == "Slice":
                x = list(ins[0])
                if len(nd.inputs) >= 3:  # opset >= 10: starts, ends[, axes[, steps]] as inputs
                    st = [int(v) for v in np.asarray(value(nd.inputs[1])).reshape(-1)]
                    en = [int(v) for v in np.asarray(value(nd.inputs[2])).reshape(-1)]
                    ax = ([int(v) for v in np.asarray(value(nd.inputs[3])).reshape(-1)]
                          if len(nd.inputs) > 3 and nd.inputs[3] else list(range(len(st))))
                else:
                    st, en = list(a["starts"]), list(a["ends"])
                    ax = list(a.get("axes", range(len(st))))
                for s_, e_, k in zip(st, en, ax):
                    k = k + len(x) if k < 0 else k
                    d = x[k]
                    lo = max(0, min(d, s_ + d if s_ < 0 else s_))
                    hi = max(lo, min(d, e_ + d if e_ < 0 else e_))
                    x[k] = hi - lo
                outs = [x]
            elif op == "Gather":
                x, idx = list(ins[0]), np.asarray(value(nd.inputs[1]))
                k = int(a.get("axis", 0))
                k = k + len(x) if k < 0 else k
                outs = [x[:k] + list(idx.shape) + x[k + 1:]]
            elif op == "Concat":
                k = int(a["axis"])
                x = list(ins[0])
                k = k + len(x) if k < 0 else k
                x[k] = sum(int(i[k]) for i in ins)
                outs = [x]
            elif op == "LSTM":
                x = ins[0]
                hidden = int(a["hidden_size"])
                dirs = 2 if str(a.get("direction", "forward")) == "bidirectional" else 1
                if int(a.get("layout", 0)):
                    outs = [[x[0], x[1], dirs, hidden], [x[0], dirs, hidden], [x[0], dirs, hidden]]
                else:
                    outs = [[x[0], dirs, x[1], hidden], [dirs, x[1], hidden], [dirs, x[1], hidden]]
        except (TypeError, KeyError, IndexError, ValueError):
            outs = []
        for name, shp in zip(nd.outputs, outs):
            if name and shp is not None and name not in shapes:
                shapes[name] = [int(d) for d in shp]
    return shapes


def load_graph(path: str, weights: Optional[str] = None, inferred: Optional[str] = None) -> Graph:
    """The graph the parser walks: structure from `path`, weight values from
    `weights` when given, intermediate shapes from `inferred` when given, else
    from the file's value_info completed by :func:`infer_shapes`."""
    m = OnnxModel.load(path)
    constants: Dict[str, np.ndarray] = {}
    for nd in m.nodes:  # modelParserONNX.py:63-65
        if nd.op_type == "Constant" and nd.attrs:
            constants[nd.outputs[0]] = np.asarray(list(nd.attrs.values())[0])
    if inferred:
        value_info = dict(OnnxModel.load(inferred).value_info)
    else:
        value_info = dict(m.value_info)
        graph_io = {k for k, _ in m.inputs} | {k for k, _ in m.outputs}
        for k, v in infer_shapes(m, constants).items():
            if k not in value_info and k not in graph_io and k not in m.initializers:
                value_info[k] = v
    true_weights = None
    if weights:
        true_weights = list(OnnxModel.load(weights).initializers.values())
    return Graph(nodes=m.nodes, inputs=list(m.inputs), outputs=list(m.outputs),
                 initializers=dict(m.initializers), value_info=value_info, constants=constants,
                 true_weights=true_weights)


def main(argv=None) -> None:
    ap = argparse.ArgumentParser(description="Write onnxModel.txt, onnxWeights.txt and variables.fpp for an .onnx model")
    ap.add_argument("--onnxfile", "-f", required=True, help=".onnx file of the trained model")
    ap.add_argument("--weights", "-w", help="unfolded export (do_constant_folding=False) holding the weights")
    ap.add_argument("--inferred", "-i", help=".onnx file with inferred shapes")
    ap.add_argument("--out", "-o", default=".", help="directory for the three files (default: the working directory)")
    args = ap.parse_args(argv)
    write_model_files(load_graph(args.onnxfile, args.weights, args.inferred), args.out)


if __name__ == "__main__":
    main()

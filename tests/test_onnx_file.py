"""The .onnx reader (rosenna_b200.onnx_file) without the onnx package.

Graphs are serialised here by a small protobuf encoder of the ONNX messages
(test infrastructure), decoded by the reader, and must give the same model
files as the in-memory graph; without value_info the reader's shape inference
must recover the shapes.  Where the reference tree exists, mnist.onnx must
decode to the committed mnist fixture."""
import os
import struct

import numpy as np
import pytest
import torch.nn as nn

from rosenna_b200 import onnx_file, writer
from rosenna_b200.writer import View
from tests import goldens

# ------------------------------------------------------------------ encoder


def _vint(v):
    v &= (1 << 64) - 1
    out = bytearray()
    while True:
        b = v & 0x7F
        v >>= 7
        if v:
            out.append(b | 0x80)
        else:
            out.append(b)
            return bytes(out)


def _key(f, w):
    return _vint((f << 3) | w)


def _ld(f, payload):
    return _key(f, 2) + _vint(len(payload)) + payload


def _varint_field(f, v):
    return _key(f, 0) + _vint(v)


def _tensor(name, arr, raw):
    arr = np.asarray(arr)
    dt = {np.dtype(np.float32): 1, np.dtype(np.int64): 7, np.dtype(np.float64): 11}[arr.dtype]
    out = b"".join(_varint_field(1, d) for d in arr.shape) + _varint_field(2, dt) + _ld(8, name.encode())
    if raw:
        out += _ld(9, arr.astype(arr.dtype.newbyteorder("<")).tobytes())
    elif dt == 1:
        out += _ld(4, struct.pack("<%df" % arr.size, *arr.reshape(-1).tolist()))
    elif dt == 7:
        out += _ld(7, b"".join(_vint(int(v)) for v in arr.reshape(-1)))
    else:
        out += _ld(10, struct.pack("<%dd" % arr.size, *arr.reshape(-1).tolist()))
    return out


def _attr(name, v):
    out = _ld(1, name.encode())
    if isinstance(v, str):
        return out + _ld(4, v.encode()) + _varint_field(20, 3)
    if isinstance(v, float):
        return out + _key(2, 5) + struct.pack("<f", v) + _varint_field(20, 1)
    if isinstance(v, (int, np.integer)):
        return out + _varint_field(3, int(v)) + _varint_field(20, 2)
    if isinstance(v, np.ndarray):
        return out + _ld(5, _tensor("", v, raw=True)) + _varint_field(20, 4)
    return out + _ld(8, b"".join(_vint(int(x)) for x in v)) + _varint_field(20, 7)


def _value_info(name, dims):
    dim_msgs = b"".join(_ld(1, _varint_field(1, d)) for d in dims)
    tensor_type = _varint_field(1, 1) + _ld(2, dim_msgs)
    return _ld(1, name.encode()) + _ld(2, _ld(1, tensor_type))


def encode(g, with_value_info=True, raw=True):
    nodes = b""
    for nd in g.nodes:
        body = b"".join(_ld(1, i.encode()) for i in nd.inputs) + b"".join(_ld(2, o.encode()) for o in nd.outputs)
        body += _ld(4, nd.op_type.encode())
        attrs = dict(nd.attrs)
        if nd.op_type == "Constant":
            attrs = {"value": np.asarray(g.constants[nd.outputs[0]])}
        body += b"".join(_ld(5, _attr(k, v)) for k, v in attrs.items())
        nodes += _ld(1, body)
    graph = nodes + _ld(2, b"g")
    graph += b"".join(_ld(5, _tensor(k, v, raw)) for k, v in g.initializers.items())
    graph += b"".join(_ld(11, _value_info(k, d)) for k, d in g.inputs)
    graph += b"".join(_ld(12, _value_info(k, d)) for k, d in g.outputs)
    if with_value_info:
        graph += b"".join(_ld(13, _value_info(k, d)) for k, d in g.value_info.items())
    return _varint_field(1, 7) + _ld(7, graph)


def _files(d):
    return {f: open(os.path.join(d, f)).read() for f in ("onnxModel.txt", "onnxWeights.txt", "variables.fpp")}


def _graphs():
    import torch

    torch.manual_seed(5)
    mlp = writer.export_sequential([nn.Linear(3, 8), nn.Tanh(), nn.Linear(8, 2), nn.Sigmoid()], [1, 3])
    cnn = writer.export_sequential([nn.Conv2d(1, 4, 3, padding=1), nn.ReLU(), nn.MaxPool2d(2, 2),
                                    nn.Conv2d(4, 6, 3, stride=2), nn.AvgPool2d(1), View(1, -1), nn.Linear(6, 3)],
                                   [1, 1, 8, 8])
    lstm = writer.export_lstm([nn.LSTM(4, 5, 1, batch_first=True)], [nn.Linear(5, 2)], 1, 6, mode="hn_head",
                              with_state=True)
    torch.manual_seed(6)
    cnn_flatten = writer.export_sequential([nn.Conv2d(1, 4, 3, padding=1), nn.ReLU(), nn.MaxPool2d(2, 2),
                                            nn.Flatten(), nn.Linear(64, 3)], [1, 1, 8, 8])
    torch.manual_seed(7)
    stacked = writer.export_stacked_lstm(nn.LSTM(3, 4, 2, batch_first=True), [nn.Linear(4, 2)], 1, 5)
    return {"mlp": mlp, "cnn": cnn, "lstm": lstm, "cnn_flatten": cnn_flatten, "stacked_lstm": stacked}


@pytest.mark.parametrize("raw", [True, False])
@pytest.mark.parametrize("name", ["mlp", "cnn", "lstm", "cnn_flatten", "stacked_lstm"])
def test_decoded_graph_writes_the_same_files(name, raw, tmp_path):
    g = _graphs()[name]
    (tmp_path / "m.onnx").write_bytes(encode(g, raw=raw))
    extra = {}
    if g.true_weights is not None:  # the unfolded export supplies the weight values in order
        gw = writer.Graph(nodes=[], inputs=[], outputs=[], value_info={},
                          initializers={f"w{i}": np.asarray(w) for i, w in enumerate(g.true_weights)})
        (tmp_path / "w.onnx").write_bytes(encode(gw, raw=raw))
        extra["weights"] = str(tmp_path / "w.onnx")
    writer.write_model_files(g, str(tmp_path / "direct"))
    writer.write_model_files(onnx_file.load_graph(str(tmp_path / "m.onnx"), **extra), str(tmp_path / "decoded"))
    assert _files(tmp_path / "direct") == _files(tmp_path / "decoded")


@pytest.mark.parametrize("name", ["mlp", "cnn", "lstm", "cnn_flatten", "stacked_lstm"])
def test_shape_inference_recovers_value_info(name, tmp_path):
    g = _graphs()[name]
    (tmp_path / "m.onnx").write_bytes(encode(g, with_value_info=False))
    m = onnx_file.OnnxModel.load(str(tmp_path / "m.onnx"))
    assert not m.value_info
    consts = {nd.outputs[0]: np.asarray(nd.attrs["value"]) for nd in m.nodes if nd.op_type == "Constant"}
    shapes = onnx_file.infer_shapes(m, consts)
    for k, dims in g.value_info.items():
        assert shapes.get(k) == list(dims), k


def test_inferred_file_supplies_the_shapes(tmp_path):
    g = _graphs()["cnn"]
    (tmp_path / "m.onnx").write_bytes(encode(g, with_value_info=False))
    (tmp_path / "i.onnx").write_bytes(encode(g))
    gi = onnx_file.load_graph(str(tmp_path / "m.onnx"), inferred=str(tmp_path / "i.onnx"))
    assert gi.value_info == {k: list(v) for k, v in g.value_info.items()}


def test_attribute_kinds_and_signed_ints():
    payload = b"".join(_ld(5, _attr(k, v)) for k, v in
                       [("i", -3), ("f", 0.5), ("s", "SAME_UPPER"), ("ints", [1, -1, 7]), ("t", np.arange(4.0))])
    node = _ld(1, b"x") + _ld(2, b"y") + _ld(4, b"Op") + payload
    model = _varint_field(1, 7) + _ld(7, _ld(1, node))
    m = onnx_file.OnnxModel(model)
    a = m.nodes[0].attrs
    assert a["i"] == -3 and a["f"] == 0.5 and a["s"] == "SAME_UPPER" and a["ints"] == [1, -1, 7]
    np.testing.assert_array_equal(a["t"], np.arange(4.0))
    assert list(a) == ["i", "f", "s", "ints", "t"]  # attribute order is kept (the MaxPool size field depends on it)


def test_truncated_file_is_an_error():
    with pytest.raises(ValueError):
        onnx_file.OnnxModel(encode(_graphs()["mlp"])[:-7])


# the roseNNa checkout, named by ROSENNA_REFERENCE_DIR (the test skips without it)
REFERENCE_MNIST = os.path.join(os.environ.get("ROSENNA_REFERENCE_DIR", ""), "goldenFiles", "mnist")


@pytest.mark.skipif(not os.environ.get("ROSENNA_REFERENCE_DIR") or not os.path.isdir(REFERENCE_MNIST),
                    reason="ROSENNA_REFERENCE_DIR does not name a roseNNa checkout")
def test_mnist_onnx_decodes_to_the_committed_fixture(tmp_path):
    g = onnx_file.load_graph(os.path.join(REFERENCE_MNIST, "mnist.onnx"))
    writer.write_model_files(g, str(tmp_path))
    assert _files(tmp_path) == _files(goldens.case_dir("mnist"))


def test_command_line_writes_the_three_files(tmp_path):
    g = _graphs()["mlp"]
    (tmp_path / "m.onnx").write_bytes(encode(g))
    onnx_file.main(["-f", str(tmp_path / "m.onnx"), "-o", str(tmp_path / "out")])
    writer.write_model_files(g, str(tmp_path / "direct"))
    assert _files(tmp_path / "out") == _files(tmp_path / "direct")


def test_flatten_writes_the_files_of_a_view(tmp_path):
    """nn.Flatten (ONNX Flatten, which modelParserONNX.py:519-523 passes through
    unwritten) is written as the variable-form Reshape entry x.view(N, -1) gives:
    the same variables.fpp and weights; onnxModel.txt differs only by the view's
    Constant node (its node count and its name line)."""
    import torch

    def stack(flat):
        torch.manual_seed(9)
        mods = [nn.Conv2d(2, 3, 3, padding=1), nn.ReLU(), nn.AvgPool2d(2, 2)]
        return mods + [nn.Flatten() if flat else View(1, -1), nn.Linear(27, 4)]

    writer.write_model_files(writer.export_sequential(stack(True), [1, 2, 6, 6]), str(tmp_path / "f"))
    writer.write_model_files(writer.export_sequential(stack(False), [1, 2, 6, 6]), str(tmp_path / "v"))
    f, v = _files(tmp_path / "f"), _files(tmp_path / "v")
    assert f["variables.fpp"] == v["variables.fpp"] and f["onnxWeights.txt"] == v["onnxWeights.txt"]
    fl, vl = f["onnxModel.txt"].splitlines(), v["onnxModel.txt"].splitlines()
    assert int(vl[0]) == int(fl[0]) + 1 and [x for x in vl[1:] if x != "Constant"] == fl[1:]

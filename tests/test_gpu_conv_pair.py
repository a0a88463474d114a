"""Two tensor-core convolutions in one kernel (conv_pair_tc_kernel): a
one-channel conv(+ReLU)+pool whose pooled output only the next conv(+ReLU)+pool
reads, with that output passed through a small per-CTA buffer instead of a
batch-sized array.  Checked against the fp64 oracle within the limits of
oracle/parity.py, and bit for bit against the same plan run as two
conv_tc_kernel launches (ROSENNA_CONV_FUSE=0): both compute the same products
in the same order, so the fused kernel changes where the intermediate lives,
not its value.

Shapes: the CNN workload (1x28x28, conv 1->8 pad 1 + max pool, conv 8->16
pad 1 + avg pool) at batches with partial tiles, a batch where CTAs split
tiles at band boundaries, paddings 0..2 on either conv, both pool kinds on
either conv, 5..8 channels between the convs, 9..16 output channels, and
images small enough that a tile has a single band."""
import numpy as np
import pytest
import torch
import torch.nn as nn

from oracle.oracle import OracleModel
from rosenna_b200 import api, workloads, writer
from tests.test_gpu_parity import assert_close

pytestmark = pytest.mark.gpu


@pytest.fixture(autouse=True)
def _device():
    assert torch.cuda.is_available(), "gpu tests need a CUDA device"
    api.set_devices([0])
    yield
    api.finalize()


def _run(model_dir, ins, fuse, monkeypatch):
    monkeypatch.setenv("ROSENNA_CONV_FUSE", "1" if fuse else "0")
    api.initialize(model_dir)
    desc = api.plan_description()
    assert ("conv_pair_tc" in desc) == fuse, desc
    out = api.use_model_rows(ins)[0]
    api.finalize()
    return out


def test_cnn_workload_pair(tmp_path, monkeypatch):
    workloads.write_model("cnn", str(tmp_path))
    oracle = OracleModel(str(tmp_path))
    for n in (1, 37, 128, 129, 1000, 4099, 19001):
        ins = workloads.make_inputs("cnn", n, seed_offset=57 + n)
        fused = _run(str(tmp_path), ins, True, monkeypatch)
        two = _run(str(tmp_path), ins, False, monkeypatch)
        np.testing.assert_array_equal(fused, two, err_msg=f"cnn n={n}: fused vs two kernels")
        sel = np.arange(n) if n <= 4099 else np.unique(np.linspace(0, n - 1, 2048).astype(np.int64))
        ref = oracle.run_batched(len(sel), [x[:, sel] for x in ins])[0]
        assert_close(fused[:, sel], ref.reshape(fused[:, sel].shape), f"cnn pair n={n}")


PAIRS = [  # (H, pad1, pool1, C2, OC2, pad2, pool2)
    (28, 1, "max", 8, 16, 1, "avg"), (28, 1, "avg", 8, 16, 1, "max"), (26, 0, "max", 8, 12, 1, "max"),
    (20, 1, "avg", 6, 16, 0, "avg"), (14, 2, "max", 8, 10, 2, "avg"), (12, 1, "max", 5, 9, 2, "max"),
    (8, 1, "avg", 7, 16, 1, "avg"), (6, 0, "max", 8, 16, 1, "max"),
]


@pytest.mark.parametrize("H,pad1,pool1,C2,OC2,pad2,pool2", PAIRS)
def test_pair_shapes(H, pad1, pool1, C2, OC2, pad2, pool2, tmp_path, monkeypatch):
    torch.manual_seed(H * 31 + pad1 * 7 + C2 * 3 + OC2 + pad2)
    c1 = nn.Conv2d(1, C2, 3, padding=pad1)
    c2 = nn.Conv2d(C2, OC2, 3, padding=pad2)
    for c in (c1, c2):
        nn.init.uniform_(c.weight, -0.5, 0.5)
        nn.init.uniform_(c.bias, -0.1, 0.1)
    pl = {"max": nn.MaxPool2d, "avg": nn.AvgPool2d}
    mods = [c1, nn.ReLU(), pl[pool1](2, 2), c2, nn.ReLU(), pl[pool2](2, 2)]
    g = writer.export_sequential(mods, [1, 1, H, H])
    writer.write_model_files(g, str(tmp_path))
    oracle = OracleModel(str(tmp_path))
    for n in (1, 129, 1000):
        ins = [np.random.default_rng(n + H).uniform(-1, 1, size=(H * H, n)).astype(np.float32)]
        fused = _run(str(tmp_path), ins, True, monkeypatch)
        two = _run(str(tmp_path), ins, False, monkeypatch)
        np.testing.assert_array_equal(fused, two, err_msg=f"{H}x{H} n={n}: fused vs two kernels")
        ref = oracle.run_batched(n, ins)[0]
        assert_close(fused, ref.reshape(fused.shape), f"pair {H}x{H} pad {pad1},{pad2} {pool1},{pool2} "
                                                       f"C2={C2} OC2={OC2} n={n}")


def test_pair_device_entry_matches_host(tmp_path, monkeypatch):
    """The device entry point (slot 0's buffer, caller's stream) and the host
    entry point (chunks over four streams, a buffer per stream) agree."""
    monkeypatch.setenv("ROSENNA_CONV_FUSE", "1")
    workloads.write_model("cnn", str(tmp_path))
    api.initialize(str(tmp_path))
    n = 40000
    ins = workloads.make_inputs("cnn", n, seed_offset=5)
    host = api.use_model_rows(ins)[0]
    d_in = [torch.from_numpy(x).cuda() for x in ins]
    d_out = torch.empty(host.shape, dtype=torch.float32, device="cuda")
    api.use_model_device(n, [x.data_ptr() for x in d_in], [d_out.data_ptr()],
                         torch.cuda.current_stream().cuda_stream)
    torch.cuda.synchronize()
    np.testing.assert_array_equal(d_out.cpu().numpy(), host)

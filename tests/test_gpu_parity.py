"""Parity of the CUDA engine (through the C ABI) with the fp64 oracle and the
golden fixtures.  Limits (fp32 engine against fp64 reference, oracle/parity.py):
max abs error <= 1e-5 over every element (the reference checker's own bound,
test/testChecker.py:14-17) and max rel error <= 1e-4 over the elements with
|ref| >= 0.1; both maxima are printed on a pass."""
import os

import numpy as np
import pytest
import torch

from oracle import parity
from oracle.oracle import OracleModel
from rosenna_b200 import api, workloads
from tests import goldens

pytestmark = pytest.mark.gpu

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))


def assert_close(out, ref, what=""):
    """Both limits of oracle/parity.py; prints both maxima (pytest -s / -rP)."""
    r = parity.compare(out, ref)
    print(f"{what}: {parity.describe(r)}")
    assert r["ok"], f"{what}: {parity.describe(r)}"
    return r


@pytest.fixture(autouse=True)
def _device():
    assert torch.cuda.is_available(), "gpu tests need a CUDA device"
    api.set_devices([0])
    yield
    api.finalize()


@pytest.mark.parametrize("case", goldens.cases())
def test_golden_case_at_export_batch(case):
    """Each reference case at its export shapes against PyTorch's fp64 output."""
    api.initialize(goldens.case_dir(case))
    ins = goldens.inputs(case)
    specs = api.input_specs()
    n = ins[0].shape[specs[0][1]]
    out = api.use_model(ins, n=n)[0]
    assert api.last_launch_count() > 0
    assert_close(out, goldens.golden(case), case)


@pytest.mark.parametrize("case", goldens.cases())
def test_golden_case_through_fixed_shape_use_model(case):
    """roseNNa's own entry point, use_model(i0,..,o0,..) on fp64 arrays of the
    export shapes (the C symbol a fixed-shape caller links against)."""
    import ctypes

    api.initialize(goldens.case_dir(case))
    ins = [np.asfortranarray(np.asarray(x, dtype=np.float64).reshape(s, order="A"))
           for x, (s, _) in zip(goldens.inputs(case), api.input_specs())]
    outs = [np.zeros(s, dtype=np.float64, order="F") for s, _ in api.output_specs()]
    L = api.lib()
    L.use_model(*[ctypes.c_void_p(a.ctypes.data) for a in ins + outs])
    assert L.rosenna_last_status() == 0, api.lib().rosenna_last_error()
    assert api.last_launch_count() > 0
    assert_close(outs[0], goldens.golden(case), case)


BATCHED_CASES = [c for c in goldens.cases() if c not in ("conv_basic", "lstm_gemm")]


@pytest.mark.parametrize("case", BATCHED_CASES)
@pytest.mark.parametrize("n", [1, 3, 129, 1000])
def test_golden_case_batched(case, n):
    """The reference case widened to a batch of n random samples, against the
    oracle calling use_model once per sample."""
    d = goldens.case_dir(case)
    api.initialize(d)
    rng = np.random.default_rng(n)
    rows = [int(np.prod(s)) // s[b] for s, b in api.input_specs()]
    ins = [rng.uniform(-1.5, 1.5, size=(r, n)).astype(np.float32) for r in rows]
    out = api.use_model_rows(ins)[0]
    ref = OracleModel(d).run_batched(n, ins)[0]
    assert_close(out, ref.reshape(out.shape), f"{case} n={n}")


def test_merged_batch_output_runs_only_at_batch_one():
    """lstm_gemm reshapes (N,T,H) to (N*T,H): its output mixes samples, so only n=1 runs."""
    api.initialize(goldens.case_dir("lstm_gemm"))
    ins = [np.ones((3, 2, 5), np.float32), np.ones((1, 3, 2), np.float32), np.ones((1, 3, 2), np.float32)]
    with pytest.raises(api.RosennaError) as e:
        api.use_model(ins, n=3)
    assert e.value.code == api.ERR_UNSUPPORTED


@pytest.mark.parametrize("name", list(workloads.WORKLOADS))
@pytest.mark.parametrize("n", [1, 7, 1000, 4099])
def test_workload_parity(name, n, tmp_path):
    workloads.write_model(name, str(tmp_path))
    api.initialize(str(tmp_path))
    ins = workloads.make_inputs(name, n, seed_offset=n)
    out = api.use_model_rows(ins)[0]
    ref = OracleModel(str(tmp_path)).run_batched(n, ins)[0]
    assert_close(out, ref.reshape(out.shape), f"{name} n={n}")


@pytest.mark.parametrize("name", ["small_mlp", "wide_mlp", "lstm", "cnn"])
def test_device_path_matches_host_path(name, tmp_path):
    workloads.write_model(name, str(tmp_path))
    api.initialize(str(tmp_path))
    n = 5003
    ins = workloads.make_inputs(name, n, seed_offset=11)
    host = api.use_model_rows(ins)[0]
    dins = [torch.from_numpy(x).cuda() for x in ins]
    dout = torch.zeros(host.shape, dtype=torch.float32, device="cuda")
    api.use_model_device(n, [x.data_ptr() for x in dins], [dout.data_ptr()], torch.cuda.current_stream().cuda_stream)
    torch.cuda.synchronize()
    assert np.array_equal(dout.cpu().numpy(), host)


def test_large_batch_small_mlp_chunks_and_tails(tmp_path):
    """More samples than one host chunk (2^20), with an odd tail."""
    workloads.write_model("small_mlp", str(tmp_path))
    api.initialize(str(tmp_path))
    n = (1 << 20) + 333
    ins = workloads.make_inputs("small_mlp", n, seed_offset=3)
    out = api.use_model_rows(ins)[0]
    ref = OracleModel(str(tmp_path)).run_batched(n, ins)[0]
    assert_close(out, ref.reshape(out.shape), "small_mlp large")


def test_fp64_entry_point(tmp_path):
    workloads.write_model("small_mlp", str(tmp_path))
    api.initialize(str(tmp_path))
    ins = workloads.make_inputs("small_mlp", 100)
    o32 = api.use_model_rows(ins)[0]
    x64 = np.asfortranarray(ins[0].astype(np.float64).T)  # logical (n, 10), Fortran order
    o64 = api.use_model([x64], n=100, dtype=np.float64)[0]
    assert np.array_equal(o64.T.astype(np.float32), o32)


@pytest.mark.parametrize("name", ["lstm", "wide_mlp", "cnn"])
def test_multi_gpu_split_matches(name, tmp_path):
    """rosenna_use_model_f32 split over the visible GPUs (contiguous sample
    ranges, weights and tensor maps per device) matches the oracle."""
    count = torch.cuda.device_count()
    if count < 2:
        pytest.skip("one GPU visible")
    api.set_devices(list(range(min(count, 4))))
    workloads.write_model(name, str(tmp_path))
    api.initialize(str(tmp_path))
    n = 10007
    ins = workloads.make_inputs(name, n, seed_offset=5)
    out = api.use_model_rows(ins)[0]
    ref = OracleModel(str(tmp_path)).run_batched(n, ins)[0]
    assert_close(out, ref.reshape(out.shape), f"{name} multi-gpu")


@pytest.mark.parametrize("path", ["tc", "tc_notail", "ffma"])
@pytest.mark.parametrize("name", ["small_mlp", "wide_mlp", "cnn"])
def test_mlp_kernel_paths(name, path, tmp_path, monkeypatch):
    """Both MLP kernels (tcgen05 3xTF32 and FFMA) on every MLP chain shape; the
    tensor-core kernel with its narrow last layer on the CUDA cores (default)
    and on the tensor cores."""
    monkeypatch.setenv("ROSENNA_MLP_PATH", "ffma" if path == "ffma" else "tc")
    monkeypatch.setenv("ROSENNA_TC_TAIL", "0" if path == "tc_notail" else "1")
    workloads.write_model(name, str(tmp_path))
    api.initialize(str(tmp_path))
    desc = api.plan_description()
    assert ("mlp_tc" in desc) == (path != "ffma"), desc
    for n in (129, 4099):
        ins = workloads.make_inputs(name, n, seed_offset=7 + n)
        out = api.use_model_rows(ins)[0]
        ref = OracleModel(str(tmp_path)).run_batched(n, ins)[0]
        assert_close(out, ref.reshape(out.shape), f"{name} {path} n={n}")


@pytest.mark.parametrize("path", ["default", "tc", "tc_unfused", "ffma"])
@pytest.mark.parametrize("name", ["lstm", "lstm2"])
def test_lstm_kernel_paths(name, path, tmp_path, monkeypatch):
    """The LSTM kernels on both LSTM workloads: by default the dual-tile
    tcgen05 kernel (4H = 128) and the fused two-layer tcgen05 kernel (H = 64);
    the tcgen05 kernel that splits one tile's gates between the column groups,
    with and without the two-layer fusion; the FFMA kernel."""
    if path == "default":
        monkeypatch.delenv("ROSENNA_LSTM_PATH", raising=False)
    else:
        monkeypatch.setenv("ROSENNA_LSTM_PATH", "ffma" if path == "ffma" else "tc")
    monkeypatch.setenv("ROSENNA_LSTM2_FUSE", "0" if path == "tc_unfused" else "1")
    workloads.write_model(name, str(tmp_path))
    api.initialize(str(tmp_path))
    desc = api.plan_description()
    assert ("lstm_tc" in desc) == (path != "ffma"), desc
    assert ("lstm_tc_dual" in desc) == (name == "lstm" and path == "default"), desc
    assert ("lstm2_tc" in desc) == (name == "lstm2" and path in ("default", "tc")), desc
    for n in (1, 129, 1000, 4099):
        ins = workloads.make_inputs(name, n, seed_offset=3 + n)
        out = api.use_model_rows(ins)[0]
        ref = OracleModel(str(tmp_path)).run_batched(n, ins)[0]
        assert_close(out, ref.reshape(out.shape), f"{name} {path} n={n}")


@pytest.mark.parametrize("conv_path", ["tiled", "direct"])
def test_cnn_conv_paths(conv_path, tmp_path):
    """The tiled conv+pool kernel and the per-element one on the CNN workload and
    the small golden CNN (run in a child process: the path is fixed at load)."""
    import subprocess, sys, textwrap
    code = textwrap.dedent(f"""
        import sys
        sys.path.insert(0, {repr(ROOT)})
        from rosenna_b200 import api, workloads
        from oracle.oracle import OracleModel
        from tests import goldens
        from tests.test_gpu_parity import assert_close
        api.set_devices([0])
        workloads.write_model('cnn', {repr(str(tmp_path))})
        api.initialize({repr(str(tmp_path))})
        for n in (1, 37, 1000):
            ins = workloads.make_inputs('cnn', n, seed_offset=11 + n)
            out = api.use_model_rows(ins)[0]
            ref = OracleModel({repr(str(tmp_path))}).run_batched(n, ins)[0]
            assert_close(out, ref.reshape(out.shape), f'cnn {conv_path} n={{n}}')
        d = goldens.case_dir('cnn_small')
        api.initialize(d)
        out = api.use_model(goldens.inputs('cnn_small'), n=1)[0]
        assert_close(out, goldens.golden('cnn_small'), 'cnn_small {conv_path}')
        print('ok')
    """)
    env = dict(os.environ, ROSENNA_CONV_PATH=conv_path)
    r = subprocess.run([sys.executable, "-c", code], env=env, capture_output=True, text=True, timeout=600)
    assert r.returncode == 0 and "ok" in r.stdout, r.stdout + r.stderr


@pytest.mark.parametrize("tail", ["1", "0"])
@pytest.mark.parametrize("case", ["gemm_small", "gemm_big", "batchnet", "droplet", "lstm_gemm_hid"])
def test_golden_mlps_on_tensor_cores(case, tail, monkeypatch):
    monkeypatch.setenv("ROSENNA_MLP_PATH", "tc")
    monkeypatch.setenv("ROSENNA_TC_TAIL", tail)
    d = goldens.case_dir(case)
    api.initialize(d)
    assert "mlp_tc" in api.plan_description()
    ins = goldens.inputs(case)
    out = api.use_model(ins, n=1)[0]
    assert_close(out, goldens.golden(case), case)
    n = 1000
    rng = np.random.default_rng(5)
    rows = [int(np.prod(s)) // s[b] for s, b in api.input_specs()]
    xs = [rng.uniform(-1.5, 1.5, size=(r, n)).astype(np.float32) for r in rows]
    out = api.use_model_rows(xs)[0]
    ref = OracleModel(d).run_batched(n, xs)[0]
    assert_close(out, ref.reshape(out.shape), f"{case} tc n={n}")


@pytest.mark.parametrize("ks,pool,pk", [(3, None, 1), (3, "max", 3), (3, "avg", 3), (5, None, 1), (5, "max", 2),
                                        (5, "avg", 2), (5, "max", 3)])
def test_conv_kernel_shapes(ks, pool, pk, tmp_path):
    """Every conv+pool kernel instantiation (3x3 and 5x5 kernels, pool windows
    1-3) on an odd image (border items), batches with partial warps, against
    the oracle."""
    import torch.nn as nn
    from rosenna_b200 import writer

    torch.manual_seed(ks * 10 + pk)
    mods = [nn.Conv2d(3, 10, ks, padding=ks // 2), nn.ReLU()]
    if pool:
        mods.append((nn.MaxPool2d if pool == "max" else nn.AvgPool2d)(pk, pk))
    g = writer.export_sequential(mods, [1, 3, 11, 11])
    writer.write_model_files(g, str(tmp_path))
    api.initialize(str(tmp_path))
    assert "conv" in api.plan_description()
    for n in (1, 45, 1000):
        ins = [np.random.default_rng(n).uniform(-1, 1, size=(3 * 11 * 11, n)).astype(np.float32)]
        out = api.use_model_rows(ins)[0]
        ref = OracleModel(str(tmp_path)).run_batched(n, ins)[0]
        assert_close(out, ref.reshape(out.shape), f"k={ks} {pool}{pk} n={n}")

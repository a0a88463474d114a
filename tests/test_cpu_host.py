"""Host-side tests that need no GPU: the C-ABI library, the plan builder, the
model-file reader/writer, error statuses, and the oracle on the workloads."""
import os
import re
import shutil

import numpy as np
import pytest

from oracle.oracle import OracleModel
from rosenna_b200 import api, workloads
from tests import goldens

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))


def test_library_exports_every_declared_symbol():
    with open(os.path.join(ROOT, "include", "rosenna.h")) as f:
        header = f.read()
    declared = set(re.findall(r"^\s*(?:void|int|int64_t|const char \*)\s*\*?(\w+)\(", header, re.M))
    assert declared == set(api.EXPORTS)
    L = api.lib()
    for name in declared:
        assert hasattr(L, name), name


@pytest.mark.parametrize("case", goldens.cases())
def test_plan_builds_for_golden_case(case):
    desc = api.check_model(goldens.case_dir(case))
    assert desc.strip()


def test_plan_fuses_the_workloads(tmp_path):
    expect = {
        "small_mlp": ["mlp b0->b1 [10x64:tanh 64x64:tanh 64x64:tanh 64x5]"],
        "wide_mlp": ["mlp b0->b1 [16x256:relu 256x256:relu 256x256:relu 256x256:relu 256x256:relu 256x8]"],
        "lstm": ["lstm b0 T=50 I=8 H=32", "mlp"],
        "cnn": ["conv", "relu maxpool k=2 s=2 -> 14x14", "relu avgpool k=2 s=2 -> 7x7", "mlp"],
        "lstm2": ["deinterleave", "lstm b0 T=100 I=12 H=64", "T=100 I=64 H=64", "mlp"],
    }
    for name, parts in expect.items():
        d = tmp_path / name
        workloads.write_model(name, str(d))
        desc = api.check_model(str(d))
        for p in parts:
            assert p in desc, (name, desc)


def test_initialize_statuses(tmp_path):
    # missing files: I/O error; no GPU here: no-device error; state error before init
    with pytest.raises(api.RosennaError) as e:
        api.initialize(str(tmp_path / "nope"))
    assert e.value.code == api.ERR_IO
    with pytest.raises(api.RosennaError) as e:
        api.use_model([np.zeros((1, 2), np.float32)])
    assert e.value.code == api.ERR_STATE


def test_fixed_shape_use_model_before_initialize_is_a_state_error():
    import ctypes

    api.finalize()
    L = api.lib()
    L.use_model(ctypes.c_void_p(0), ctypes.c_void_p(0))  # roseNNa's own two-array call form
    assert L.rosenna_last_status() == api.ERR_STATE


@pytest.mark.parametrize("own_prototype", [True, False])
def test_header_serves_fixed_shape_callers(own_prototype, tmp_path):
    """A C file may declare use_model with its model's own argument count (as
    the reference's examples do) or take the header's declaration."""
    if not shutil.which("gcc"):
        pytest.skip("no C compiler")
    src = tmp_path / "caller.c"
    proto = "#define ROSENNA_NO_LEGACY_USE_MODEL\n" if own_prototype else ""
    decl = "void use_model(double *i0, double *o0);\n" if own_prototype else ""
    call = "use_model(x, y);" if own_prototype else "use_model(x, y, 0, 0, 0, 0, 0, 0, 0, 0, 0, 0, 0, 0, 0, 0);"
    src.write_text(proto + '#include "rosenna.h"\n' + decl +
                   "void run(double *x, double *y) { initialize(); " + call + " }\n")
    import subprocess

    r = subprocess.run(["gcc", "-std=c99", "-Wall", "-Werror", "-fsyntax-only", "-I", os.path.join(ROOT, "include"),
                        str(src)], capture_output=True, text=True)
    assert r.returncode == 0, r.stderr


def test_initialize_without_gpu_reports_no_device():
    import torch

    if torch.cuda.is_available():
        pytest.skip("a GPU is present")
    with pytest.raises(api.RosennaError) as e:
        api.initialize(goldens.case_dir("gemm_small"))
    assert e.value.code == api.ERR_NO_DEVICE


def test_malformed_and_unsupported_models(tmp_path):
    src = goldens.case_dir("gemm_small")
    d = tmp_path / "m"
    shutil.copytree(src, d)
    # truncated weights file
    with open(d / "onnxWeights.txt", "w") as f:
        f.write("0.5 0.25\n")
    with pytest.raises(api.RosennaError) as e:
        api.check_model(str(d))
    assert e.value.code == api.ERR_FORMAT
    # forms the engine does not batch: an unknown op, a product of two per-sample values
    for k, entry in enumerate(["('Softmax', ['input'], [2])", "('MatMul', ['input', 'input'], [2])"]):
        u = tmp_path / f"u{k}"
        shutil.copytree(src, u)
        v = (u / "variables.fpp").read_text().replace("('Relu', ['input'], [2])", entry, 1)
        (u / "variables.fpp").write_text(v)
        with pytest.raises(api.RosennaError) as e:
            api.check_model(str(u))
        assert e.value.code == api.ERR_UNSUPPORTED, entry
    # a broken variables.fpp literal
    shutil.copytree(src, tmp_path / "b")
    (tmp_path / "b" / "variables.fpp").write_text("#:set architecture = [('Gemm', ['input', 1], None\n")
    with pytest.raises(api.RosennaError) as e:
        api.check_model(str(tmp_path / "b"))
    assert e.value.code == api.ERR_FORMAT


@pytest.mark.parametrize("name", list(workloads.WORKLOADS))
def test_oracle_matches_torch_on_workloads(name, tmp_path):
    mod = workloads.write_model(name, str(tmp_path))
    n = 5
    ins = workloads.make_inputs(name, n)
    out = OracleModel(str(tmp_path)).run_batched(n, ins)[0]
    ref = workloads.torch_reference(name, mod, ins)[0]
    np.testing.assert_allclose(out.reshape(ref.shape), ref, rtol=0, atol=1e-12)


def test_writer_weights_round_trip(tmp_path):
    """Values printed by the writer read back to the exact fp32 weights (modelParserONNX.py:82-86)."""
    import torch

    mod = workloads.write_model("small_mlp", str(tmp_path))
    lines = (tmp_path / "onnxWeights.txt").read_text().splitlines()
    w0 = np.array([float(v) for v in lines[0].split()])
    ref = mod[0].weight.detach().numpy().astype(np.float64).flatten(order="F")
    assert np.array_equal(w0, ref)
    assert torch.float32 == mod[0].weight.dtype

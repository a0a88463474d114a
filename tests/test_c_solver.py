"""The example C solver (rosenna_b200/examples/solver.c) compiled with gcc,
linked against librosenna_b200.so and run the way examples/cAPI.c runs
roseNNa: initialize() on the model files in the working directory, then a
batched use_model through the C ABI.  Without a GPU it must report the
no-device status; on a GPU its first sample must match the fp64 oracle."""
import os
import shutil
import subprocess

import numpy as np
import pytest

from oracle import parity
from oracle.oracle import OracleModel
from rosenna_b200 import api
from tests import goldens

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
LIBDIR = os.path.join(ROOT, "rosenna_b200")


def build_solver(tmp_path):
    if not shutil.which("gcc"):
        pytest.skip("no C compiler")
    api.lib()  # the engine library exists
    exe = str(tmp_path / "solver")
    r = subprocess.run(["gcc", "-std=c99", "-Wall", "-Werror", os.path.join(LIBDIR, "examples", "solver.c"),
                        "-I", os.path.join(ROOT, "include"), "-L", LIBDIR, "-lrosenna_b200",
                        f"-Wl,-rpath,{LIBDIR}", "-o", exe], capture_output=True, text=True)
    assert r.returncode == 0, r.stderr
    return exe


def run_in_case(exe, tmp_path, case, n):
    d = tmp_path / case
    shutil.copytree(goldens.case_dir(case), d)
    return subprocess.run([exe, str(n)], cwd=str(d), capture_output=True, text=True, timeout=300)


def test_c_solver_links_and_reports_no_device(tmp_path):
    import torch

    if torch.cuda.is_available():
        pytest.skip("a GPU is present (the gpu test runs the solver)")
    exe = build_solver(tmp_path)
    r = run_in_case(exe, tmp_path, "gemm_big", 4)
    assert r.returncode == 0, r.stderr
    assert f"initialize: status {api.ERR_NO_DEVICE}" in r.stdout, r.stdout


@pytest.mark.gpu
@pytest.mark.parametrize("case", ["gemm_big", "batchnet", "cnn_small"])
def test_c_solver_matches_oracle(case, tmp_path):
    exe = build_solver(tmp_path)
    n = 1000
    r = run_in_case(exe, tmp_path, case, n)
    assert r.returncode == 0, r.stdout + r.stderr
    lines = r.stdout.splitlines()
    assert lines[0].startswith("use_model: status 0"), r.stdout
    got = np.array([float(v) for v in lines[1].split()])
    m = OracleModel(goldens.case_dir(case))
    rows = [int(np.prod(s)) for s in m.input_shapes]
    ref = m.run_batched(1, [np.ones(k) for k in rows])[0]
    res = parity.compare(got, ref)
    print(f"{case}: {parity.describe(res)}")
    assert res["ok"], parity.describe(res)

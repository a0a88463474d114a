"""Python binding of the engine's C ABI (include/rosenna.h) via ctypes.

Mirrors roseNNa's interface: ``initialize()`` then ``use_model(inputs...)``
(fLibrary/reader.f90:38, fLibrary/modelCreator.fpp:42), with a leading batch of
independent samples.  Arrays are the reference layout: the Fortran-order array
of the ONNX shape with its batch dimension widened to n.

The compiled library (librosenna_b200.so, built in-tree by build()) is required:
there is no CPU fallback, every call runs the CUDA kernels.
"""
from __future__ import annotations

import ctypes
import os
import subprocess
from typing import List, Optional, Sequence

import numpy as np

_HERE = os.path.dirname(os.path.abspath(__file__))
LIB_PATH = os.path.join(_HERE, "librosenna_b200.so")

OK, ERR_IO, ERR_FORMAT, ERR_UNSUPPORTED, ERR_SHAPE, ERR_CUDA, ERR_NO_DEVICE, ERR_STATE, ERR_ARG = range(9)

# every symbol include/rosenna.h declares
EXPORTS = [
    "initialize", "rosenna_initialize", "rosenna_initialize_from", "rosenna_check_model", "rosenna_finalize",
    "rosenna_set_devices", "rosenna_last_status", "rosenna_last_error", "rosenna_num_inputs", "rosenna_num_outputs",
    "rosenna_input_shape", "rosenna_output_shape", "rosenna_use_model_f32", "rosenna_use_model_f64",
    "rosenna_use_model_device_f32", "rosenna_use_model_device_noalloc_f32", "rosenna_last_launch_count",
    "rosenna_plan_description", "use_model", "rosenna_step_timing_begin", "rosenna_step_timing_end",
    "rosenna_step_count", "rosenna_step_info",
]


class RosennaError(RuntimeError):
    def __init__(self, code: int, msg: str):
        super().__init__(f"rosenna error {code}: {msg}")
        self.code = code


def build() -> None:
    """Compile librosenna_b200.so for sm_100a (nvcc; no GPU needed)."""
    subprocess.run(["make", "-s", "-j8", "-C", os.path.join(_HERE, "csrc")], check=True)


_lib = None


def lib():
    """The loaded C library (raises if it was not built)."""
    global _lib
    if _lib is not None:
        return _lib
    if not os.path.exists(LIB_PATH):
        raise RuntimeError(f"{LIB_PATH} is missing: run rosenna_b200.api.build() (the engine has no CPU path)")
    L = ctypes.CDLL(LIB_PATH)
    c_int, c_i64, c_char_p, c_void_p = ctypes.c_int, ctypes.c_int64, ctypes.c_char_p, ctypes.c_void_p
    PP = ctypes.POINTER(c_void_p)
    L.initialize.restype = None
    L.use_model.restype = None
    L.rosenna_initialize.restype = c_int
    L.rosenna_initialize_from.argtypes = [c_char_p, c_char_p, c_char_p]
    L.rosenna_check_model.argtypes = [c_char_p, c_char_p, c_char_p]
    L.rosenna_set_devices.argtypes = [ctypes.POINTER(c_int), c_int]
    L.rosenna_last_error.restype = c_char_p
    L.rosenna_input_shape.argtypes = [c_int, ctypes.POINTER(c_i64), c_int, ctypes.POINTER(c_int)]
    L.rosenna_output_shape.argtypes = [c_int, ctypes.POINTER(c_i64), c_int, ctypes.POINTER(c_int)]
    L.rosenna_use_model_f32.argtypes = [c_i64, PP, PP]
    L.rosenna_use_model_f64.argtypes = [c_i64, PP, PP]
    L.rosenna_use_model_device_f32.argtypes = [c_i64, PP, PP, c_void_p]
    L.rosenna_use_model_device_noalloc_f32.argtypes = [c_i64, PP, PP, c_void_p]
    L.rosenna_last_launch_count.restype = c_i64
    L.rosenna_plan_description.restype = c_char_p
    L.rosenna_step_timing_begin.argtypes = [c_i64]
    L.rosenna_step_timing_end.argtypes = [ctypes.POINTER(ctypes.c_double), ctypes.POINTER(c_i64), c_int]
    L.rosenna_step_info.argtypes = [c_int, c_char_p, c_int, ctypes.POINTER(ctypes.c_double)]
    _lib = L
    return L


def _check(rc: int) -> None:
    if rc != 0:
        raise RosennaError(rc, lib().rosenna_last_error().decode())


def _ptrs(addrs: Sequence[int]):
    return (ctypes.c_void_p * max(1, len(addrs)))(*addrs)


def _model_paths(model_dir: Optional[str], model_txt, weights_txt, variables):
    if model_dir is not None:
        model_txt = model_txt or os.path.join(model_dir, "onnxModel.txt")
        weights_txt = weights_txt or os.path.join(model_dir, "onnxWeights.txt")
        variables = variables or os.path.join(model_dir, "variables.fpp")
    return model_txt, weights_txt, variables


def set_devices(ids: Sequence[int]) -> None:
    arr = (ctypes.c_int * max(1, len(ids)))(*ids)
    _check(lib().rosenna_set_devices(arr, len(ids)))


def initialize(model_dir: Optional[str] = None, model_txt=None, weights_txt=None, variables=None) -> None:
    """initialize() of reader.f90:38; with no arguments it reads the files in the CWD."""
    if model_dir is None and model_txt is None:
        _check(lib().rosenna_initialize())
        return
    m, w, v = _model_paths(model_dir, model_txt, weights_txt, variables)
    _check(lib().rosenna_initialize_from(m.encode(), w.encode(), v.encode() if v else None))


def check_model(model_dir: str) -> str:
    """Builds the launch plan without a GPU; returns its description."""
    m, w, v = _model_paths(model_dir, None, None, None)
    _check(lib().rosenna_check_model(m.encode(), w.encode(), v.encode()))
    return lib().rosenna_plan_description().decode()


def finalize() -> None:
    _check(lib().rosenna_finalize())


def plan_description() -> str:
    return lib().rosenna_plan_description().decode()


def last_launch_count() -> int:
    return int(lib().rosenna_last_launch_count())


def _shapes(fn, count):
    out = []
    dims = (ctypes.c_int64 * 8)()
    b = ctypes.c_int()
    for i in range(count):
        r = fn(i, dims, 8, ctypes.byref(b))
        if r < 0:
            _check(-r)
        out.append((tuple(int(dims[k]) for k in range(r)), int(b.value)))
    return out


def input_specs():
    """[(export shape, batch dim)] per model input."""
    n = lib().rosenna_num_inputs()
    if n < 0:
        _check(-n)
    return _shapes(lib().rosenna_input_shape, n)


def output_specs():
    n = lib().rosenna_num_outputs()
    if n < 0:
        _check(-n)
    return _shapes(lib().rosenna_output_shape, n)


def batched_shape(shape, bdim, n):
    s = list(shape)
    s[bdim] = n
    return tuple(s)


def use_model(inputs: Sequence[np.ndarray], n: Optional[int] = None, dtype=np.float32) -> List[np.ndarray]:
    """Batched use_model on host arrays.

    inputs: arrays with the logical batched shapes (any memory order; converted
    to Fortran order).  Returns Fortran-order arrays of the batched output shapes."""
    ins_spec, outs_spec = input_specs(), output_specs()
    if len(inputs) != len(ins_spec):
        raise ValueError(f"model takes {len(ins_spec)} inputs, got {len(inputs)}")
    if n is None:
        shape0, b0 = ins_spec[0]
        n = int(np.shape(inputs[0])[b0])
    ins = [np.asfortranarray(np.asarray(x, dtype=dtype).reshape(batched_shape(s, b, n), order="A"))
           for x, (s, b) in zip(inputs, ins_spec)]
    outs = [np.zeros(batched_shape(s, b, n), dtype=dtype, order="F") for s, b in outs_spec]
    fn = lib().rosenna_use_model_f32 if dtype == np.float32 else lib().rosenna_use_model_f64
    _check(fn(n, _ptrs([a.ctypes.data for a in ins]), _ptrs([a.ctypes.data for a in outs])))
    return outs


def use_model_ptrs(n: int, in_ptrs: Sequence[int], out_ptrs: Sequence[int]) -> None:
    """Host-array use_model on raw pointers (fp32, reference layout)."""
    _check(lib().rosenna_use_model_f32(n, _ptrs(in_ptrs), _ptrs(out_ptrs)))


def use_model_device(n: int, in_ptrs: Sequence[int], out_ptrs: Sequence[int], stream: int = 0) -> None:
    """use_model on device pointers of the current device, enqueued on `stream`."""
    _check(lib().rosenna_use_model_device_f32(n, _ptrs(in_ptrs), _ptrs(out_ptrs), ctypes.c_void_p(stream)))


def use_model_rows(inputs_rows: Sequence[np.ndarray], n: Optional[int] = None) -> List[np.ndarray]:
    """use_model on (rows, n) fp32 arrays (row r = per-sample element r of every
    sample: the reference layout viewed as a C-order matrix); returns (rows, n)."""
    outs_spec = output_specs()
    if n is None:
        n = int(inputs_rows[0].shape[1])
    ins = [np.ascontiguousarray(x, dtype=np.float32) for x in inputs_rows]
    outs = []
    for s, b in outs_spec:
        rows = int(np.prod(s)) // s[b]
        outs.append(np.zeros((rows, n), dtype=np.float32))
    _check(lib().rosenna_use_model_f32(n, _ptrs([a.ctypes.data for a in ins]), _ptrs([a.ctypes.data for a in outs])))
    return outs


def use_model_device_noalloc(n: int, in_ptrs: Sequence[int], out_ptrs: Sequence[int], stream: int = 0) -> None:
    """The allocation-free device entry point (no cudaMalloc/cudaFree during the
    call; intermediates come from a fixed 64 MiB array per GPU, so n is bounded)."""
    _check(lib().rosenna_use_model_device_noalloc_f32(n, _ptrs(in_ptrs), _ptrs(out_ptrs), ctypes.c_void_p(stream)))


def step_info():
    """[(kernel name, algorithmic flops per sample)] per plan step."""
    n = lib().rosenna_step_count()
    if n < 0:
        _check(-n)
    out = []
    buf = ctypes.create_string_buffer(128)
    f = ctypes.c_double()
    for i in range(n):
        _check(lib().rosenna_step_info(i, buf, 128, ctypes.byref(f)))
        out.append((buf.value.decode(), float(f.value)))
    return out


def step_timing_begin(max_records: int) -> None:
    """Record a CUDA event pair around every plan step of the next calls (up to
    max_records steps per GPU)."""
    _check(lib().rosenna_step_timing_begin(max_records))


def step_timing_end():
    """[(summed ms, runs)] per plan step since step_timing_begin."""
    n = lib().rosenna_step_count()
    if n < 0:
        _check(-n)
    ms = (ctypes.c_double * max(1, n))()
    runs = (ctypes.c_int64 * max(1, n))()
    _check(lib().rosenna_step_timing_end(ms, runs, n))
    return [(float(ms[i]), int(runs[i])) for i in range(n)]

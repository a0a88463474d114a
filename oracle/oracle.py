"""ctypes binding of the CPU oracle (liboracle.so, built from rosenna_oracle.c).

TEST INFRASTRUCTURE ONLY: imported by tests/, __graft_entry__.smoke() and the
cpu_baseline leg of bench.py, never by the rosenna_b200 package.

The oracle is an fp64 restatement of roseNNa's Fortran path (fLibrary/reader.f90,
fLibrary/layers.f90, fLibrary/activation_funcs.f90 and the use_model body that
fLibrary/modelCreator.fpp generates).  Arrays cross this boundary in the
reference layout: the Fortran column-major array of the ONNX shape.
"""
import ctypes
import os
import subprocess

import numpy as np

_HERE = os.path.dirname(os.path.abspath(__file__))
_LIB_PATH = os.path.join(_HERE, "liboracle.so")
_lib = None


def build():
    """Compile liboracle.so (gcc, -O3, OpenMP)."""
    subprocess.run(["make", "-s", "-C", _HERE], check=True)


def _load():
    global _lib
    if _lib is not None:
        return _lib
    if not os.path.exists(_LIB_PATH):
        build()
    lib = ctypes.CDLL(_LIB_PATH)
    P = ctypes.c_void_p
    lib.ro_load.restype = P
    lib.ro_load.argtypes = [ctypes.c_char_p, ctypes.c_char_p, ctypes.c_char_p, ctypes.c_char_p, ctypes.c_int]
    lib.ro_free.argtypes = [P]
    lib.ro_num_inputs.argtypes = [P]
    lib.ro_num_outputs.argtypes = [P]
    lib.ro_input_shape.argtypes = [P, ctypes.c_int, ctypes.POINTER(ctypes.c_int)]
    lib.ro_output_shape.argtypes = [P, ctypes.c_int, ctypes.POINTER(ctypes.c_int)]
    DPP = ctypes.POINTER(ctypes.c_void_p)
    lib.ro_run.argtypes = [P, DPP, DPP, ctypes.c_char_p, ctypes.c_int]
    lib.ro_run_batched.argtypes = [P, ctypes.c_int64, DPP, DPP, ctypes.POINTER(ctypes.c_int),
                                   ctypes.POINTER(ctypes.c_int), ctypes.c_int, ctypes.c_char_p, ctypes.c_int]
    lib.ro_max_threads.restype = ctypes.c_int
    _lib = lib
    return lib


def _ptrs(arrays):
    return (ctypes.c_void_p * len(arrays))(*[a.ctypes.data for a in arrays])


class OracleModel:
    """One model loaded from onnxModel.txt / onnxWeights.txt / variables.fpp."""

    def __init__(self, model_dir):
        lib = _load()
        err = ctypes.create_string_buffer(512)
        paths = [os.path.join(model_dir, f).encode() for f in ("onnxModel.txt", "onnxWeights.txt", "variables.fpp")]
        self._h = lib.ro_load(paths[0], paths[1], paths[2], err, 512)
        if not self._h:
            raise RuntimeError("oracle load failed: " + err.value.decode())
        self._lib = lib
        dims = (ctypes.c_int * 8)()
        self.input_shapes = []
        for i in range(lib.ro_num_inputs(self._h)):
            r = lib.ro_input_shape(self._h, i, dims)
            self.input_shapes.append(tuple(dims[j] for j in range(r)))
        self.output_shapes = []
        for i in range(lib.ro_num_outputs(self._h)):
            r = lib.ro_output_shape(self._h, i, dims)
            self.output_shapes.append(tuple(dims[j] for j in range(r)))
        self.input_pre = self._input_pre(os.path.join(model_dir, "variables.fpp"))

    def _input_pre(self, variables_fpp):
        """Elements in front of each input's batch index in the reference layout:
        the batch is dim 1 of an input first read by an LSTM ((T, N, I) and
        (1, N, H) forms) or a Slice (a stacked LSTM's (L, N, H) state), else dim 0."""
        import ast

        first = {}
        with open(variables_fpp) as f:
            for line in f:
                if line.startswith("#:set architecture"):
                    for e in ast.literal_eval(line.split("=", 1)[1].strip()):
                        names = e[1] if isinstance(e[1], (list, tuple)) else []
                        for nm in names:
                            if isinstance(nm, str) and nm not in first:
                                first[nm] = e[0]
        with open(variables_fpp) as f:
            true_inputs = [ast.literal_eval(ln.split("=", 1)[1].strip()) for ln in f if ln.startswith("#:set trueInputs")][0]
        pre = []
        for name, shape in true_inputs:
            b = 1 if first.get(name) in ("LSTM", "Slice") and len(shape) >= 2 else 0
            pre.append(int(np.prod(shape[:b])) if b else 1)
        return pre

    def __del__(self):
        if getattr(self, "_h", None):
            self._lib.ro_free(self._h)
            self._h = None

    def run(self, inputs):
        """One use_model call at the export shapes.  `inputs` are numpy arrays of
        the logical ONNX shapes; returns the outputs with the logical shapes."""
        ins = [np.asfortranarray(np.asarray(x, dtype=np.float64).reshape(s)) for x, s in zip(inputs, self.input_shapes)]
        outs = [np.zeros(s, dtype=np.float64, order="F") for s in self.output_shapes]
        err = ctypes.create_string_buffer(512)
        rc = self._lib.ro_run(self._h, _ptrs(ins), _ptrs(outs), err, 512)
        if rc:
            raise RuntimeError("oracle run failed: " + err.value.decode())
        return outs

    def run_batched(self, n, inputs, in_pre=None, out_pre=None, threads=None):
        """Per-sample loop over a batch of n (model exported at batch 1), on
        `threads` OpenMP threads (default: every host core this process may use).

        `inputs` are float64 arrays in the batched reference layout (any shape
        holding that memory order); in_pre / out_pre give the elements in front
        of each array's batch index (default: from the model); returns flat
        float64 outputs in the reference layout."""
        if threads is None:
            threads = host_cores()
        if in_pre is None:
            in_pre = self.input_pre
        if out_pre is None:
            out_pre = [1] * len(self.output_shapes)
        ins = [np.ascontiguousarray(x, dtype=np.float64).reshape(-1) for x in inputs]
        outs = [np.zeros(int(np.prod(s)) * n, dtype=np.float64) for s in self.output_shapes]
        ip = (ctypes.c_int * len(in_pre))(*in_pre)
        op = (ctypes.c_int * len(out_pre))(*out_pre)
        err = ctypes.create_string_buffer(512)
        rc = self._lib.ro_run_batched(self._h, n, _ptrs(ins), _ptrs(outs), ip, op, threads, err, 512)
        if rc:
            raise RuntimeError("oracle batched run failed: " + err.value.decode())
        return outs


def max_threads():
    """OpenMP's default team size (honours OMP_NUM_THREADS)."""
    return _load().ro_max_threads()


def host_cores():
    """Host CPUs this process may run on, whatever OMP_NUM_THREADS says (torchrun
    sets it to 1); passed explicitly as the oracle's thread count."""
    import os

    try:
        return len(os.sched_getaffinity(0))
    except (AttributeError, OSError):
        return os.cpu_count() or 1

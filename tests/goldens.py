"""Readers for the fixtures under tests/golden/ (written by tests/golden/make_golden.py)."""
import os

import numpy as np

GOLDEN = os.path.join(os.path.dirname(os.path.abspath(__file__)), "golden")


def cases():
    return sorted(d for d in os.listdir(GOLDEN) if os.path.isdir(os.path.join(GOLDEN, d)) and not d.startswith("_"))


def case_dir(name):
    return os.path.join(GOLDEN, name)


def _read_pairs(path):
    with open(path) as f:
        lines = [ln for ln in f.read().splitlines() if ln.strip()]
    out = []
    for i in range(0, len(lines), 2):
        shape = tuple(int(v) for v in lines[i].split())
        vals = np.array([float(v) for v in lines[i + 1].split()], dtype=np.float64)
        out.append(vals.reshape(shape))
    return out


def inputs(name):
    """Inputs in logical (C-order numpy) form."""
    return _read_pairs(os.path.join(GOLDEN, name, "inputs.txt"))


def golden(name):
    """PyTorch fp64 output, logical shape."""
    return _read_pairs(os.path.join(GOLDEN, name, "golden.txt"))[0]

"""The oracle (CPU fp64 restatement of roseNNa) against the golden fixtures.

The reference's own checker compares shapes exactly and values with an absolute
tolerance of 1e-5 (test/testChecker.py:12-17).  Both sides here are fp64, so the
oracle is also held to 1e-12."""
import numpy as np
import pytest

from oracle.oracle import OracleModel
from tests import goldens


@pytest.mark.parametrize("case", goldens.cases())
def test_oracle_matches_golden(case):
    m = OracleModel(goldens.case_dir(case))
    ins = goldens.inputs(case)
    out = m.run(ins)[0]
    ref = goldens.golden(case)
    # shapes: the reference compares the SHAPE line (testChecker.py:12)
    assert int(np.prod(out.shape)) == ref.size
    np.testing.assert_allclose(np.asarray(out).reshape(ref.shape), ref, rtol=0, atol=1e-12)

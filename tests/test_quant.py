"""The checkpoint quantizer's arithmetic order, on the CPU: the oracle
restatement (oracle/quant.py, the summation order of the GPU kernel) against
the unmodified reference's quantizers on the seeded cases
(tests/golden/quant_cases.npz, made by tests/golden/gen_quant_golden.py)."""
import os
import sys

import numpy as np
import pytest

from oracle import quant as OQ

sys.path.insert(0, os.path.join(os.path.dirname(os.path.abspath(__file__)), "golden"))
from quant_cases import cases  # noqa: E402

CASES = cases()


@pytest.mark.parametrize("case", CASES, ids=[c[0] for c in CASES])
def test_oracle_quantizer_vs_reference(golden, case):
    d = golden("quant_cases")
    name, w, kind, kw = case
    K = w.shape[1]
    if kind == "mse":
        alpha = np.linspace(kw.get("amin", 0.55), 1.0, kw.get("nalpha", 17))
        sal = None
        if "salience" in kw:
            s = np.asarray(kw["salience"], dtype=np.float64)
            sal = (s * s) / float((s * s).mean())
        best = OQ.group_scales(w, alpha, sal)
    else:
        best = OQ.group_scales(w)
    e = OQ.shared_exponent(best)
    if kind == "tight":
        dd = 0
        while dd < 15 and np.round(best.max() * np.exp2(15 - (e - dd - 1))) <= 65535:
            dd += 1
        e -= dd
    w4, m = OQ.pack_codes(w, best, e)
    assert e == int(d[f"{name}_e"])
    assert np.array_equal(m, d[f"{name}_m"]), name
    assert np.array_equal(w4, d[f"{name}_w4"]), name
    assert K % 128 == 0


def test_numpy_group_sum_order():
    """numpy's float64 sum over a contiguous 128-element axis is the
    eight-accumulator order the kernel restates."""
    rng = np.random.default_rng(7)
    x = (rng.normal(size=(64, 32, 128)) * np.exp(rng.normal(size=(64, 32, 128)) * 6)) ** 2
    assert np.array_equal(x.sum(axis=2), OQ._group_sum(x))

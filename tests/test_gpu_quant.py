"""The GPU checkpoint quantizer (fable5_llm_b200.quant over f5_quant_w4_*)
against the unmodified reference's quantizers: w4 codes, m mantissas, e and
sh bit-identical on the seeded cases of tests/golden/quant_cases.py, the
packed image equal to pack_ddr_rows of those arrays, and the refusals."""
import os
import sys

import numpy as np
import pytest

from fable5_llm_b200 import quant as Q
from oracle import quant as OQ
from fable5_llm_b200.w4a8_ref import pack_ddr_rows

sys.path.insert(0, os.path.join(os.path.dirname(os.path.abspath(__file__)), "golden"))
from quant_cases import cases  # noqa: E402

pytestmark = pytest.mark.gpu
CASES = cases()


@pytest.mark.parametrize("case", CASES, ids=[c[0] for c in CASES])
def test_gpu_quantizer_vs_reference(golden, case):
    d = golden("quant_cases")
    name, w, kind, kw = case
    if kind == "mse":
        q = Q.quant_linear_mse(w, **kw)
        w4, m, e, sh = q["w4"], q["m"], q["e"], q["sh"]
        assert q["g"] == 128
    elif kind == "max":
        w4, m, e, sh = Q.quantize_weights(w)
    else:
        q = Q.quant_linear(w, tighten_e=True, mse_scale=False)
        w4, m, e, sh = q["w4"], q["m"], q["e"], q["sh"]
    assert (e, sh) == (int(d[f"{name}_e"]), int(d[f"{name}_sh"])), name
    assert np.array_equal(m, d[f"{name}_m"]), name
    assert np.array_equal(w4, d[f"{name}_w4"]), name


def test_gpu_quantizer_image_is_pack_ddr_rows(golden):
    d = golden("quant_cases")
    name, w, _, _ = CASES[1]
    img, N, K, e, sh = Q.quant_linear_image(w)
    ref, _ = pack_ddr_rows(d[f"{name}_w4"], d[f"{name}_m"])
    assert (N, K, e) == (w.shape[0], w.shape[1], int(d[f"{name}_e"]))
    assert img.cpu().numpy().tobytes() == ref


def test_gpu_quantizer_refusals():
    w = np.zeros((4, 1024), dtype=np.float32)
    with pytest.raises(NotImplementedError):
        Q.quant_linear(w, hess=np.eye(1024))
    with pytest.raises(SystemExit):
        Q.quant_linear(w, mse_scale=False, salience=np.ones(1024))
    with pytest.raises(ValueError):
        Q.quant_linear_mse(w, salience=np.ones(1000))
    with pytest.raises(NotImplementedError):
        Q.quant_layer({"type": "full_attention"}, w8=True)
    # all-zero matrix: every group takes the 1e-12 scale floor (the oracle
    # restatement gives the same m and e)
    q = Q.quant_linear_mse(w)
    best = OQ.group_scales(w, np.linspace(0.55, 1.0, 17))
    e = OQ.shared_exponent(best)
    w4, m = OQ.pack_codes(w, best, e)
    assert not q["w4"].any() and q["e"] == e and np.array_equal(q["m"], m)

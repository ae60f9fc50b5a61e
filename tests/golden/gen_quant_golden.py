#!/usr/bin/env python3
"""Generate ``quant_cases.npz``: the UNMODIFIED reference's quantizers
(``quant_linear_mse`` / ``quant_linear``, ref/layer_fixed.py:981-1111, and
``quantize_weights``, ref/w4a8_ref.py:154-180) on the seeded matrices of
quant_cases.py.  Stored per case: the w4 codes, the m mantissas, e and sh.

Run where the reference checkout exists, with the environment variable
F5_REFERENCE set to its root directory; the GPU box never runs it.

    python tests/golden/gen_quant_golden.py
"""
from __future__ import annotations

import os
import sys

import numpy as np

REF = os.environ.get("F5_REFERENCE")
if not REF or not os.path.isdir(os.path.join(REF, "ref")):
    sys.exit("set F5_REFERENCE to the root of the reference checkout (the directory holding ref/)")
HERE = os.path.dirname(os.path.abspath(__file__))
os.environ["FABLE5_MODEL"] = "9b"
sys.dont_write_bytecode = True
sys.path.insert(0, os.path.join(REF, "ref"))
sys.path.insert(0, HERE)

import layer_fixed as LF      # noqa: E402  (reference)
import w4a8_ref as W          # noqa: E402  (reference)
from quant_cases import cases  # noqa: E402


def main():
    out = {}
    for name, m, kind, kw in cases():
        if kind == "mse":
            q = LF.quant_linear_mse(m, **kw)
            w4, mm, e, sh = q["w4"], q["m"], q["e"], q["sh"]
        elif kind == "max":
            w4, mm, e, sh = W.quantize_weights(np.asarray(m, dtype=np.float64))
        else:
            q = LF.quant_linear(m, tighten_e=True, mse_scale=False)
            w4, mm, e, sh = q["w4"], q["m"], q["e"], q["sh"]
        out[f"{name}_w4"] = np.asarray(w4, dtype=np.int8)
        out[f"{name}_m"] = np.asarray(mm, dtype=np.uint16)
        out[f"{name}_e"] = np.int64(e)
        out[f"{name}_sh"] = np.int64(sh)
        print(f"{name}: {kind} e={e} sh={sh}")
    np.savez_compressed(os.path.join(HERE, "quant_cases.npz"), **out)


if __name__ == "__main__":
    main()

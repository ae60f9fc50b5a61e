"""Drop-in for ref/fixedpoint.py (integer primitives), computed on the GPU.

Scalar arguments return Python ints like the reference; array arguments
return int64 arrays (the reference's scalar functions, vectorised).
"""
from __future__ import annotations

import numpy as np

from . import _lib as L

I64 = np.int64


def _ops():
    from . import ops
    return ops


def _scalar_or_array(op, x, arg0=0):
    a = np.asarray(x, dtype=I64)
    out = _ops().prim(op, a.reshape(-1), arg0=arg0).reshape(a.shape)
    return int(out) if a.ndim == 0 else out


def dyn_quant_i8(x16):
    """ref/fixedpoint.py:24-33 -> (int8 x8, e)."""
    import torch
    x = np.asarray(x16, dtype=I64).reshape(-1)
    assert (np.abs(x) <= 32768).all(), "DYNQ8 input must be an int16-range vector"
    x8, meta = _ops().dynq8(_ops().to_dev(x.astype(np.int16)), x.size, 0)
    torch.cuda.synchronize()
    return x8.cpu().numpy(), int(meta[0])


def rsqrt_q(v, P):
    """ref/fixedpoint.py:56-75 -> (r, e)."""
    assert int(v) > 0
    r, e = _ops().prim(L.PR_RSQRT, np.array([int(v)]), arg0=int(P), want2=True)
    return int(r[0]), int(e[0])


def recip_q(v, P):
    """ref/fixedpoint.py:179-198 -> (r, e)."""
    assert int(v) > 0
    r, e = _ops().prim(L.PR_RECIP, np.array([int(v)]), arg0=int(P), want2=True)
    return int(r[0]), int(e[0])


def exp2_frac_q16(f):
    """ref/fixedpoint.py:99-106."""
    return _scalar_or_array(L.PR_EXP2_FRAC, f)


def exp_neg_q(x_q16):
    """ref/fixedpoint.py:109-121."""
    assert (np.asarray(x_q16) <= 0).all()
    return _scalar_or_array(L.PR_EXP_NEG, x_q16)


def sigmoid_q(x_q12):
    """ref/fixedpoint.py:135-147."""
    return _scalar_or_array(L.PR_SIGMOID, x_q12)


def softplus_q(x_q12):
    """ref/fixedpoint.py:150-165."""
    return _scalar_or_array(L.PR_SOFTPLUS, x_q12)


def silu_q(x_q12):
    """ref/fixedpoint.py:168-171."""
    return _scalar_or_array(L.PR_SILU, x_q12)

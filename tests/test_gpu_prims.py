"""GPU parity of every integer primitive of the law against the oracle
(bit-exact), over the full input domains the decode path reaches."""
import numpy as np
import pytest

import oracle as O
from fable5_llm_b200 import _lib as L
from fable5_llm_b200 import ops

pytestmark = pytest.mark.gpu
I64 = np.int64


def test_rshr():
    rng = np.random.default_rng(1)
    v = np.concatenate([rng.integers(-(1 << 50), 1 << 50, 200000),
                        np.array([5, -5, 3, -3, 1, -1, 0, 2, -2], dtype=I64)])
    s = rng.integers(-10, 45, v.size)
    got = ops.prim(L.PR_RSHR, v, in2=s)
    assert np.array_equal(got, O.rshr_v(v, s))


@pytest.mark.parametrize("op,fn,lo,hi", [
    (L.PR_SIGMOID, O.sigmoid_q, -(1 << 18), 1 << 18),
    (L.PR_SOFTPLUS, O.softplus_q, -(1 << 18), 1 << 18),
    (L.PR_SILU, O.silu_q, -(1 << 21), 1 << 21),
    (L.PR_EXP2_FRAC, O.exp2_frac_q16, 0, 1 << 16),
])
def test_lut_functions_exhaustive(op, fn, lo, hi):
    x = np.arange(lo, hi, dtype=I64)
    assert np.array_equal(ops.prim(op, x), fn(x))


def test_exp_neg():
    x = np.concatenate([-np.arange(0, 1 << 22, dtype=I64),
                        -np.random.default_rng(2).integers(1 << 22, 1 << 44, 100000)])
    assert np.array_equal(ops.prim(L.PR_EXP_NEG, x), O.exp_neg_q(x))


@pytest.mark.parametrize("op,fn", [(L.PR_RSQRT, O.rsqrt_q), (L.PR_RECIP, O.recip_q)])
def test_rsqrt_recip(op, fn):
    rng = np.random.default_rng(3)
    v = np.concatenate([rng.integers(1, 1 << 48, 20000), (np.int64(1) << np.arange(0, 48)),
                        (np.int64(1) << np.arange(1, 48)) - 1, np.arange(1, 5000)])
    P = rng.integers(0, 48, v.size)
    r, e = ops.prim(op, v, in2=P, want2=True)
    ref = [fn(int(a), int(b)) for a, b in zip(v, P)]
    assert np.array_equal(r, np.array([a for a, _ in ref]))
    assert np.array_equal(e, np.array([b for _, b in ref]))


def test_bf_shift_dynq8_e():
    m = np.concatenate([np.arange(0, 200000, dtype=I64),
                        np.random.default_rng(4).integers(0, 1 << 44, 20000)])
    assert np.array_equal(ops.prim(L.PR_BF_SHIFT, m), np.array([O.bf_shift(int(a)) for a in m]))
    m2 = np.arange(0, 70000, dtype=I64)
    ref = np.array([O.dyn_quant_i8(np.array([a]))[1] for a in m2])
    assert np.array_equal(ops.prim(L.PR_DYNQ8_E, m2), ref)


def test_norm_scales(golden):
    d = golden("ref_prims")
    o32, k, o16 = d["nb_o32"], d["nb_k"], d["nb_o16"]
    ss32 = (o32 * o32).sum(axis=1)
    ss16 = (o16 * o16).sum(axis=1)
    assert np.array_equal(ops.prim(L.PR_DN_NORM_SCALE, ss32, arg0=128, in2=k), d["nb_m_float"])
    assert np.array_equal(ops.prim(L.PR_EPS_NORM_SCALE, ss16, arg0=7, in2=k), d["nb_m_eps"])
    # a wider random sweep against the oracle
    rng = np.random.default_rng(5)
    blocks = np.round(rng.normal(0, 1, (3000, 128)) * (10.0 ** rng.uniform(-1, 7, 3000))[:, None]).astype(I64)
    ks = np.array([O.bf_shift(int(np.abs(b).max())) for b in blocks])
    ss = (blocks * blocks).sum(axis=1)
    ref = np.array([O.dn_norm_scale(b, int(kk)) for b, kk in zip(blocks, ks)])
    assert np.array_equal(ops.prim(L.PR_DN_NORM_SCALE, ss, arg0=128, in2=ks), ref)

"""CPU restatement of the W4 checkpoint quantizers (TEST INFRASTRUCTURE ONLY).

Follows ref/layer_fixed.py:981-1030 (quant_linear_mse) and
ref/w4a8_ref.py:154-180 (quantize_weights) with the group error summed in the
explicit order the GPU kernel uses (fable5_llm_b200/csrc/f5_quant.cu): eight
running sums over elements j, j+8, ..., j+120 of a 128-weight group, then
((r0+r1)+(r2+r3))+((r4+r5)+(r6+r7)).  That is numpy's own order for a
contiguous 128-element float64 reduction, which the committed reference
fixtures (tests/golden/quant_cases.npz) pin.  Only tests/ import this.
"""
import numpy as np


def _group_sum(x):
    """x [..., 128] -> float64 sums in the eight-accumulator order."""
    r = x.reshape(x.shape[:-1] + (16, 8))
    acc = r[..., 0, :].copy()
    for i in range(1, 16):
        acc = acc + r[..., i, :]
    a01 = acc[..., 0] + acc[..., 1]
    a23 = acc[..., 2] + acc[..., 3]
    a45 = acc[..., 4] + acc[..., 5]
    a67 = acc[..., 6] + acc[..., 7]
    return (a01 + a23) + (a45 + a67)


def group_scales(W, alpha=None, sal=None, g=128):
    """Every group's chosen scale (alpha None: the max|W|/7 rule)."""
    W = np.asarray(W, dtype=np.float64)
    N, K = W.shape
    Wg = W.reshape(N, K // g, g)
    smax = np.maximum(np.abs(Wg).max(axis=2), 1e-12)
    best_s = smax / 7.0
    if alpha is None:
        return best_s
    best_e = np.full(best_s.shape, np.inf)
    sw = None if sal is None else np.asarray(sal, dtype=np.float64).reshape(1, K // g, g)
    for a in alpha:
        s = (smax / 7.0) * a
        q = np.clip(np.rint(Wg / s[:, :, None]), -8, 7)
        d = q * s[:, :, None] - Wg
        e2 = d * d
        if sw is not None:
            e2 = e2 * sw
        err = _group_sum(e2)
        upd = err < best_e
        best_s = np.where(upd, s, best_s)
        best_e = np.where(upd, err, best_e)
    return best_s


def pack_codes(W, best_s, e, g=128):
    """(w4 [N, K] int8, m [N, K/g] uint16) for shared exponent e."""
    W = np.asarray(W, dtype=np.float64)
    N, K = W.shape
    m = np.clip(np.rint(best_s * np.exp2(15 - e)), 1, 65535).astype(np.uint16)
    eff = m.astype(np.float64) * np.exp2(e - 15)
    w4 = np.clip(np.rint(W.reshape(N, K // g, g) / eff[:, :, None]), -8, 7).astype(np.int8)
    return w4.reshape(N, K), m


def shared_exponent(best_s):
    return int(np.ceil(np.log2(best_s.max()))) + 1

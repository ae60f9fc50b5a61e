"""Drop-in for ref/w4a8_ref.py (the W4A8 matvec law and row wire format).

Same names, arguments and return types as the reference; ``matvec_y32`` and
``rshift_round`` compute on the GPU through the C ABI (f5_matvec_y32_host,
f5_prim_dev).  Packing helpers are host data-format code, like the
reference's.  Range assertions raise AssertionError as the reference does.
"""
from __future__ import annotations

import numpy as np

from . import _lib as L

G = 128                 # ref/w4a8_ref.py:73
G_WIRE = (128, 64)
K_PER_WBEAT = 128
SCALES_PER_BEAT = 32


def rshift_round(v, s):
    """ref/w4a8_ref.py:90-99 (GPU element-wise)."""
    from . import ops
    a = np.asarray(v, dtype=np.int64)
    if a.size == 0:
        return a
    out = ops.prim(L.PR_RSHR, a.reshape(-1), arg0=int(s)).reshape(a.shape)
    return out if a.ndim else np.int64(out.reshape(())[()])


def row_beats(K, g=G):
    """ref/w4a8_ref.py:102-108."""
    assert g in G_WIRE, f"group size {g} has no defined wire format"
    assert K % K_PER_WBEAT == 0, f"K={K} must be a multiple of {K_PER_WBEAT}"
    return K // K_PER_WBEAT, (K // g + SCALES_PER_BEAT - 1) // SCALES_PER_BEAT


def row_stride(K, g=G):
    """ref/w4a8_ref.py:111-114."""
    wb, sb = row_beats(K, g)
    return (wb + sb) * 64


def group_size_of(w4, m, g=None):
    """ref/w4a8_ref.py:143-151."""
    K = np.asarray(w4).shape[1]
    ng = np.asarray(m).shape[1]
    assert ng > 0 and K % ng == 0, f"m has {ng} groups, incompatible with K={K}"
    gi = K // ng
    if g is not None:
        assert int(g) == gi, f"declared g={g} but w4/m imply {gi}"
    return gi


def final_shift(K, g=G):
    """The sh rule of ref/w4a8_ref.py:177-179."""
    NG = K // g
    return max(0, (NG * 65535 * (g * 8 * 127)).bit_length() - 31)


def pack_w4(w4):
    """ref/w4a8_ref.py:331-334: low nibble = even k."""
    u = (np.asarray(w4).astype(np.int16) & 0xF).astype(np.uint8)
    return (u[:, 0::2] | (u[:, 1::2] << 4)).astype(np.uint8)


def unpack_w4(packed, K):
    """ref/w4a8_ref.py:337-346."""
    p = np.asarray(packed, dtype=np.uint8)
    lo = (p & 0xF).astype(np.int8)
    hi = (p >> 4).astype(np.int8)
    out = np.empty((p.shape[0], K), dtype=np.int8)
    out[:, 0::2] = np.where(lo > 7, lo - 16, lo)
    out[:, 1::2] = np.where(hi > 7, hi - 16, hi)
    return out


def pack_ddr_rows(w4, m, g=None):
    """ref/w4a8_ref.py:349-370 -> (image bytes, row stride)."""
    w4 = np.asarray(w4)
    N, K = w4.shape
    g = group_size_of(w4, m, g)
    stride = row_stride(K, g)
    img = np.zeros((N, stride), dtype=np.uint8)
    img[:, :K // 2] = pack_w4(w4)
    mb = np.asarray(m).astype("<u2").view(np.uint8).reshape(N, -1)
    img[:, K // 2:K // 2 + mb.shape[1]] = mb
    return img.tobytes(), stride


def unpack_ddr_rows(img, nrows, K, g=G):
    """ref/w4a8_ref.py:429-446."""
    stride = row_stride(K, g)
    a = np.frombuffer(img, dtype=np.uint8) if isinstance(img, (bytes, bytearray)) else np.asarray(img, np.uint8)
    assert a.size == nrows * stride, f"image is {a.size}B, expected {nrows}*{stride}"
    a = a.reshape(nrows, stride)
    NG = K // g
    return unpack_w4(a[:, :K // 2], K), a[:, K // 2:K // 2 + 2 * NG].copy().view("<u2").reshape(nrows, NG)


def matvec_y32_img(img, N, K, sh, x8, g=G):
    """matvec_y32 straight from a packed image (DDRWeights.matvec,
    ref/seq_model.py:431-452), on the GPU."""
    from . import ops
    a = np.frombuffer(img, dtype=np.uint8) if isinstance(img, (bytes, bytearray)) else np.asarray(img, np.uint8)
    return ops.matvec_y32_host(a, N, K, g, sh, np.asarray(x8, dtype=np.int8))


def matvec_y32(w4, m, sh, x8, g=None):
    """ref/w4a8_ref.py:254-289 -> int32 y (N,), on the GPU."""
    w4 = np.asarray(w4)
    N, K = w4.shape
    g = group_size_of(w4, m, g)
    img, _ = pack_ddr_rows(w4, m, g)
    return matvec_y32_img(img, N, K, sh, x8, g)

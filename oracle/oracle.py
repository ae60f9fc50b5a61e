"""numpy restatement of the reference's integer decode law (TEST ORACLE).

TEST INFRASTRUCTURE ONLY: imported by ``tests/``, ``__graft_entry__.smoke``
and the CPU legs of ``bench.py`` as the checker.  The product path
(``fable5_llm_b200``) never imports this module.

Every function restates one function of coreyhahn/fable5_llm and cites it as
``file:line`` (paths inside that project).  The arithmetic is numpy int64
with Python-int scalars where the reference uses Python ints; the per-element
Python loops of the reference are vectorised here (same integer results -- the
tests pin that against fixtures made by the unmodified reference).

Parity pinning: ``tests/golden/*.npz`` hold the reference's own committed
golden vectors (``tb/vec_s1..s4``, ``tb/vectors/s1..s4``, the LUT ROMs) and
outputs of the unmodified reference run on seeded inputs; see
``tests/test_oracle_golden.py``.
"""
from __future__ import annotations

import ctypes
import math
import os

import numpy as np

I64 = np.int64

# ---------------------------------------------------------------------------
# 9B operating point (ref/layer_fixed.py:103-147, ref/qwen3_5_9b_config.json)
# ---------------------------------------------------------------------------
RS_F = 7          # ref/layer_fixed.py:103 RS_F_BY_TAG["9b"]
QKV_F = 8         # ref/layer_fixed.py:136
NRM_F = 14        # ref/layer_fixed.py:137
S_F = 13          # ref/layer_fixed.py:138
GAT_F = 15        # ref/layer_fixed.py:144
CW_F = 13         # ref/layer_fixed.py:145
ROPE_F = 15       # ref/layer_fixed.py:146
DN_NORM_F = 11    # ref/layer_fixed.py:404
M_Q15_MAX = 65535  # ref/layer_fixed.py:406
EPS = 1e-6        # rms_norm_eps of the 9B config (ref/layer_ref.py:35)
EPS_Q = 40        # ref/layer_fixed.py:649
EPS_M = int(round(EPS * (1 << EPS_Q)))   # ref/layer_fixed.py:650 -> 1099512
G = 128           # ref/w4a8_ref.py:73


class Geometry:
    """Qwen3.5-9B decode geometry (ref/layer_ref.py:25-49).

    ``n_layers``/``vocab``/``layer_types`` may be reduced for fast tests; every
    per-layer shape stays the 9B one.
    """

    H = 4096
    NQ = 16
    NKV = 4
    HD = 256
    ROT = 64
    THETA = 10000000.0
    FFN = 12288
    LNH = 32
    LNKH = 16
    LDK = 128
    LDV = 128
    CONV_K = 4
    VREP = LNH // LNKH
    LKD = LNKH * LDK
    LVD = LNH * LDV
    CONV_DIM = 2 * LKD + LVD

    def __init__(self, n_layers=32, vocab=248320, layer_types=None):
        if layer_types is None:
            layer_types = [("full_attention" if (i % 4) == 3 else
                            "linear_attention") for i in range(n_layers)]
        assert len(layer_types) == n_layers
        self.n_layers = n_layers
        self.vocab = vocab
        self.layer_types = list(layer_types)


GEOM_9B = Geometry()


# ---------------------------------------------------------------------------
# L1 primitives
# ---------------------------------------------------------------------------
def rshr(v, s):
    """Round-half-away-from-zero arithmetic right shift; s<0 = exact left
    shift.  Restates ref/w4a8_ref.py:90-99 (rshift_round)."""
    v = np.asarray(v, dtype=I64)
    s = int(s)
    if s == 0:
        return v.copy()
    if s < 0:
        return v << I64(-s)
    add = I64(1) << I64(s - 1)
    return np.where(v >= 0, (v + add) >> I64(s), -((-v + add) >> I64(s)))


def rshr_v(v, s):
    """rshr with an element-wise shift array (same rule per element)."""
    v = np.asarray(v, dtype=I64)
    s = np.broadcast_to(np.asarray(s, dtype=I64), v.shape)
    sp = np.maximum(s, 1)
    add = I64(1) << (sp - 1)
    right = np.where(v >= 0, (v + add) >> sp, -((-v + add) >> sp))
    left = v << np.maximum(-s, 0)
    return np.where(s > 0, right, np.where(s < 0, left, v))


def rshr_int(v: int, s: int) -> int:
    """Python-int rshr (unbounded), same rule as ref/w4a8_ref.py:90-99."""
    if s == 0:
        return v
    if s < 0:
        return v << (-s)
    add = 1 << (s - 1)
    return (v + add) >> s if v >= 0 else -((-v + add) >> s)


def clip16(x):
    """ref/layer_fixed.py:809."""
    return np.clip(np.asarray(x, dtype=I64), -32768, 32767)


# ---- LUT tables, restating the float formulas of ref/fixedpoint.py ----
def rsqrt_lut():
    """512-entry Q15 seed (ref/fixedpoint.py:42-53)."""
    i = np.arange(256)
    lo = 1.0 + (i + 0.5) / 256.0
    hi = 2.0 + 2.0 * (i + 0.5) / 256.0
    return np.round((1.0 / np.sqrt(np.concatenate([lo, hi]))) * (1 << 15)).astype(I64)


def recip_lut():
    """256-entry Q15 seed (ref/fixedpoint.py:186-188)."""
    m = 1.0 + (np.arange(256) + 0.5) / 256.0
    return np.round((1.0 / m) * (1 << 15)).astype(I64)


def exp2_lut():
    """257-entry Q16 table of 2^(i/256) (ref/fixedpoint.py:91-96)."""
    f = np.arange(257) / 256.0
    return np.round((2.0 ** f) * (1 << 16)).astype(I64)


def _pwl_x():
    return -16.0 + 32.0 * np.arange(257) / 256.0


def sigmoid_lut():
    """257-entry Q15 sigmoid, saturated at 32767 (ref/fixedpoint.py:128-147)."""
    return np.minimum(np.round((1.0 / (1.0 + np.exp(-_pwl_x()))) * (1 << 15)).astype(I64),
                      32767)


def softplus_lut():
    """257-entry Q12 softplus (ref/fixedpoint.py:153-157)."""
    return np.round(np.log1p(np.exp(_pwl_x())) * (1 << 12)).astype(I64)


RSQRT_LUT = rsqrt_lut()
RECIP_LUT = recip_lut()
EXP2_LUT = exp2_lut()
SIGMOID_LUT = sigmoid_lut()
SOFTPLUS_LUT = softplus_lut()


def dyn_quant_i8(x16):
    """DYNQ8: minimal e with (max|x| + (1<<e>>1)) >> e <= 127; x8 =
    clip(rshr(x,e), -127, 127).  ref/fixedpoint.py:24-33."""
    x = np.asarray(x16, dtype=I64)
    m = int(np.abs(x).max()) if x.size else 0
    e = 0
    while (m + ((1 << e) >> 1)) >> e > 127:
        e += 1
    x8 = np.clip(rshr(x, e) if e else x, -127, 127).astype(np.int8)
    return x8, e


def rsqrt_q(v: int, P: int):
    """1/sqrt(v*2^-P) = r*2^-30*2^e.  ref/fixedpoint.py:56-75.  Python ints
    (floor shifts), exactly as the reference."""
    v = int(v)
    assert v > 0
    s = v.bit_length() - 32
    if (s - P) % 2 != 0:
        s += 1
    m = (v >> s) if s >= 0 else (v << -s)
    E = s - P + 30
    idx = ((m >> 22) & 0xFF) if m < (1 << 31) else (256 | ((m >> 23) & 0xFF))
    r = int(RSQRT_LUT[idx]) << 15
    for _ in range(2):
        r2 = (r * r) >> 30
        mr2 = (m * r2) >> 30
        r = (r * ((3 << 30) - mr2)) >> 31
    return r, -E // 2


def recip_q(v: int, P: int):
    """1/(v*2^-P) = r*2^-30*2^e.  ref/fixedpoint.py:179-198."""
    v = int(v)
    assert v > 0
    n = v.bit_length()
    sh = n - 31
    m = (v >> sh) if sh >= 0 else (v << -sh)
    idx = (m - (1 << 30)) >> 22
    r = int(RECIP_LUT[min(int(idx), 255)]) << 15
    for _ in range(2):
        mr = (m * r) >> 30
        r = (r * ((2 << 30) - mr)) >> 30
    return r, -(sh + 30 - P)


def exp2_frac_q16(f):
    """PWL 2^(f/2^16), Q16 (ref/fixedpoint.py:99-106); vectorised."""
    f = np.asarray(f, dtype=I64)
    i, lo = f >> 8, f & 0xFF
    a, b = EXP2_LUT[i], EXP2_LUT[i + 1]
    return a + (((b - a) * lo + 128) >> 8)


def exp_neg_q(x_q16):
    """exp(x) for x<=0 in Q16 -> Q30 (ref/fixedpoint.py:109-121); vectorised."""
    x = np.asarray(x_q16, dtype=I64)
    assert (x <= 0).all()
    t = (x * I64(94548)) >> 16
    n = (-t + 0xFFFF) >> 16
    f = t + (n << 16)
    v = exp2_frac_q16(np.where(n >= 31, 0, f))
    left = v << np.clip(14 - n, 0, 62)
    right = v >> np.clip(n - 14, 0, 62)
    return np.where(n >= 31, I64(0), np.where(n <= 14, left, right))


def sigmoid_q(x_q12):
    """Q12 -> Q15 PWL sigmoid (ref/fixedpoint.py:135-147); vectorised."""
    x = np.clip(np.asarray(x_q12, dtype=I64), -16 << 12, (16 << 12) - 1)
    u = x + (16 << 12)
    i, lo = u >> 9, u & 0x1FF
    a, b = SIGMOID_LUT[i], SIGMOID_LUT[i + 1]
    return a + (((b - a) * lo + 256) >> 9)


def softplus_q(x_q12):
    """Q12 -> Q12 PWL softplus (ref/fixedpoint.py:150-165); vectorised."""
    x = np.asarray(x_q12, dtype=I64)
    u = np.clip(x + (16 << 12), 0, (32 << 12) - 1)
    i, lo = u >> 9, u & 0x1FF
    a, b = SOFTPLUS_LUT[i], SOFTPLUS_LUT[i + 1]
    mid = a + (((b - a) * lo + 256) >> 9)
    return np.where(x >= (16 << 12), x, np.where(x < (-16 << 12), I64(0), mid))


def silu_q(x_q12):
    """x*sigmoid(x), Q12 (ref/fixedpoint.py:168-171); vectorised."""
    x = np.asarray(x_q12, dtype=I64)
    return rshr(x * sigmoid_q(x), 15)


# ---------------------------------------------------------------------------
# W4A8 matvec and the row wire format (ref/w4a8_ref.py)
# ---------------------------------------------------------------------------
def row_beats(K, g=G):
    """ref/w4a8_ref.py:102-108."""
    assert g in (128, 64) and K % 128 == 0
    return K // 128, (K // g + 31) // 32


def row_stride(K, g=G):
    """ref/w4a8_ref.py:111-114."""
    wb, sb = row_beats(K, g)
    return (wb + sb) * 64


def final_shift(K, g=G):
    """sh = bitlen(NG*65535*(g*8*127)) - 31 (ref/w4a8_ref.py:177-179)."""
    NG = K // g
    return max(0, (NG * 65535 * (g * 8 * 127)).bit_length() - 31)


def pack_w4(w4):
    """(N,K) int4 codes -> (N,K/2) bytes, low nibble = even k
    (ref/w4a8_ref.py:331-334)."""
    u = (np.asarray(w4).astype(np.int16) & 0xF).astype(np.uint8)
    return (u[:, 0::2] | (u[:, 1::2] << 4)).astype(np.uint8)


def unpack_w4(packed, K):
    """ref/w4a8_ref.py:337-346."""
    packed = np.asarray(packed, dtype=np.uint8)
    lo = (packed & 0xF).astype(np.int8)
    hi = (packed >> 4).astype(np.int8)
    lo = np.where(lo > 7, lo - 16, lo).astype(np.int8)
    hi = np.where(hi > 7, hi - 16, hi).astype(np.int8)
    out = np.empty((packed.shape[0], K), dtype=np.int8)
    out[:, 0::2] = lo
    out[:, 1::2] = hi
    return out


def pack_ddr_rows(w4, m, g=G):
    """Per row [K/128 weight beats | ceil(NG/32) scale beats], tail zeroed
    (ref/w4a8_ref.py:349-370).  Returns (uint8 image (N, stride), stride)."""
    N, K = np.asarray(w4).shape
    stride = row_stride(K, g)
    img = np.zeros((N, stride), dtype=np.uint8)
    img[:, :K // 2] = pack_w4(w4)
    mb = np.asarray(m).astype("<u2").view(np.uint8).reshape(N, -1)
    img[:, K // 2:K // 2 + mb.shape[1]] = mb
    return img, stride


def unpack_ddr_rows(img, nrows, K, g=G):
    """ref/w4a8_ref.py:429-446."""
    stride = row_stride(K, g)
    a = np.asarray(img, dtype=np.uint8).reshape(nrows, stride)
    w4 = unpack_w4(a[:, :K // 2], K)
    NG = K // g
    m = a[:, K // 2:K // 2 + 2 * NG].copy().view("<u2").reshape(nrows, NG)
    return w4, m


def matvec_y32_np(w4, m, sh, x8, g=None):
    """Pure-numpy ref/w4a8_ref.py:254-289 (small shapes only)."""
    w4 = np.asarray(w4)
    N, K = w4.shape
    NG = np.asarray(m).shape[1]
    g = K // NG if g is None else g
    acc = (w4.reshape(N, NG, g).astype(I64)
           * np.asarray(x8).astype(I64).reshape(1, NG, g)).sum(axis=2)
    assert np.abs(acc).max() < (1 << 31)
    p = (np.asarray(m).astype(I64) * acc).sum(axis=1)
    y = rshr(p, sh)
    assert np.abs(y).max() < (1 << 31)
    return y.astype(np.int32)


# ---- the C restatement of the hot loop (oracle/c/f5_oracle.c) ----
_CLIB = None


def _clib():
    global _CLIB
    if _CLIB is None:
        here = os.path.dirname(os.path.abspath(__file__))
        path = os.path.join(here, "_build", "libf5oracle.so")
        if not os.path.exists(path):
            from . import build as _b
            _b.build()
        lib = ctypes.CDLL(path)
        lib.f5o_matvec_rows.restype = ctypes.c_int
        lib.f5o_matvec_rows.argtypes = [
            ctypes.c_void_p, ctypes.c_long, ctypes.c_int, ctypes.c_int,
            ctypes.c_int, ctypes.c_void_p, ctypes.c_int, ctypes.c_void_p,
            ctypes.c_void_p, ctypes.c_int]
        lib.f5o_num_threads.restype = ctypes.c_int
        _CLIB = lib
    return _CLIB


_THREADS = 0   # 0: the OpenMP default (OMP_NUM_THREADS)


def set_threads(n):
    """Thread count of every later C matvec (0: the OpenMP default).  A
    launcher such as torchrun sets OMP_NUM_THREADS=1; a CPU baseline that
    wants the host's cores sets them here explicitly."""
    global _THREADS
    _THREADS = max(0, int(n))


def oracle_threads():
    return _THREADS if _THREADS > 0 else int(_clib().f5o_num_threads())


def matvec_img(img, N, K, sh, x8, g=G, want_p=False, threads=0):
    """matvec_y32 over a packed DDR image (the DDRWeights.matvec view,
    ref/seq_model.py:431-452), computed by the C restatement."""
    img = np.ascontiguousarray(img, dtype=np.uint8)
    stride = row_stride(K, g)
    assert img.size >= N * stride
    x8 = np.ascontiguousarray(x8, dtype=np.int8)
    assert x8.size == K
    y = np.empty(N, dtype=np.int32)
    p = np.empty(N, dtype=I64) if want_p else None
    rc = _clib().f5o_matvec_rows(
        img.ctypes.data, stride, N, K, g, x8.ctypes.data, int(sh),
        y.ctypes.data, p.ctypes.data if p is not None else None, int(threads) if threads > 0 else _THREADS)
    if rc != 0:
        raise AssertionError(f"oracle matvec overflow assertion (rc={rc})")
    return (y, p) if want_p else y


class QMat:
    """A quantized matvec matrix held as its packed DDR image.

    Mirrors the reference dict {"w4","m","e","sh","g"} (ref/layer_fixed.py:
    1111) with the weights in the ``pack_ddr_rows`` wire form."""

    def __init__(self, img, N, K, e, sh=None, g=G):
        self.img = np.ascontiguousarray(img, dtype=np.uint8).reshape(N, row_stride(K, g))
        self.N, self.K, self.e, self.g = int(N), int(K), int(e), int(g)
        self.sh = final_shift(K, g) if sh is None else int(sh)

    @classmethod
    def from_dict(cls, qw):
        img, _ = pack_ddr_rows(qw["w4"], qw["m"], qw.get("g", G))
        N, K = qw["w4"].shape
        return cls(img, N, K, qw["e"], qw["sh"], qw.get("g", G))

    def to_dict(self):
        w4, m = unpack_ddr_rows(self.img, self.N, self.K, self.g)
        return {"w4": w4, "m": m, "e": self.e, "sh": self.sh, "g": self.g}

    def rows(self, r0, r1):
        return QMat(self.img[r0:r1], r1 - r0, self.K, self.e, self.sh, self.g)


def matvec_fx(qm: QMat, x16):
    """DYNQ8 + matvec_y32 (ref/layer_fixed.py:1201-1221)."""
    x8, e_x = dyn_quant_i8(x16)
    return matvec_img(qm.img, qm.N, qm.K, qm.sh, x8, qm.g), e_x


def matvec_to(qm: QMat, x16, in_f, out_f):
    """Second shift (15-e-sh) - e_x + in_f - out_f, either direction
    (ref/layer_fixed.py:1224-1236)."""
    y32, e_x = matvec_fx(qm, x16)
    sh = (15 - qm.e - qm.sh) - e_x + in_f - out_f
    y = y32.astype(I64)
    return rshr(y, sh) if sh >= 0 else y << I64(-sh)


# ---------------------------------------------------------------------------
# L2 vector blocks (ref/layer_fixed.py)
# ---------------------------------------------------------------------------
def bf_shift(absmax, guard=0):
    """ref/layer_fixed.py:442-467."""
    m = int(absmax)
    if m <= 0:
        return 0
    k = m.bit_length() - 15 + int(guard)
    if k > 0 and rshr_int(m, k) > 32767:
        k += 1
    return k


def attn_o_shift(absmax):
    """bf_shift clamped at 0 (ref/layer_fixed.py:489-506)."""
    return max(bf_shift(absmax), 0)


def rmsnorm_fx(x16, w_q14, in_f, one_plus):
    """ref/layer_fixed.py:1242-1278."""
    x = np.asarray(x16, dtype=I64)
    n = x.size
    nbits = n.bit_length() - 1
    assert (1 << nbits) == n, "N must be a power of two"
    ss = int((x * x).sum())
    if ss == 0:
        ss = 1
    r, e = rsqrt_q(ss, 2 * in_f + nbits)
    y = rshr(x * I64(r), 30 - e)
    y = np.clip(y, -(1 << 32), (1 << 32) - 1)
    w = np.asarray(w_q14, dtype=I64)
    scale = w + (1 << 14) if one_plus else w
    return clip16(rshr(y * scale, 14))


def l2norm_fx(x16, in_f, out_f):
    """ref/layer_fixed.py:1322-1330."""
    x = np.asarray(x16, dtype=I64)
    ss = int((x * x).sum())
    if ss == 0:
        ss = 1
    r, e = rsqrt_q(ss, 2 * in_f)
    return clip16(rshr(x * I64(r), in_f + 30 - e - out_f))


def rope_cos_sin(pos, geom=GEOM_9B):
    """float32 cos/sin over ROT dims (ref/layer_ref.py:84-90)."""
    ROT = geom.ROT
    inv = 1.0 / (geom.THETA ** (np.arange(0, ROT, 2, dtype=np.float64) / ROT))
    f = pos * inv
    emb = np.concatenate([f, f])
    return np.cos(emb).astype(np.float32), np.sin(emb).astype(np.float32)


def rope_tables_q15(pos, geom=GEOM_9B):
    """ref/layer_fixed.py:1333-1337."""
    cos, sin = rope_cos_sin(pos, geom)
    return (np.clip(np.round(cos * (1 << ROPE_F)), -32767, 32767).astype(I64),
            np.clip(np.round(sin * (1 << ROPE_F)), -32767, 32767).astype(I64))


def rope_fx(x16, cos_q, sin_q, rot=64):
    """Rotate the first ROT dims (ref/layer_fixed.py:1340-1348)."""
    x = np.asarray(x16, dtype=I64)
    xr, xp = x[..., :rot], x[..., rot:]
    h = rot // 2
    rr = np.concatenate([-xr[..., h:], xr[..., :h]], axis=-1)
    y = rshr(xr * cos_q + rr * sin_q, ROPE_F)
    return clip16(np.concatenate([y, xp], axis=-1))


def kv_quant(v16, in_f):
    """ref/layer_fixed.py:1377-1380."""
    x8, e = dyn_quant_i8(v16)
    return x8.astype(np.int8), e - in_f


def dn_norm_scale(o32, k_h):
    """Float64 gated-norm scale (ref/layer_fixed.py:509-546)."""
    x = np.asarray(o32, dtype=I64)
    ss = int((x * x).sum())                      # numpy int64 (wraps)
    mean = ss / float(1 << (2 * S_F)) / float(len(x))
    s = 1.0 / np.sqrt(mean + EPS)
    A = s * (2.0 ** (DN_NORM_F - S_F))
    m_raw = round(A * (2.0 ** (15 + k_h)))
    return int(np.clip(m_raw, 0, M_Q15_MAX))


def eps_ss_addend(k, in_f=S_F, n_log2=7):
    """ref/layer_fixed.py:681-691."""
    return rshr_int(EPS_M, EPS_Q - (2 * (int(in_f) - int(k)) + n_log2))


def eps_norm_scale(x16, k, in_f=S_F, out_f=DN_NORM_F):
    """Integer EPS-NORM scale (ref/layer_fixed.py:694-767)."""
    x = np.asarray(x16, dtype=I64)
    n = x.size
    nbits = n.bit_length() - 1
    ss = int((x * x).sum())
    v = ss + eps_ss_addend(k, in_f, nbits)
    if v <= 0:
        v = 1
    p = 2 * int(in_f) + nbits
    r, e = rsqrt_q(v, p)
    sh = int(in_f) - int(out_f) + 15 - int(e)
    return int(np.clip(rshr_int(r, sh), 0, M_Q15_MAX))


def script_norm_fx(o32, o16, k_h, w_q14, norm_mode="float"):
    """Gated RMSNorm, float (default) or integer EPS-NORM mode
    (ref/layer_fixed.py:1281-1319, 770-781)."""
    if norm_mode == "eps":
        scale = eps_norm_scale(o16, k_h)
    else:
        scale = dn_norm_scale(o32, k_h)
    t = clip16(rshr(clip16(o16) * I64(scale), 15))
    return clip16(rshr(t * np.asarray(w_q14, dtype=I64), 14))


# ---------------------------------------------------------------------------
# caches (GPU-friendly arrays; converters to the reference dict layout)
# ---------------------------------------------------------------------------
class AttnCache:
    """int8 K/V mantissas + per-(token, kv head) exponents.

    Reference layout: {"k": [[(k8, ke)] * NKV] * T, "v": ...}
    (ref/layer_fixed.py:1400-1401, 1654-1656)."""

    def __init__(self, max_T, geom=GEOM_9B):
        self.k8 = np.zeros((geom.NKV, max_T, geom.HD), dtype=np.int8)
        self.ke = np.zeros((geom.NKV, max_T), dtype=np.int8)
        self.v8 = np.zeros((geom.NKV, max_T, geom.HD), dtype=np.int8)
        self.ve = np.zeros((geom.NKV, max_T), dtype=np.int8)
        self.T = 0
        self.attn_o_shift = 0

    def to_ref(self):
        NKV = self.k8.shape[0]
        return {"k": [[(self.k8[h, t].copy(), int(self.ke[h, t])) for h in range(NKV)]
                      for t in range(self.T)],
                "v": [[(self.v8[h, t].copy(), int(self.ve[h, t])) for h in range(NKV)]
                      for t in range(self.T)]}

    @classmethod
    def from_ref(cls, c, max_T, geom=GEOM_9B):
        a = cls(max_T, geom)
        a.T = len(c["k"])
        for t in range(a.T):
            for h in range(geom.NKV):
                a.k8[h, t], a.ke[h, t] = c["k"][t][h]
                a.v8[h, t], a.ve[h, t] = c["v"][t][h]
        return a


class DNCache:
    """conv window int64 [CONV_DIM, 3] (oldest first) + state S int16
    [LNH, LDK, LDV] (ref/layer_fixed.py:1654-1666)."""

    def __init__(self, geom=GEOM_9B):
        self.conv = np.zeros((geom.CONV_DIM, geom.CONV_K - 1), dtype=I64)
        self.S = np.zeros((geom.LNH, geom.LDK, geom.LDV), dtype=np.int16)
        self.sat = 0
        self.dn_o_shift = []

    def to_ref(self):
        return {"conv": self.conv.copy(), "S": self.S.copy()}

    @classmethod
    def from_ref(cls, c, geom=GEOM_9B):
        a = cls(geom)
        a.conv[...] = c["conv"]
        a.S[...] = c["S"]
        return a


# ---------------------------------------------------------------------------
# attention / DeltaNet / MLP / layer
# ---------------------------------------------------------------------------
def attn_decode_fx(xn16, qa, cache: AttnCache, pos, geom=GEOM_9B):
    """ref/layer_fixed.py:1383-1449.  qa: {"q_proj","k_proj","v_proj",
    "o_proj": QMat, "q_norm","k_norm": int64[HD]}."""
    NQ, NKV, HD = geom.NQ, geom.NKV, geom.HD
    qg = matvec_to(qa["q_proj"], xn16, RS_F, QKV_F).reshape(NQ, 2 * HD)
    q16, gate = clip16(qg[:, :HD]), clip16(qg[:, HD:])
    k16 = clip16(matvec_to(qa["k_proj"], xn16, RS_F, QKV_F).reshape(NKV, HD))
    v16 = clip16(matvec_to(qa["v_proj"], xn16, RS_F, QKV_F).reshape(NKV, HD))
    cos_q, sin_q = rope_tables_q15(pos, geom)
    qn = np.stack([rope_fx(rmsnorm_fx(q16[h], qa["q_norm"], QKV_F, True), cos_q, sin_q, geom.ROT)
                   for h in range(NQ)])
    kn = np.stack([rope_fx(rmsnorm_fx(k16[h], qa["k_norm"], QKV_F, True), cos_q, sin_q, geom.ROT)
                   for h in range(NKV)])
    t_new = cache.T
    for h in range(NKV):
        cache.k8[h, t_new], cache.ke[h, t_new] = kv_quant(kn[h], QKV_F)
        cache.v8[h, t_new], cache.ve[h, t_new] = kv_quant(v16[h], QKV_F)
    cache.T = T = t_new + 1
    group = NQ // NKV
    SCALE_Q15 = int(round((1 << 15) / np.sqrt(HD)))
    out = np.zeros((NQ, HD), dtype=I64)
    for h in range(NQ):
        kv = h // group
        k8 = cache.k8[kv, :T].astype(I64)
        ke = cache.ke[kv, :T].astype(I64)
        dot = k8 @ qn[h]
        s = rshr(dot * I64(SCALE_Q15), 15)
        f = QKV_F - ke - 16
        sc = rshr_v(s, f)
        mx = int(sc.max())
        es = exp_neg_q(np.minimum(sc - mx, 0))
        r, re = recip_q(int(es.sum()), 30)
        p = np.clip(rshr(es * I64(r), 30 - re + 15), 0, 1 << 15)
        v8 = cache.v8[kv, :T].astype(I64)
        ve = cache.ve[kv, :T].astype(I64)
        term = p[:, None] * v8
        out[h] = rshr_v(term, (15 - ve - QKV_F)[:, None]).sum(axis=0)
    og = sigmoid_q(rshr(gate.reshape(-1), QKV_F - 12))
    prod = out.reshape(-1) * og
    k_a = attn_o_shift(int(np.abs(prod).max()))
    gated = rshr(prod, k_a)
    cache.attn_o_shift = k_a
    y = matvec_to(qa["o_proj"], clip16(gated), QKV_F + GAT_F - k_a, RS_F)
    return clip16(y)


def deltanet_decode_fx(xn16, qd, state: DNCache, geom=GEOM_9B, norm_mode="float"):
    """ref/layer_fixed.py:1493-1580 (int16 state container, the default
    dn_state_narrow law ref/layer_fixed.py:336-348).  qd: {"in_qkv","in_z",
    "in_b","in_a","out": QMat, "conv_w": int64[C,4], "dt_bias_q12","A_q15":
    int64[LNH], "norm_w_q14": int64[LDV]}."""
    LNH, LDK, LDV, LNKH, LKD, VREP = (geom.LNH, geom.LDK, geom.LDV, geom.LNKH,
                                       geom.LKD, geom.VREP)
    qkv16 = clip16(matvec_to(qd["in_qkv"], xn16, RS_F, RS_F))
    z16 = clip16(matvec_to(qd["in_z"], xn16, RS_F, QKV_F)).reshape(LNH, LDV)
    b_q12 = clip16(matvec_to(qd["in_b"], xn16, RS_F, 12))
    a_q12 = clip16(matvec_to(qd["in_a"], xn16, RS_F, 12))

    win = np.concatenate([state.conv, qkv16[:, None]], axis=1)
    state.conv = win[:, 1:].copy()
    acc = (win.astype(I64) * np.asarray(qd["conv_w"], dtype=I64)).sum(axis=1)
    pre = np.clip(rshr(acc, RS_F + CW_F - 12), -(1 << 20), (1 << 20) - 1)
    conv_out = clip16(silu_q(pre))
    qkv = rshr(conv_out, 12 - QKV_F)
    q = qkv[:LKD].reshape(LNKH, LDK)
    k = qkv[LKD:2 * LKD].reshape(LNKH, LDK)
    v = qkv[2 * LKD:].reshape(LNH, LDV)

    beta = sigmoid_q(b_q12)
    sp = softplus_q(a_q12 + np.asarray(qd["dt_bias_q12"], dtype=I64))
    g_q16 = -rshr(np.asarray(qd["A_q15"], dtype=I64) * sp, 15 + 12 - 16)
    decay = np.minimum(rshr(exp_neg_q(np.minimum(g_q16, 0)), 15), 32767)

    INV_SQRT_DK_Q15 = int(round((1 << 15) / np.sqrt(LDK)))
    qn_k = np.stack([rshr(l2norm_fx(q[j], QKV_F, NRM_F) * I64(INV_SQRT_DK_Q15), 15)
                     for j in range(LNKH)])
    kn_k = np.stack([l2norm_fx(k[j], QKV_F, NRM_F) for j in range(LNKH)])
    kh = np.arange(LNH) // VREP
    qn, kn = qn_k[kh], kn_k[kh]                    # (LNH, LDK)

    Sh = rshr(state.S.astype(I64) * decay[:, None, None], GAT_F)
    kv_mem = rshr((Sh * kn[:, :, None]).sum(axis=1), NRM_F)
    v_s = (rshr(v, QKV_F - S_F) if QKV_F >= S_F else v << I64(S_F - QKV_F))
    delta = rshr((v_s - kv_mem) * beta[:, None], GAT_F)
    Sh = Sh + rshr(kn[:, :, None] * delta[:, None, :], NRM_F)
    state.sat += int((np.abs(Sh) > 32767).sum())
    Sh = clip16(Sh)
    o32 = rshr((Sh * qn[:, :, None]).sum(axis=1), NRM_F)     # (LNH, LDV)
    state.S[...] = Sh.astype(np.int16)
    k_log = [bf_shift(int(np.abs(o32[h]).max())) for h in range(LNH)]
    o16 = np.stack([clip16(rshr(o32[h], k_log[h])) for h in range(LNH)])
    state.dn_o_shift = k_log

    zg = clip16(silu_q(rshr(z16, QKV_F - 12)))
    on = np.zeros((LNH, LDV), dtype=I64)
    for h in range(LNH):
        nh = script_norm_fx(o32[h], o16[h], k_log[h], qd["norm_w_q14"], norm_mode)
        on[h] = rshr(nh * zg[h], 12)
    y = matvec_to(qd["out"], clip16(on.reshape(-1)), DN_NORM_F, RS_F)
    return clip16(y)


def mlp_fx(xn16, qm):
    """ref/layer_fixed.py:1597-1604."""
    g = matvec_to(qm["gate"], xn16, RS_F, 12)
    u = matvec_to(qm["up"], xn16, RS_F, RS_F)
    sg = clip16(silu_q(np.clip(g, -(1 << 20), (1 << 20) - 1)))
    prod = clip16(rshr(sg * u, 12))
    return clip16(matvec_to(qm["down"], prod, RS_F, RS_F))


def layer_decode_fx(x16, qw, cache, pos, geom=GEOM_9B, norm_mode="float"):
    """ref/layer_fixed.py:1669-1677."""
    xn = rmsnorm_fx(x16, qw["ln1"], RS_F, True)
    if qw["type"] == "full_attention":
        h = attn_decode_fx(xn, qw["attn"], cache, pos, geom)
    else:
        h = deltanet_decode_fx(xn, qw["dn"], cache, geom, norm_mode)
    x16 = clip16(np.asarray(x16, dtype=I64) + h)
    xn = rmsnorm_fx(x16, qw["ln2"], RS_F, True)
    return clip16(x16 + mlp_fx(xn, qw["mlp"]))


def argmax_first(y):
    """np.argmax (first max wins) -- ref/gen_model_script.py:641 and the
    AMAX32 strictly-greater scan ref/gen_layer_script.py:1424-1433."""
    return int(np.argmax(np.asarray(y)))


class OracleRunner:
    """Full-model integer decode step, restating FxRunner.step
    (ref/fidelity_check.py:404-448) and the token loop of
    ref/gen_model_script.py:602-650."""

    def __init__(self, model, max_T=64, norm_mode="float"):
        self.m = model
        self.geom = model.geom
        self.max_T = max_T
        self.norm_mode = norm_mode
        self.reset()

    def reset(self):
        self.caches = [AttnCache(self.max_T, self.geom) if t == "full_attention"
                       else DNCache(self.geom) for t in self.geom.layer_types]
        self.layer_out = []
        self.resid_max = 0
        self.resid_clip = 0

    def step_logits(self, tok, pos):
        m = self.m
        x = m.emb_row(tok).astype(I64)
        self.layer_out = []
        for i, qw in enumerate(m.layers):
            x = layer_decode_fx(x, qw, self.caches[i], pos, self.geom, self.norm_mode)
            self.layer_out.append(x.copy())
            self.resid_max = max(self.resid_max, int(np.abs(x).max()))      # ref/fidelity_check.py:430
            self.resid_clip += int(((x >= 32767) | (x <= -32768)).sum())   # :431
        xn = rmsnorm_fx(x, m.ln_f_q12, RS_F, False)
        x8, _ = dyn_quant_i8(xn)
        h = m.head
        return matvec_img(h.img, h.N, h.K, h.sh, x8, h.g)

    def step(self, tok, pos):
        y = self.step_logits(tok, pos)
        return argmax_first(y), y

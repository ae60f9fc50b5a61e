"""Seeded synthetic Qwen3.5-9B integer model (bench and test inputs).

There is no checkpoint here, so every benchmark and parity case runs on
seeded synthetic weights with the 9B shapes, generated directly in the
reference's integer dict layout:

* W4 matrices: packed ``pack_ddr_rows`` images (ref/w4a8_ref.py:349-370).
  Two code laws: ``uniform`` -- every byte uniform, i.e. two int4 codes
  uniform in [-8, 7] (the standalone matvec / LM-head cases, which must
  reach the -8 rail); ``symmetric`` -- each nibble read as sign-magnitude,
  codes in [-7, 7] with zero mean (the full-model cases: U{-8..7} has mean
  -0.5, and that common-mode bias drives a 32-layer random model into
  whole-vector residual saturation within four layers).
  Group mantissas m are uniform in [2^13, 2^14) -- the range
  ``quantize_weights`` produces (ref/w4a8_ref.py:171-173).  The per-matrix
  exponent e is fixed per role (input projections ``E_IN``, residual-adding
  projections one step lower ``E_RES``, cf. the ``out_scale`` idea of
  ref/layer_ref.py:143-166); ``sh`` is the reference's rule
  (ref/w4a8_ref.py:177-179).
* Bytes come from a counter-based hash (splitmix64 finaliser over
  (seed, matrix id, word index)), so any row range of any matrix can be
  regenerated independently, on the host (numpy, here) or on the device
  (``f5_synth_w4_image`` in the CUDA library) with identical bytes.
* Embedding rows: int16 = (b0 + b1) - 255 from two hash bytes per element
  (a triangular stand-in for round(N(0,1) * 2^7), std ~105).
* Small vector parameters (norm gains, conv taps, gates) use
  ``np.random.default_rng`` with the distributions of ref/layer_ref.py:107-166
  made integer (ref/layer_fixed.py:1360-1375, 1455-1490, 1607-1651).
"""
from __future__ import annotations

import numpy as np

I64 = np.int64
U64 = np.uint64
MASK64 = (1 << 64) - 1

GOLDEN = 0x9E3779B97F4A7C15
C1 = 0xBF58476D1CE4E5B9
C2 = 0x94D049BB133111EB
KM = 0xD1B54A32D192ED03
KS = 0xABC98388FB8FAC03

E_IN = -6       # input projections
E_RES = -9      # residual-adding projections (o_proj, dn out, mlp down)
E_HEAD = -6

# matrix ids: layer * 16 + slot
SLOT = {"in_qkv": 0, "in_z": 1, "in_b": 2, "in_a": 3, "out": 4,
        "q_proj": 0, "k_proj": 1, "v_proj": 2, "o_proj": 3,
        "gate": 8, "up": 9, "down": 10}
MID_HEAD = 1 << 20
MID_EMB = (1 << 20) + 1
STREAM_W, STREAM_M, STREAM_E = 0, 1, 2


def _mix_int(z: int) -> int:
    z &= MASK64
    z = ((z ^ (z >> 30)) * C1) & MASK64
    z = ((z ^ (z >> 27)) * C2) & MASK64
    return z ^ (z >> 31)


def stream_key(seed: int, mid: int, stream: int) -> int:
    return _mix_int((seed * GOLDEN + mid * KM + stream * KS + 1) & MASK64)


def _mix_arr(z):
    z = z ^ (z >> U64(30))
    z = z * U64(C1)
    z = z ^ (z >> U64(27))
    z = z * U64(C2)
    return z ^ (z >> U64(31))


def hash_words(key: int, start: int, count: int):
    """word(i) = mix64(key + (i+1)*GOLDEN) for i in [start, start+count)."""
    i = np.arange(start + 1, start + count + 1, dtype=U64)
    with np.errstate(over="ignore"):
        return _mix_arr(U64(key) + i * U64(GOLDEN))


def row_stride(K, g=128):
    return (K // 128 + (K // g + 31) // 32) * 64


def final_shift(K, g=128):
    NG = K // g
    return max(0, (NG * 65535 * (g * 8 * 127)).bit_length() - 31)


def _sym_byte_lut():
    """byte -> byte with each nibble c mapped to the two's-complement code of
    (c & 7) * (-1 if c & 8 else 1)."""
    c = np.arange(16)
    v = np.where(c & 8, -(c & 7), c & 7) & 0xF
    b = np.arange(256)
    return (v[b & 0xF] | (v[b >> 4] << 4)).astype(np.uint8)


SYM_LUT = _sym_byte_lut()


def w4_image(seed, mid, N, K, g=128, r0=0, r1=None, symmetric=False):
    """Rows [r0, r1) of the packed image of matrix ``mid`` -> uint8
    (r1-r0, stride)."""
    r1 = N if r1 is None else r1
    n = r1 - r0
    stride = row_stride(K, g)
    NG = K // g
    wpr = K // 16                      # 8-byte words of weight bytes per row
    img = np.zeros((n, stride), dtype=np.uint8)
    kw = stream_key(seed, mid, STREAM_W)
    w = hash_words(kw, r0 * wpr, n * wpr)
    wb = w.view(np.uint8).reshape(n, K // 2)
    img[:, :K // 2] = SYM_LUT[wb] if symmetric else wb
    km = stream_key(seed, mid, STREAM_M)
    m = (hash_words(km, r0 * NG, n * NG) & U64(0x1FFF)) | U64(0x2000)
    img[:, K // 2:K // 2 + 2 * NG] = m.astype("<u2").view(np.uint8).reshape(n, 2 * NG)
    return img


def emb_rows(seed, toks, H=4096):
    """int16 embedding rows for token ids ``toks``."""
    toks = np.atleast_1d(np.asarray(toks, dtype=np.int64))
    ke = stream_key(seed, MID_EMB, STREAM_E)
    out = np.empty((toks.size, H), dtype=np.int16)
    for i, t in enumerate(toks):
        w = hash_words(ke, int(t) * (H // 4), H // 4)
        b = w.view(np.uint8).reshape(H, 2).astype(np.int16)
        out[i] = b[:, 0] + b[:, 1] - 255
    return out


# ---------------------------------------------------------------------------
# model description
# ---------------------------------------------------------------------------
def dn_shapes(g):
    return {"in_qkv": (g.CONV_DIM, g.H), "in_z": (g.LVD, g.H), "in_b": (g.LNH, g.H),
            "in_a": (g.LNH, g.H), "out": (g.H, g.LVD)}


def attn_shapes(g):
    return {"q_proj": (g.NQ * g.HD * 2, g.H), "k_proj": (g.NKV * g.HD, g.H),
            "v_proj": (g.NKV * g.HD, g.H), "o_proj": (g.H, g.NQ * g.HD)}


def mlp_shapes(g):
    return {"gate": (g.FFN, g.H), "up": (g.FFN, g.H), "down": (g.H, g.FFN)}


RES_MATS = ("out", "o_proj", "down")


class MatSpec:
    __slots__ = ("name", "layer", "mid", "N", "K", "e", "sh", "g", "symmetric")

    def __init__(self, name, layer, mid, N, K, e, g=128, symmetric=True):
        self.name, self.layer, self.mid = name, layer, mid
        self.N, self.K, self.e, self.g = N, K, e, g
        self.sh = final_shift(K, g)
        self.symmetric = symmetric

    def image(self, seed, r0=0, r1=None):
        return w4_image(seed, self.mid, self.N, self.K, self.g, r0, r1, self.symmetric)

    @property
    def stride(self):
        return row_stride(self.K, self.g)

    @property
    def nbytes(self):
        return self.N * self.stride


def matrix_specs(geom):
    """Every W4 matrix of the model in decode order (249 at 9B)."""
    out = []
    for i, lt in enumerate(geom.layer_types):
        body = attn_shapes(geom) if lt == "full_attention" else dn_shapes(geom)
        for nm, (N, K) in list(body.items()) + list(mlp_shapes(geom).items()):
            e = E_RES if nm in RES_MATS else E_IN
            out.append(MatSpec(nm, i, i * 16 + SLOT[nm], N, K, e))
    out.append(MatSpec("head", -1, MID_HEAD, geom.vocab, geom.H, E_HEAD))
    return out


def vector_params(seed, geom):
    """Per-layer integer vector parameters + ln_f (numpy default_rng)."""
    layers = []
    for i, lt in enumerate(geom.layer_types):
        rng = np.random.default_rng([seed, i])
        p = {"ln1": np.round(rng.normal(0, 0.1, geom.H) * (1 << 14)).astype(I64),
             "ln2": np.round(rng.normal(0, 0.1, geom.H) * (1 << 14)).astype(I64)}
        if lt == "full_attention":
            p["q_norm"] = np.round(rng.normal(0, 0.1, geom.HD) * (1 << 14)).astype(I64)
            p["k_norm"] = np.round(rng.normal(0, 0.1, geom.HD) * (1 << 14)).astype(I64)
        else:
            p["conv_w"] = np.round(rng.normal(0, 0.3, (geom.CONV_DIM, geom.CONV_K))
                                   * (1 << 13)).astype(I64)
            p["dt_bias_q12"] = np.full(geom.LNH, 4096, dtype=I64)
            p["A_q15"] = np.clip(np.round(rng.uniform(0.5, 8, geom.LNH) * (1 << 15)),
                                 0, (1 << 18) - 1).astype(I64)
            p["norm_w_q14"] = np.round((1 + rng.normal(0, 0.1, geom.LDV))
                                       * (1 << 14)).astype(I64)
        layers.append(p)
    rng = np.random.default_rng([seed, 1 << 16])
    ln_f = np.round((1 + rng.normal(0, 0.1, geom.H)) * (1 << 12)).astype(I64)
    return layers, ln_f


def token_ids(seed, n, vocab):
    """Seeded random prompt token ids in [0, vocab)."""
    return np.random.default_rng([seed, 7]).integers(0, vocab, n).astype(np.int64)


def matvec_input(seed, K=4096, rs_f=7):
    """Config-1 activation: x ~ N(0,1) fp32 -> x16 = round(x * 2^rs_f)."""
    x = np.random.default_rng([seed, 11]).normal(0, 1.0, K).astype(np.float32)
    return np.round(x.astype(np.float64) * (1 << rs_f)).astype(I64)

"""Drop-in for ref/layer_fixed.py at the 9B operating point, on the GPU.

Same names, arguments and return values as the reference for the decode
path: ``matvec_fx``, ``matvec_to``, ``rmsnorm_fx``, ``layer_decode_fx``,
``new_cache_fx``, ``kv_quant``, ``bf_shift`` and the norm-scale helpers.
Quantized matrices are the reference's dicts ``{"w4","m","e","sh","g"}``;
caches are the reference's dicts and lists and are mutated in place the way
the reference mutates them.  Like the reference's module-global
``SEQ_NORM``, the DeltaNet gated-norm law is chosen by the module global
``SEQ_NORM`` (False: float64 host scale; True: integer EPS-NORM).

``layer_decode_fx`` runs one layer through a single-layer GPU context that
is cached per layer dict (at most ``MAX_LAYER_CTX`` of them, least recently
used evicted; ``release_layer`` / ``clear_layer_cache`` free them); the
cache state is uploaded before and read back after every call, so this
entry point is for parity and drop-in use -- the production path is
``fable5_llm_b200.model.DecodeModel.decode_step``.
"""
from __future__ import annotations

import numpy as np

from . import _lib as L
from .config import CW_F, DN_NORM_F, GAT_F, NRM_F, QKV_F, ROPE_F, RS_F, S_F, Geometry  # noqa: F401
from .w4a8_ref import G, matvec_y32

I64 = np.int64
SEQ_NORM = False
EPS_RMS_Q = 1
M_Q15_MAX = 65535


def clip16(x):
    """ref/layer_fixed.py:809."""
    return np.clip(np.asarray(x, dtype=I64), -32768, 32767)


def _ops():
    from . import ops
    return ops


def bf_shift(absmax, guard=0):
    """ref/layer_fixed.py:442-467 (GPU)."""
    k = int(_ops().prim(L.PR_BF_SHIFT, np.array([int(absmax)]))[0]) if int(absmax) > 0 else 0
    return k + int(guard) if guard and int(absmax) > 0 else k


def dn_o_shift(o32, note=True):
    """ref/layer_fixed.py:470-486."""
    return bf_shift(int(np.abs(np.asarray(o32, dtype=I64)).max()))


def attn_o_shift(absmax, note=True):
    """ref/layer_fixed.py:489-506."""
    return max(bf_shift(absmax), 0)


def dn_norm_scale(o32, k_h, note=True):
    """ref/layer_fixed.py:509-546 (GPU, IEEE float64)."""
    x = np.asarray(o32, dtype=I64)
    ss = np.array([int((x * x).sum())], dtype=I64)
    return int(_ops().prim(L.PR_DN_NORM_SCALE, ss, arg0=len(x), in2=np.array([int(k_h)]))[0])


def eps_norm_scale(x16, k, in_f=None, out_f=None, note=True):
    """ref/layer_fixed.py:694-767 (GPU; in_f = S_F, out_f = DN_NORM_F)."""
    assert in_f in (None, S_F) and out_f in (None, DN_NORM_F), "only the DeltaNet formats are bound"
    x = np.asarray(x16, dtype=I64)
    nbits = x.size.bit_length() - 1
    ss = np.array([int((x * x).sum())], dtype=I64)
    return int(_ops().prim(L.PR_EPS_NORM_SCALE, ss, arg0=nbits, in2=np.array([int(k)]))[0])


def qw_codes(qw):
    """ref/layer_fixed.py:1152-1165 (W4 only on this path)."""
    assert "w8" not in qw, "W8 images are not part of the 9B W4A8 decode path"
    return qw["w4"], False


def matvec_fx(qw, x16, out_f):
    """ref/layer_fixed.py:1201-1221 -> (y32, e_x)."""
    from .fixedpoint import dyn_quant_i8
    x8, e_x = dyn_quant_i8(x16)
    w, _ = qw_codes(qw)
    return matvec_y32(w, qw["m"], qw["sh"], x8, g=qw.get("g", G)), e_x


def matvec_to(qw, x16, in_f, out_f):
    """ref/layer_fixed.py:1224-1236 -> int64 y."""
    y32, e_x = matvec_fx(qw, x16, out_f)
    sh = (15 - qw["e"] - qw["sh"]) - e_x + in_f - out_f
    y = y32.astype(I64)
    from .w4a8_ref import rshift_round
    return rshift_round(y, sh) if sh >= 0 else y << I64(-sh)


def rmsnorm_fx(x16, w_q14, in_f, one_plus):
    """ref/layer_fixed.py:1242-1278 (GPU)."""
    import torch
    x = np.asarray(x16, dtype=I64)
    n = x.size
    if n & (n - 1):
        raise SystemExit(f"rmsnorm_fx: N={n} is not a power of two")
    ops = _ops()
    xn, _, _ = ops.rmsnorm_dynq8(ops.to_dev(clip16(x).astype(np.int16)),
                                 ops.to_dev(np.asarray(w_q14, dtype=I64).astype(np.int32)), n, in_f, one_plus)
    torch.cuda.synchronize()
    return xn.cpu().numpy().astype(I64)


def kv_quant(v16, in_f):
    """ref/layer_fixed.py:1377-1380."""
    from .fixedpoint import dyn_quant_i8
    x8, e = dyn_quant_i8(v16)
    return x8.astype(np.int8), e - in_f


def new_cache_fx(layer_type):
    """ref/layer_fixed.py:1654-1666."""
    g = Geometry()
    if layer_type == "full_attention":
        return {"k": [], "v": []}
    return {"conv": np.zeros((g.CONV_DIM, g.CONV_K - 1), dtype=I64),
            "S": np.zeros((g.LNH, g.LDK, g.LDV), dtype=np.int16)}


# GPU contexts of the layer dicts seen by layer_decode_fx, most recently used
# last.  Each entry holds the dict itself and every array it was uploaded
# from, so a cached id can never be handed to another dict (the dict stays
# alive while cached) and a matrix or vector replaced inside the dict is seen
# as a change.  Arrays modified in place are not detected: call
# release_layer(qw) (or clear_layer_cache()) after editing one.
_CTX = {}
MAX_LAYER_CTX = 40


def _leaves(qw):
    """(path, value) of every array and scalar of a layer dict, in a fixed order."""
    out = []

    def walk(p, v):
        if isinstance(v, dict):
            for k in sorted(v):
                walk(p + (k,), v[k])
        else:
            out.append((p, v))
    walk((), qw)
    return out


def _same_leaves(a, b):
    if len(a) != len(b):
        return False
    for (pa, va), (pb, vb) in zip(a, b):
        if pa != pb:
            return False
        if isinstance(va, np.ndarray) or isinstance(vb, np.ndarray):
            if va is not vb:
                return False
        elif type(va) is not type(vb) or va != vb:
            return False
    return True


class _LayerCtx:
    def __init__(self, qw, max_T):
        from .model import DecodeModel
        self.qw = qw
        self.leaves = _leaves(qw)
        self.type = qw["type"]
        self.max_T = max_T
        self.mode = SEQ_NORM
        self.m = DecodeModel(Geometry(1, 16, [self.type]), max_T=max_T,
                             norm_mode="eps" if SEQ_NORM else "float", max_pos=max(max_T, 4096))
        self.m.upload_layer(0, qw)

    def close(self):
        self.m.close()


def release_layer(qw):
    """Free the GPU context that layer_decode_fx holds for this dict."""
    c = _CTX.pop(id(qw), None)
    if c is not None:
        c.close()


def clear_layer_cache():
    """Free every GPU context that layer_decode_fx holds."""
    for c in list(_CTX.values()):
        c.close()
    _CTX.clear()


def _layer_ctx(qw, T):
    key = id(qw)
    c = _CTX.pop(key, None)
    need = max(64, 1 << (T + 1).bit_length())
    if c is not None and (c.qw is not qw or c.max_T < T + 1 or c.mode != SEQ_NORM or c.type != qw["type"]
                          or not _same_leaves(c.leaves, _leaves(qw))):
        c.close()
        c = None
    if c is None:
        while len(_CTX) >= MAX_LAYER_CTX:
            _CTX.pop(next(iter(_CTX))).close()
        c = _LayerCtx(qw, need)
    _CTX[key] = c
    return c


def layer_decode_fx(x16, qw, cache, pos):
    """ref/layer_fixed.py:1669-1677: one decoder layer, cache mutated in place."""
    attn = qw["type"] == "full_attention"
    T = len(cache["k"]) if attn else 0
    c = _layer_ctx(qw, T)
    m = c.m
    if attn:
        m.set_kv(0, cache)
    else:
        m.set_dn_state(0, 3, cache)    # any T works for the ring; 3 keeps slots 0..2
    y = m.layer_step(0, clip16(x16), T if attn else 3, pos)
    if attn:
        kv = m.get_kv(0, T + 1)
        cache["k"].append(kv["k"][T])
        cache["v"].append(kv["v"][T])
        cache["attn_o_shift"] = int(m.read(L.BUF_KA, 0)[0])
    else:
        st = m.get_dn_state(0, 4)
        cache["conv"] = st["conv"]
        cache["S"][...] = st["S"]
        cache["dn_o_shift"] = [int(v) for v in m.read(L.BUF_DN_KH, 0)]
    return y

"""Drop-in for the reference's checkpoint quantizers, computed on the GPU.

Same names, arguments, return values and refusals as
``quantize_weights`` (ref/w4a8_ref.py:154-180), ``quant_linear_mse``,
``quant_linear``, ``quant_attn``, ``quant_deltanet``, ``quant_mlp`` and
``quant_layer`` (ref/layer_fixed.py:981-1111, 1354-1376, 1455-1494,
1586-1651).  Every weight matrix goes through ``f5_quant_w4_scales`` /
``f5_quant_w4_pack`` (fable5_llm_b200/csrc/f5_quant.cu): the group-scale
search and the codes are computed on the device in IEEE binary64 in the
reference's own operation and summation order, so the w4 / m / e / sh
results are bit-identical to the reference's numpy quantizer.  The per-layer
vectors (norm gains, conv taps, gate constants) are a few thousand values
and are rounded on the host with the reference's formulas.

``quant_linear_image`` returns the packed row image (the format the decode
engines keep resident) without unpacking it, which is what a checkpoint
loader uploads.

Not built: the GPTQ quantizer (``hess``, ref/gptq.py), the W8 format
(``w8=True``) and the calibration-statistics plumb (FABLE5_CALIB_STATS);
each raises ``NotImplementedError`` where the reference would run it.
"""
from __future__ import annotations

import ctypes
import os

import numpy as np

from . import _lib as L
from .w4a8_ref import final_shift, row_stride

G = 128
I64 = np.int64
f32 = np.float32

# gate_unit port limits (ref/layer_fixed.py:805-806): dt_bias Q12 and A Q15
DT_Q12_MIN, DT_Q12_MAX = -32768, 32767
A_Q15_MAX = (1 << 18) - 1
CW_F = 13           # conv tap fraction bits (ref/layer_fixed.py:145)


def _torch():
    import torch
    return torch


def _salience_weights(salience, K, g):
    """ref/layer_fixed.py:943-978 -> float64 [K] (None when unweighted)."""
    if salience is None:
        return None
    s = np.asarray(salience, dtype=np.float64).reshape(-1)
    if s.shape[0] != K:
        raise ValueError(f"salience has {s.shape[0]} entries but the matrix has K={K} input channels")
    if not np.all(np.isfinite(s)) or np.any(s < 0.0):
        raise ValueError("salience must be finite and non-negative (it is a mean |activation| per input channel)")
    w = s * s
    mean = float(w.mean())
    if not mean > 0.0:
        raise ValueError("salience is identically zero -- no input channel carries signal")
    return w / mean


def _device_matrix(W):
    """(device tensor, is_f64, N, K): float32 stays float32 (exact in the
    reference's float64), anything else goes up as float64."""
    torch = _torch()
    if isinstance(W, torch.Tensor):
        t = W.detach()
        if t.dtype not in (torch.float32, torch.float64):
            t = t.to(torch.float64)
        t = t.cuda().contiguous()
    else:
        a = np.asarray(W)
        if a.dtype != np.float32:
            a = a.astype(np.float64)
        t = torch.from_numpy(np.ascontiguousarray(a)).cuda()
    if t.dim() != 2:
        raise ValueError(f"weight matrix must be 2-D, got shape {tuple(t.shape)}")
    N, K = int(t.shape[0]), int(t.shape[1])
    return t, int(t.dtype == torch.float64), N, K


def _scales(t, f64, N, K, g, alpha, sal):
    """Every group's scale (device float64 [N, K/g]) and their maximum."""
    torch = _torch()
    from .ops import ptr, stream_ptr
    best = torch.empty((N, K // g), dtype=torch.float64, device="cuda")
    smax = torch.zeros(1, dtype=torch.int64, device="cuda")
    al = np.ascontiguousarray(alpha if alpha is not None else np.zeros(0), dtype=np.float64)
    d_sal = torch.from_numpy(np.ascontiguousarray(sal, dtype=np.float64)).cuda() if sal is not None else None
    L.check(L.lib().f5_quant_w4_scales(ptr(t), f64, N, K, g,
                                       al.ctypes.data_as(ctypes.c_void_p) if al.size else None,
                                       int(al.size), ptr(d_sal), ptr(best), ptr(smax), stream_ptr()),
            "f5_quant_w4_scales")
    mx = np.array([int(smax.item())], dtype=np.int64).view(np.float64)[0]
    return best, float(mx)


def _shared_exponent(smax):
    """ref/w4a8_ref.py:171 (host numpy, like the reference)."""
    return int(np.ceil(np.log2(np.float64(smax)))) + 1


def _pack(t, f64, N, K, g, best, e, arrays=True):
    torch = _torch()
    from .ops import ptr, stream_ptr
    img = torch.empty(N * row_stride(K, g), dtype=torch.uint8, device="cuda")
    w4 = torch.empty((N, K), dtype=torch.int8, device="cuda") if arrays else None
    m = torch.empty((N, K // g), dtype=torch.int16, device="cuda") if arrays else None
    L.check(L.lib().f5_quant_w4_pack(ptr(t), f64, N, K, g, ptr(best), int(e), ptr(img), ptr(w4), ptr(m),
                                     stream_ptr()), "f5_quant_w4_pack")
    return img, w4, m


def _check_g(K, g):
    if g != G:
        raise NotImplementedError(f"group size {g}: this build quantizes the g = 128 wire format only")
    assert K % g == 0, f"K={K} not divisible by group size {g}"


def _mse(Wf, nalpha, amin, g, salience, arrays):
    t, f64, N, K = _device_matrix(Wf)
    _check_g(K, g)
    sal = _salience_weights(salience, K, g)
    best, smax = _scales(t, f64, N, K, g, np.linspace(amin, 1.0, nalpha), sal)
    e = _shared_exponent(smax)
    img, w4, m = _pack(t, f64, N, K, g, best, e, arrays)
    return img, w4, m, e, N, K


def quant_linear_mse(Wf, nalpha=17, amin=0.55, g=G, salience=None):
    """ref/layer_fixed.py:981-1030: MSE-optimal group scales, on the GPU."""
    _, w4, m, e, N, K = _mse(Wf, nalpha, amin, g, salience, True)
    return {"w4": w4.cpu().numpy(), "m": m.cpu().numpy().view(np.uint16), "e": e, "g": int(g),
            "sh": final_shift(K, g)}


def quantize_weights(W, g=G):
    """ref/w4a8_ref.py:154-180: the max|W_g|/7 rule -> (w4, m, e, sh)."""
    t, f64, N, K = _device_matrix(W)
    _check_g(K, g)
    best, smax = _scales(t, f64, N, K, g, None, None)
    e = _shared_exponent(smax)
    _, w4, m = _pack(t, f64, N, K, g, best, e)
    return w4.cpu().numpy(), m.cpu().numpy().view(np.uint16), e, final_shift(K, g)


def quant_linear(Wf, tighten_e=False, mse_scale=True, g=G, salience=None, hess=None):
    """ref/layer_fixed.py:1033-1111 (W4 paths)."""
    if hess is not None:
        if salience is not None:
            raise SystemExit("GPTQ takes its scale-search weights from the Hessian diagonal; passing "
                             "`salience` as well would silently weight it twice")
        if not mse_scale or tighten_e:
            raise SystemExit("GPTQ is only defined on the MSE group-scale rule (mse_scale=True, tighten_e=False)")
        raise NotImplementedError("the GPTQ error-feedback quantizer (ref/gptq.py) is not part of this build")
    if mse_scale:
        assert not tighten_e, "tighten_e is only implemented for the max-rule quantizer (see quant_linear_mse)"
        return quant_linear_mse(Wf, g=g, salience=salience)
    if salience is not None:
        raise SystemExit("salience weighting is only defined for the MSE group-scale rule (mse_scale=True); "
                         "the historical max|W_g|/7 rule has no scale search to weight")
    t, f64, N, K = _device_matrix(Wf)
    _check_g(K, g)
    best, smax = _scales(t, f64, N, K, g, None, None)
    e = _shared_exponent(smax)
    if tighten_e:
        # ref/layer_fixed.py:1100-1110: lower e while max(m) still fits uint16
        d = 0
        while d < 15 and np.round(np.float64(smax) * np.exp2(15 - (e - d - 1))) <= 65535:
            d += 1
        e -= d
    _, w4, m = _pack(t, f64, N, K, g, best, e)
    return {"w4": w4.cpu().numpy(), "m": m.cpu().numpy().view(np.uint16), "e": int(e), "sh": final_shift(K, g),
            "g": int(g)}


def quant_linear_image(Wf, mse_scale=True, g=G, salience=None):
    """(packed row image as a device uint8 tensor [N * stride], N, K, e, sh):
    quant_linear's result in the resident row format, never unpacked."""
    if mse_scale:
        img, _, _, e, N, K = _mse(Wf, 17, 0.55, g, salience, False)
        return img, N, K, e, final_shift(K, g)
    t, f64, N, K = _device_matrix(Wf)
    _check_g(K, g)
    best, smax = _scales(t, f64, N, K, g, None, None)
    e = _shared_exponent(smax)
    img, _, _ = _pack(t, f64, N, K, g, best, e, arrays=False)
    return img, N, K, e, final_shift(K, g)


# ---- layers (ref/layer_fixed.py:1354-1651) ----
def _refuse(w8, layer_idx=None):
    if w8:
        raise NotImplementedError("the W8 weight format is not part of the W4A8 decode path")
    if os.environ.get("FABLE5_CALIB_STATS"):
        raise NotImplementedError("calibrated quantization (FABLE5_CALIB_STATS) is not part of this build")


def res_scaled(W, s):
    """ref/layer_fixed.py:1354-1357: W * s in float64 (s a power of two)."""
    W = np.asarray(W, dtype=np.float64)
    return W if s == 1.0 else W * np.float64(s)


def _q14(v):
    return np.round(np.asarray(v) * (1 << 14)).astype(I64)


def quant_attn(wf, res_scale=1.0, tighten_e=False, mse_scale=True, g=G, layer_idx=None, w8=False):
    """ref/layer_fixed.py:1360-1376."""
    _refuse(w8, layer_idx)

    def q(W):
        return quant_linear(W, tighten_e, mse_scale, g)
    return {
        "q_proj": q(wf["q_proj"]),
        "k_proj": q(wf["k_proj"]),
        "v_proj": q(wf["v_proj"]),
        "o_proj": q(res_scaled(wf["o_proj"], res_scale) if res_scale != 1.0 else wf["o_proj"]),
        "q_norm": _q14(wf["q_norm"]),
        "k_norm": _q14(wf["k_norm"]),
    }


def quant_deltanet(wf, res_scale=1.0, tighten_e=False, mse_scale=True, g=G, layer_idx=None, w8=False):
    """ref/layer_fixed.py:1455-1494."""
    _refuse(w8, layer_idx)
    dt_spec = np.round(np.asarray(wf["dt_bias"]) * (1 << 12)).astype(I64)
    A_spec = np.round(np.exp(wf["A_log"]) * (1 << 15)).astype(I64)
    dt_q = np.clip(dt_spec, DT_Q12_MIN, DT_Q12_MAX)
    A_q = np.clip(A_spec, 0, A_Q15_MAX)

    def q(W):
        return quant_linear(W, tighten_e, mse_scale, g)
    qd = {
        "in_qkv": q(wf["in_qkv"]),
        "in_z": q(wf["in_z"]),
        "in_b": q(wf["in_b"]),
        "in_a": q(wf["in_a"]),
        "out": q(res_scaled(wf["out"], res_scale) if res_scale != 1.0 else wf["out"]),
        "conv_w": np.round(np.asarray(wf["conv_w"]) * (1 << CW_F)).astype(I64),
        "dt_bias_q12": dt_q,
        "negA_q15": A_q,
        "norm_w_q14": _q14(wf["norm_w"]),
    }
    qd["A_q15"] = A_q
    qd["gate_sat"] = [(int(h), int(dt_spec[h]), int(dt_q[h]), int(A_spec[h]), int(A_q[h]))
                      for h in range(len(dt_q)) if dt_spec[h] != dt_q[h] or A_spec[h] != A_q[h]]
    return qd


def quant_mlp(wf, res_scale=1.0, tighten_e=False, mse_scale=True, g=G, layer_idx=None, w8=False):
    """ref/layer_fixed.py:1586-1594."""
    _refuse(w8, layer_idx)
    q = {k: quant_linear(wf[k], tighten_e, mse_scale, g) for k in ("gate", "up")}
    q["down"] = quant_linear(res_scaled(wf["down"], res_scale) if res_scale != 1.0 else wf["down"],
                             tighten_e, mse_scale, g)
    return q


def layer_vectors(wf):
    """The integer vectors of quant_layer (ref/layer_fixed.py:1369-1370,
    1460-1493, 1640-1641) without quantizing any matrix: {"ln1", "ln2",
    "type", and "attn": {"q_norm", "k_norm"} or "dn": {"conv_w",
    "dt_bias_q12", "A_q15", "negA_q15", "norm_w_q14", "gate_sat"}}."""
    out = {"ln1": _q14(wf["ln1"]), "ln2": _q14(wf["ln2"]), "type": wf["type"]}
    if wf["type"] == "full_attention":
        a = wf["attn"]
        out["attn"] = {"q_norm": _q14(a["q_norm"]), "k_norm": _q14(a["k_norm"])}
    else:
        d = wf["dn"]
        dt_spec = np.round(np.asarray(d["dt_bias"]) * (1 << 12)).astype(I64)
        A_spec = np.round(np.exp(d["A_log"]) * (1 << 15)).astype(I64)
        dt_q = np.clip(dt_spec, DT_Q12_MIN, DT_Q12_MAX)
        A_q = np.clip(A_spec, 0, A_Q15_MAX)
        out["dn"] = {"conv_w": np.round(np.asarray(d["conv_w"]) * (1 << CW_F)).astype(I64),
                     "dt_bias_q12": dt_q, "negA_q15": A_q, "norm_w_q14": _q14(d["norm_w"]), "A_q15": A_q,
                     "gate_sat": [(int(h), int(dt_spec[h]), int(dt_q[h]), int(A_spec[h]), int(A_q[h]))
                                  for h in range(len(dt_q)) if dt_spec[h] != dt_q[h] or A_spec[h] != A_q[h]]}
    return out


def quant_layer(wf, res_scale=1.0, tighten_e=False, mse_scale=True, g=G, layer_idx=None, w8=False):
    """ref/layer_fixed.py:1607-1651."""
    _refuse(w8, layer_idx)
    qw = {"ln1": _q14(wf["ln1"]), "ln2": _q14(wf["ln2"]),
          "mlp": quant_mlp(wf["mlp"], res_scale, tighten_e, mse_scale, g, layer_idx, w8),
          "type": wf["type"]}
    if wf["type"] == "full_attention":
        qw["attn"] = quant_attn(wf["attn"], res_scale, tighten_e, mse_scale, g, layer_idx, w8)
    else:
        qw["dn"] = quant_deltanet(wf["dn"], res_scale, tighten_e, mse_scale, g, layer_idx, w8)
    return qw

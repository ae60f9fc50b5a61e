"""Device-level wrappers over the C ABI (torch tensors as device buffers).

PyTorch is only plumbing here: it allocates device memory and provides the
current CUDA stream; every computation is a kernel of libf5b200.so.
"""
from __future__ import annotations

import ctypes

import numpy as np
import torch

from . import _lib as L

I64 = np.int64


def stream_ptr():
    return ctypes.c_void_p(torch.cuda.current_stream().cuda_stream)


def ptr(t):
    return None if t is None else ctypes.c_void_p(t.data_ptr())


def to_dev(a, dtype=None):
    a = np.ascontiguousarray(a if dtype is None else np.asarray(a, dtype=dtype))
    return torch.from_numpy(a).cuda()


def seg(w, out, rows, mode, e=0, out_f=0, w2=None, e2=0, out_f2=0, p_out=None, out_row0=0):
    s = L.GemvSeg()
    s.w = w.data_ptr()
    s.w2 = w2.data_ptr() if w2 is not None else None
    s.out = out.data_ptr() if out is not None else None
    s.p_out = p_out.data_ptr() if p_out is not None else None
    s.rows, s.e, s.e2, s.out_f, s.out_f2 = rows, e, e2, out_f, out_f2
    s.mode, s.out_row0 = mode, out_row0
    return s


def gemv(segs, K, g, sh, x8, xmeta=None, argmax=None, err=None, max_blocks=0, pdl=False):
    """Launch a fused GEMV on the current stream (no sync)."""
    arr = (L.GemvSeg * len(segs))(*segs)
    if err is None:
        err = torch.zeros(1, dtype=torch.int32, device="cuda")
    L.check(L.lib().f5_gemv_dev(arr, len(segs), K, g, sh, ptr(x8), ptr(xmeta), ptr(argmax),
                                ptr(err), max_blocks, int(pdl), stream_ptr()), "f5_gemv_dev")
    return err


def prim(op, x, arg0=0, in2=None, want2=False):
    """Evaluate an integer primitive element-wise on the GPU -> numpy."""
    x = np.ascontiguousarray(np.asarray(x, dtype=I64).reshape(-1))
    dx = to_dev(x)
    d2 = to_dev(np.asarray(in2, dtype=I64).reshape(-1)) if in2 is not None else None
    out = torch.empty_like(dx)
    out2 = torch.empty_like(dx) if want2 else None
    L.check(L.lib().f5_prim_dev(op, ptr(dx), ptr(d2), ptr(out), ptr(out2), x.size, arg0, 0,
                                stream_ptr()), "f5_prim_dev")
    torch.cuda.synchronize()
    r = out.cpu().numpy()
    return (r, out2.cpu().numpy()) if want2 else r


def rmsnorm_dynq8(x16_dev, w_dev, n, in_f, one_plus, want_xn=True):
    xn = torch.empty(n, dtype=torch.int16, device="cuda") if want_xn else None
    x8 = torch.empty(n, dtype=torch.int8, device="cuda")
    meta = torch.zeros(2, dtype=torch.int32, device="cuda")
    L.check(L.lib().f5_rmsnorm_dynq8_dev(ptr(x16_dev), ptr(w_dev), n, in_f, int(one_plus), ptr(xn),
                                         ptr(x8), ptr(meta), stream_ptr()), "f5_rmsnorm_dynq8_dev")
    return xn, x8, meta


def dynq8(x16_dev, n, in_f):
    x8 = torch.empty(n, dtype=torch.int8, device="cuda")
    meta = torch.zeros(2, dtype=torch.int32, device="cuda")
    L.check(L.lib().f5_dynq8_dev(ptr(x16_dev), n, in_f, ptr(x8), ptr(meta), stream_ptr()), "f5_dynq8_dev")
    return x8, meta


def synth_w4(d_img, nrows, K, g, row0, key_w, key_m, symmetric):
    L.check(L.lib().f5_synth_w4_dev(ptr(d_img), nrows, K, g, row0, key_w, key_m, int(symmetric),
                                    stream_ptr()), "f5_synth_w4_dev")


def synth_emb(d_emb, nrows, H, row0, key_e):
    L.check(L.lib().f5_synth_emb_dev(ptr(d_emb), nrows, H, row0, key_e, stream_ptr()), "f5_synth_emb_dev")


def matvec_y32_host(img, N, K, g, sh, x8, want_p=False):
    img = np.ascontiguousarray(img, dtype=np.uint8)
    x8 = np.ascontiguousarray(x8, dtype=np.int8)
    y = np.empty(N, dtype=np.int32)
    p = np.empty(N, dtype=I64) if want_p else None
    rc = L.lib().f5_matvec_y32_host(img.ctypes.data, N, K, g, sh, x8.ctypes.data, y.ctypes.data,
                                    p.ctypes.data if p is not None else None)
    if rc == L.F5_EOVERFLOW:
        raise AssertionError("y32 overflow -- sh miscomputed")
    L.check(rc, "f5_matvec_y32_host")
    return (y, p) if want_p else y


def batch_matvec_y32(d_img, N, K, sh, d_x8, want_p=False):
    """Batched matvec_y32 on the tensor cores: d_x8 [B][K] int8 (device),
    d_img the packed image (device, 256-byte aligned) -> (y32 [B][N], err
    word[, p [B][N]]) as device tensors, launched on the current stream."""
    B = int(d_x8.shape[0])
    ws_bytes = L.lib().f5_batch_matvec_ws_bytes(N, K, B)
    if not ws_bytes:
        raise ValueError(f"batched matvec: unsupported shape N={N} K={K} B={B}")
    ws = torch.empty(ws_bytes + 256, dtype=torch.uint8, device="cuda")
    off = (-ws.data_ptr()) % 256
    y = torch.empty((B, N), dtype=torch.int32, device="cuda")
    p = torch.empty((B, N), dtype=torch.int64, device="cuda") if want_p else None
    err = torch.zeros(1, dtype=torch.int32, device="cuda")
    L.check(L.lib().f5_batch_matvec_y32_dev(ptr(d_img), N, K, 128, sh, ptr(d_x8), B, ptr(y), ptr(p),
                                            ctypes.c_void_p(ws.data_ptr() + off), ws_bytes, ptr(err),
                                            stream_ptr()), "f5_batch_matvec_y32_dev")
    return (y, err, p) if want_p else (y, err)

"""Drop-in for the seq_model matvec engine, ``DDRWeights``
(ref/seq_model.py:305-452), on the GPU.

The reference's SEQ-stream executor (``SeqExec``, ref/seq_model.py:610-1145)
runs every MVGO record through ``DDRWeights.matvec(wbase, nrows, sh, ng, g,
x8)``: the record's WBASE selects a weight image (wid) and a first row,
``nrows`` rows of that image are multiplied with the int8 window ``x8`` by
``matvec_y32`` (ref/w4a8_ref.py:254-289), and the int64 y32 vector comes back.
This class keeps the same constructor, class methods and ``matvec``
signature and answers from the GPU: every image is uploaded once into device
memory in its packed row format, and each call runs ``f5_gemv_dev`` over the
requested row range.

Plan (the ``"weights"`` entry of a stream's ``.seq.json``): ``{wid: {base,
nrows, k, ng, sh, g, stride, nbeats[, w8]}}``.  As in the reference, a WBASE
resolves to the plan entry with the largest base not above it and must be
row-aligned inside that image, the call's shape words must equal the
plan's, and ``x8`` must hold K bytes.  W8 images (``"w8": true``) and the
per-channel repacked layout (``meta["weight_repack"]``) are refused with
``NotImplementedError``: this build streams W4 rows on one GPU.
"""
from __future__ import annotations

import json
import os

import numpy as np

from .w4a8_ref import pack_ddr_rows, row_stride

I64 = np.int64


class DDRWeights(object):
    """WBASE -> rows of a packed W4 image, multiplied on the GPU."""

    def __init__(self, plan, meta=None):
        self.plan = {int(k): dict(v) for k, v in plan.items()}
        self.meta = meta or {}
        if any(isinstance(p["base"], (list, tuple)) for p in self.plan.values()) or self.meta.get("weight_repack"):
            raise NotImplementedError("per-channel repacked weight plans are not supported (single-GPU W4 rows)")
        if any(p.get("w8", False) for p in self.plan.values()):
            raise NotImplementedError("W8 weight images are not part of the W4A8 decode path")
        for wid, p in self.plan.items():
            if int(p["stride"]) != row_stride(int(p["k"]), int(p.get("g", 128))):
                raise ValueError(f"wid {wid}: stride {p['stride']} is not the W4 row stride of k={p['k']}")
        self.byaddr = sorted((int(p["base"]), int(w)) for w, p in self.plan.items())
        self._dev = {}       # wid -> device image (torch uint8 [nrows * stride])

    # ---- construction (ref/seq_model.py:366-400) ----
    @classmethod
    def from_files(cls, prefix, plan, meta=None):
        """Images from ``<prefix>.weights.json`` and its ``_w<wid>.bin`` files."""
        self = cls(plan, meta)
        d = os.path.dirname(os.path.abspath(prefix)) or "."
        man = json.load(open(prefix + ".weights.json"))
        for wid, m in man.items():
            if not wid.isdigit() or int(wid) not in self.plan:
                continue
            p = self.plan[int(wid)]
            path = os.path.join(d, m["file"])
            want = int(p["nrows"]) * int(p["stride"])
            got = os.path.getsize(path)
            if got != want:
                raise ValueError(f"wid {wid}: {m['file']} is {got} B, the plan's "
                                 f"{p['nrows']} x {p['stride']} B image is {want} B")
            self._upload(int(wid), np.fromfile(path, dtype=np.uint8))
        return self

    @classmethod
    def from_wids(cls, wids, plan, meta=None):
        """Images from live quantized matrices: ``{key: (wid, {"w4", "m", ...})}``."""
        self = cls(plan, meta)
        for (wid, qw) in wids.values():
            img, _ = pack_ddr_rows(qw["w4"], qw["m"], qw.get("g", 128))
            self._upload(int(wid), np.frombuffer(img, dtype=np.uint8))
        return self

    @classmethod
    def from_images(cls, images, plan, meta=None):
        """Images given directly: ``{wid: uint8 array}`` (host) or device tensors."""
        self = cls(plan, meta)
        for wid, img in images.items():
            self._upload(int(wid), img)
        return self

    def _upload(self, wid, img):
        import torch
        p = self.plan[wid]
        n = int(p["nrows"]) * int(p["stride"])
        if isinstance(img, torch.Tensor):
            t = img.reshape(-1)
            if t.device.type != "cuda" or t.dtype != torch.uint8 or t.numel() != n:
                raise ValueError(f"wid {wid}: a device image must be uint8 cuda [{n}]")
        else:
            a = np.ascontiguousarray(np.asarray(img, dtype=np.uint8).reshape(-1))
            if a.size != n:
                raise ValueError(f"wid {wid}: image holds {a.size} B, expected {n}")
            t = torch.from_numpy(a).cuda()
        self._dev[wid] = t

    # ---- lookup (ref/seq_model.py:402-436) ----
    def _lookup(self, wbase, chan=None):
        """(wid, first row, plan entry, rows left in the image)."""
        wbase = int(wbase)
        wid = None
        lo, hi = 0, len(self.byaddr) - 1
        while lo <= hi:
            mid = (lo + hi) // 2
            if self.byaddr[mid][0] <= wbase:
                wid = self.byaddr[mid][1]
                lo = mid + 1
            else:
                hi = mid - 1
        if wid is None:
            raise AssertionError(f"WBASE {wbase:#x} below the weight region")
        p = self.plan[wid]
        off = wbase - int(p["base"])
        if not (0 <= off < int(p["nrows"]) * int(p["stride"])):
            raise AssertionError(f"WBASE {wbase:#x} does not land inside wid {wid}")
        if off % int(p["stride"]):
            raise AssertionError(f"WBASE {wbase:#x} is not row-aligned in wid {wid}")
        r0 = off // int(p["stride"])
        return wid, r0, p, int(p["nrows"]) - r0

    # ---- the engine (ref/seq_model.py:438-452) ----
    def matvec(self, wbase, nrows, sh, ng, g, x8, w8=False, chan=None):
        """int64 y32 [nrows] of rows [r0, r0 + nrows) of the image at WBASE."""
        import torch

        from . import _lib as L
        from . import ops
        if w8:
            raise NotImplementedError("W8 rows are not part of the W4A8 decode path")
        wid, r0, p, avail = self._lookup(wbase, chan)
        if nrows > avail:
            raise AssertionError("MVGO row chunk overruns the image")
        if sh != p["sh"] or g != p.get("g", 128) or ng != p["ng"]:
            raise AssertionError(f"wid {wid}: SHAPE (sh={sh} ng={ng} g={g}) != manifest "
                                 f"(sh={p['sh']} ng={p['ng']} g={p.get('g', 128)})")
        K = int(p["k"])
        x8 = np.asarray(x8, dtype=np.int8).reshape(-1)
        if x8.size != K:
            raise AssertionError(f"XWIN holds {x8.size} bytes, K={K}")
        if wid not in self._dev:
            raise KeyError(f"wid {wid}: no image loaded")
        stride = int(p["stride"])
        w = self._dev[wid][r0 * stride:(r0 + nrows) * stride]
        y = torch.empty(nrows, dtype=torch.int32, device="cuda")
        err = torch.zeros(1, dtype=torch.int32, device="cuda")
        s = ops.seg(w, y, nrows, L.GM_Y32)
        ops.gemv([s], K, int(g), int(sh), ops.to_dev(x8), err=err)
        torch.cuda.synchronize()
        if int(err.item()) & 1:
            raise AssertionError("y32 overflow -- sh miscomputed (ref/w4a8_ref.py:288)")
        return y.cpu().numpy().astype(I64)

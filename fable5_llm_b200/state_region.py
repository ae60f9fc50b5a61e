"""The reference's DDR state-region image: every layer's decode state in one
flat byte image (``<prefix>.state.bin``, planned by the ``state`` entry of
``<prefix>.weights.json``), read and written here so a reference artifact's
state loads into a ``DecodeModel`` and a GPU run's state can be compared with
the reference executor's byte for byte.

Layout (SEQ_ISA v2.1 B15.1 as written by ref/gen_layer_script.py:1672-1751
and read by ref/seq_model.py:149-302; the sizes are sw/hwmap.py:621-628).
The image covers [plan["dn"], plan["end"]) and holds three regions:
  * dn: one 1 MiB block per DeltaNet layer index d (the d-th DeltaNet layer
    of the stack): S as little-endian int16 [LNH=32][LDK=128][LDV=128];
  * kv: one 2 MiB block per (attention layer index a, kv head h, K|V) at
    block number (a * 4 + h) * 2 + (0 for K, 1 for V): T rows of HD = 256
    int8 codes from offset 0, and T int8 exponents from offset 1 MiB;
  * cv: one 128 KiB block per DeltaNet layer index d: CONV_DIM = 8192 rows
    of 16 bytes -- the 4 conv taps (int16 Q13), then the 3-sample conv
    window (int16, oldest first), then 2 zero bytes.
Blocks a model does not use stay zero.  T (the tokens in the KV cache) is
not in the image; the caller supplies it.
"""
from __future__ import annotations

import hashlib

import numpy as np

DN_LAYER = 1 << 20
KV_STRIDE = 1 << 21
KV_EXP_OFF = 1 << 20
CV_STRIDE = 1 << 17
N_DN, N_KV_LAYERS = 24, 8
T_MAX = 4096
LNH, LDK, LDV, CONV_DIM, NKV, HD = 32, 128, 128, 8192, 4, 256


def slots(layer_types):
    """[(layer type, dn index, kv index)]: a layer's index among the layers
    of its own kind (the slot rule of ref/gen_token_script.py:102-137)."""
    out, d, a = [], 0, 0
    for lt in layer_types:
        if lt == "full_attention":
            out.append((lt, None, a))
            a += 1
        else:
            out.append((lt, d, None))
            d += 1
    return out


class StateRegion(object):
    def __init__(self, plan, data=None):
        self.plan = {k: int(plan[k]) for k in ("dn", "kv", "cv", "end")}
        n = self.plan["end"] - self.plan["dn"]
        if data is None:
            self.mem = np.zeros(n, dtype=np.uint8)
        else:
            self.mem = np.frombuffer(bytearray(data), dtype=np.uint8)
            if self.mem.size != n:
                raise ValueError(f"state image is {self.mem.size} B, the plan spans {n} B")

    @classmethod
    def load(cls, prefix):
        """``<prefix>.state.bin`` under the plan of ``<prefix>.weights.json``."""
        import json
        plan = json.load(open(prefix + ".weights.json")).get("state")
        if plan is None:
            return None
        with open(prefix + ".state.bin", "rb") as f:
            return cls(plan, f.read())

    def sha256(self):
        return hashlib.sha256(self.mem.tobytes()).hexdigest()

    # ---- block addressing ----
    def _dn(self, d):
        if not 0 <= d < N_DN:
            raise ValueError(f"DN layer index {d} outside 0..{N_DN - 1}")
        o = self.plan["dn"] - self.plan["dn"] + d * DN_LAYER
        return self.mem[o:o + DN_LAYER]

    def _kv(self, a, h, v):
        if not (0 <= a < N_KV_LAYERS and 0 <= h < NKV):
            raise ValueError(f"KV block (layer {a}, head {h}) outside the region")
        o = self.plan["kv"] - self.plan["dn"] + ((a * 4 + h) * 2 + v) * KV_STRIDE
        return self.mem[o:o + KV_STRIDE]

    def _cv(self, d):
        if not 0 <= d < N_DN:
            raise ValueError(f"CV layer index {d} outside 0..{N_DN - 1}")
        o = self.plan["cv"] - self.plan["dn"] + d * CV_STRIDE
        return self.mem[o:o + CV_STRIDE].reshape(CONV_DIM, 16)

    # ---- typed views ----
    def dn_state(self, d):
        return self._dn(d).view("<i2").reshape(LNH, LDK, LDV).astype(np.int16)

    def conv(self, d):
        """(taps int64 [CONV_DIM, 4], window int64 [CONV_DIM, 3] oldest first)."""
        r = self._cv(d)
        return (r[:, 0:8].copy().view("<i2").astype(np.int64),
                r[:, 8:14].copy().view("<i2").astype(np.int64))

    def kv(self, a, T):
        """(k8 [T, NKV, HD] int8, ke [T, NKV] int8, v8, ve)."""
        if not 0 <= T <= T_MAX:
            raise ValueError(f"T={T} outside 0..{T_MAX}")
        out = []
        for v in (0, 1):
            rows = np.stack([self._kv(a, h, v)[:T * HD].view(np.int8).reshape(T, HD) for h in range(NKV)], axis=1)
            ex = np.stack([self._kv(a, h, v)[KV_EXP_OFF:KV_EXP_OFF + T].view(np.int8) for h in range(NKV)], axis=1)
            out += [rows, ex]
        return tuple(out)

    def put_dn_state(self, d, S):
        self._dn(d)[:] = np.ascontiguousarray(np.asarray(S).astype("<i2")).reshape(-1).view(np.uint8)

    def put_conv(self, d, taps, window):
        r = self._cv(d)
        r[:, 0:8] = np.ascontiguousarray(np.asarray(taps).astype("<i2")).view(np.uint8).reshape(CONV_DIM, 8)
        r[:, 8:14] = np.ascontiguousarray(np.asarray(window).astype("<i2")).view(np.uint8).reshape(CONV_DIM, 6)
        r[:, 14:16] = 0

    def put_kv(self, a, k8, ke, v8, ve):
        T = k8.shape[0]
        for v, (rows, ex) in enumerate(((k8, ke), (v8, ve))):
            for h in range(NKV):
                blk = self._kv(a, h, v)
                blk[:T * HD] = np.ascontiguousarray(rows[:, h]).reshape(-1).view(np.uint8)
                blk[KV_EXP_OFF:KV_EXP_OFF + T] = np.ascontiguousarray(ex[:, h]).view(np.uint8)

    # ---- a DecodeModel's state in and out ----
    def apply_to(self, model, T):
        """Load every layer's state of ``model`` from this image at T
        tokens; returns the conv taps per DeltaNet layer (they travel in the
        image, ref/gen_token_script.py:197-200)."""
        taps = {}
        for i, (lt, d, a) in enumerate(slots(model.geom.layer_types)):
            if lt == "full_attention":
                if T == 0:
                    continue          # an empty cache: nothing to load
                k8, ke, v8, ve = self.kv(a, T)
                model.load_state_image(i, np.concatenate([np.ascontiguousarray(x).reshape(-1).view(np.uint8)
                                                          for x in (k8, ke, v8, ve)]), T)
            else:
                tp, win = self.conv(d)
                taps[i] = tp
                model.set_dn_state(i, T, {"S": self.dn_state(d), "conv": win})
        return taps

    @classmethod
    def from_model(cls, plan, model, T, conv_taps):
        """The image of ``model``'s state at T tokens (``conv_taps``: the
        int taps [CONV_DIM, 4] of each DeltaNet layer, by layer index)."""
        self = cls(plan)
        for i, (lt, d, a) in enumerate(slots(model.geom.layer_types)):
            if lt == "full_attention":
                self.put_kv(a, *model._kv_arrays(i, T))
            else:
                st = model.get_dn_state(i, T)
                self.put_dn_state(d, st["S"])
                self.put_conv(d, conv_taps[i], st["conv"])
        return self

"""Batched decode: B independent greedy sequences over one resident model.

``BatchModel`` owns an ``f5_bctx`` (include/f5b200.h) that borrows the
weights of a loaded ``DecodeModel`` (kept alive here) and holds B
sequences' decode state.  Every projection of the step runs as a W4A8 GEMM
of the B quantized inputs on the tensor cores; per sequence the results are
those of the single-sequence step, bit for bit.
"""
from __future__ import annotations

import ctypes

import numpy as np

from . import _lib as L

I64 = np.int64


def _p(a):
    return ctypes.c_void_p(a.ctypes.data)


class BatchModel:
    def __init__(self, model, batch, max_T=None):
        self.model = model                      # the weights' owner must outlive the batch
        self.geom = model.geom
        self.B = int(batch)
        self.max_T = (int(max_T or model.max_T) + 15) & ~15
        self.lib = L.lib()
        h = ctypes.c_void_p()
        L.check(self.lib.f5_bctx_create(model.h, self.B, self.max_T, ctypes.byref(h)), "f5_bctx_create")
        self.h = h

    def close(self):
        if getattr(self, "h", None):
            self.lib.f5_bctx_destroy(self.h)
            self.h = None

    def __del__(self):
        try:
            self.close()
        except Exception:
            pass

    # ---- positions / state ----
    def reset(self):
        L.check(self.lib.f5_bctx_reset(self.h), "f5_bctx_reset")

    def set_position(self, T, pos, seq=-1):
        L.check(self.lib.f5_bctx_set_position(self.h, int(seq), int(T), int(pos)), "f5_bctx_set_position")

    def position(self, seq):
        T, pos = ctypes.c_int(), ctypes.c_int()
        L.check(self.lib.f5_bctx_get_position(self.h, int(seq), ctypes.byref(T), ctypes.byref(pos)),
                "f5_bctx_get_position")
        return T.value, pos.value

    # ---- steps ----
    def step(self, tokens):
        """One step of every sequence -> (next tokens int32[B], their y32)."""
        tok = np.ascontiguousarray(np.asarray(tokens, dtype=np.int32).reshape(self.B))
        nt = np.empty(self.B, dtype=np.int32)
        mv = np.empty(self.B, dtype=np.int32)
        L.check(self.lib.f5_bctx_step(self.h, _p(tok), _p(nt), _p(mv)), "f5_bctx_step")
        return nt, mv

    def prefill(self, seq, tokens):
        """Ingest a prompt into sequence seq layer-major (f5_bctx_prefill)
        -> (the argmax after its last token, that token's y32 logit); the
        state equals len(tokens) decode steps' and the next step of seq is
        fed that argmax."""
        tok = np.ascontiguousarray(np.asarray(tokens, dtype=np.int32).reshape(-1))
        nt, mv = ctypes.c_int32(), ctypes.c_int32()
        L.check(self.lib.f5_bctx_prefill(self.h, int(seq), _p(tok), int(tok.size), ctypes.byref(nt),
                                         ctypes.byref(mv)), "f5_bctx_prefill")
        return int(nt.value), int(mv.value)

    def launch(self, n):
        """Enqueue n greedy steps (each sequence fed its own argmax)."""
        L.check(self.lib.f5_bctx_launch(self.h, int(n)), "f5_bctx_launch")

    def sync(self):
        nt = np.empty(self.B, dtype=np.int32)
        mv = np.empty(self.B, dtype=np.int32)
        L.check(self.lib.f5_bctx_sync(self.h, _p(nt), _p(mv)), "f5_bctx_sync")
        return nt, mv

    def time_step(self, reps=2):
        """Per-kernel-class device time of one eager batched step (CUDA
        events around every launch); advances every sequence reps steps."""
        out = np.zeros(14, dtype=np.float64)
        L.check(self.lib.f5_bctx_time_step(self.h, int(reps), _p(out), 14), "f5_bctx_time_step")
        kinds = ("prep", "gemm", "epi", "dn", "attn", "other")
        r = {f"{k}_ms": float(out[i]) for i, k in enumerate(kinds)}
        r["gemm_bytes"] = float(out[7])
        r["launches"] = int(out[12])
        r["sum_ms"] = float(out[13])
        return r

    def stream_handle(self):
        sp = ctypes.c_void_p()
        L.check(self.lib.f5_bctx_stream(self.h, ctypes.byref(sp)), "f5_bctx_stream")
        return sp.value

    # ---- TOPK-32 capture and per-sequence sampling (sw/chat_seq.py:1776-1928) ----
    def set_logits(self, on=True):
        """Store the LM head's y32 logits of every sequence each step."""
        L.check(self.lib.f5_bctx_set_logits(self.h, int(on)), "f5_bctx_set_logits")

    def logits(self, seq):
        return self.read(seq, L.BUF_LOGITS)

    def topk(self):
        """The last step's TOPK-32 capture of every sequence (needs
        set_logits(True) before the step) -> list of sampling.TopK32Result."""
        from .sampling import TopK32Result
        res = (L.TopK32 * self.B)()
        L.check(self.lib.f5_bctx_topk(self.h, ctypes.byref(res)), "f5_bctx_topk")
        return [TopK32Result.from_struct(r) for r in res]

    def sample_step(self, tokens, samplers):
        """One step of every sequence whose next tokens are drawn by
        samplers[b] (sampling.Sampler) from that sequence's capture list
        -> (tokens int32[B], per-sequence info)."""
        self.step(tokens)
        picks = [s.pick(r.values, r.indices, r.e_x) for s, r in zip(samplers, self.topk())]
        return np.array([t for t, _ in picks], dtype=np.int32), [i for _, i in picks]

    # ---- buffers of one sequence ----
    def _size(self, what):
        g = self.geom
        return {L.BUF_X16: (g.H, np.int16), L.BUF_ON16: (g.LVD, np.int16), L.BUF_QKV16: (g.CONV_DIM, np.int16),
                L.BUF_Z16: (g.LVD, np.int16), L.BUF_B16: (g.LNH, np.int16), L.BUF_A16: (g.LNH, np.int16),
                L.BUF_K16: (g.NKV * g.HD, np.int16), L.BUF_V16: (g.NKV * g.HD, np.int16),
                L.BUF_PROD64: (g.NQ * g.HD, I64), L.BUF_QKVC16: (g.CONV_DIM, np.int16),
                L.BUF_GATES: (2 * g.LNH, np.int32), L.BUF_QG16: (g.NQ * g.HD * 2, np.int16),
                L.BUF_PROD16: (g.FFN, np.int16), L.BUF_DN_S: (g.LNH * g.LDK * g.LDV, np.int16),
                L.BUF_DN_CONV: (g.CONV_DIM * 4, np.int16), L.BUF_DN_KH: (g.LNH, np.int32),
                L.BUF_K8: (g.NKV * self.max_T * g.HD, np.int8), L.BUF_KE: (g.NKV * self.max_T, np.int8),
                L.BUF_V8: (g.NKV * self.max_T * g.HD, np.int8), L.BUF_VE: (g.NKV * self.max_T, np.int8),
                L.BUF_KA: (1, np.int32), L.BUF_LOGITS: (g.vocab, np.int32)}[what]

    def read(self, seq, what, layer=0):
        n, dt = self._size(what)
        out = np.empty(n, dtype=dt)
        L.check(self.lib.f5_bctx_read(self.h, int(seq), what, int(layer), _p(out), out.nbytes), f"bctx read({what})")
        return out

    def write(self, seq, what, layer, arr):
        n, dt = self._size(what)
        a = np.ascontiguousarray(np.asarray(arr, dtype=dt).reshape(n))
        L.check(self.lib.f5_bctx_write(self.h, int(seq), what, int(layer), _p(a), a.nbytes), f"bctx write({what})")

    _STATE = {"D": (L.BUF_DN_S, L.BUF_DN_CONV), "A": (L.BUF_K8, L.BUF_KE, L.BUF_V8, L.BUF_VE)}

    def load_sequence_from(self, seq, model):
        """Copy a single-sequence model's whole decode state and position
        into sequence `seq` (same max_T)."""
        assert model.max_T == self.max_T
        for i, lt in enumerate(self.geom.layer_types):
            for buf in self._STATE["A" if lt == "full_attention" else "D"]:
                self.write(seq, buf, i, model.read(buf, i))
        T, pos = model.position()
        self.set_position(T, pos, seq)

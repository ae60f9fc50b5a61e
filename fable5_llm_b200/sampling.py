"""TOPK-32 capture and the seeded sampler that draws from it.

The reference samples on the host from the list its LM-head top-k unit
captures on the device (sw/chat_seq.py:1756-1775): candidates
``(values int32[k], indices int64[k], e_x)`` in the head's integer domain,
then ``Sampler.pick`` (sw/chat_seq.py:1776-1928) dequantises, applies
temperature, top-k and top-p and draws one token with a seeded
``np.random.default_rng``.  Here the capture unit is the CUDA kernel pair
``f5_topk32_dev`` / ``f5_ctx_topk`` (fable5_llm_b200/csrc/f5_topk.cu) and
``Sampler`` is the same host math over its 32 entries; greedy (temp 0)
returns entry 0, the LM head's argmax.
"""
from __future__ import annotations

import ctypes
import os
import time
from dataclasses import dataclass

import numpy as np

from . import _lib as L

DEFAULT_TOP_K = 50          # sw/chat_seq.py:293
DEFAULT_TOP_P = 1.0         # sw/chat_seq.py:294 (1.0 = off)
DEFAULT_TEMP = 0.0          # sw/chat_seq.py:295 (0.0 = greedy)
SEED_BITS = 63              # sw/chat_seq.py:296


class SamplingError(ValueError):
    """Invalid sampler settings or candidate sets (the reference raises
    ChatSeqError, a RuntimeError, for the same conditions)."""


@dataclass
class TopK32Result:
    values: np.ndarray      # int64[count], value descending, ties by ascending index
    indices: np.ndarray     # int64[count]
    ovf_lit: int
    ovf_disp: int
    amax_idx: int
    amax_val: int
    e_x: int
    n: int

    @property
    def count(self):
        return int(self.values.size)

    @classmethod
    def from_struct(cls, r):
        c = int(r.count)
        return cls(values=np.array(r.val[:c], dtype=np.int64), indices=np.array(r.idx[:c], dtype=np.int64),
                   ovf_lit=int(r.ovf_lit), ovf_disp=int(r.ovf_disp), amax_idx=int(r.amax_idx),
                   amax_val=int(r.amax_val), e_x=int(r.e_x), n=int(r.n))


def topk32(values) -> TopK32Result:
    """TOPK-32 of an int32 array on the GPU (host array in, element index =
    position); the semantics of the reference unit (tb/scripts/
    gen_topk_cases.py:20-45)."""
    v = np.ascontiguousarray(np.asarray(values, dtype=np.int32).reshape(-1))
    r = L.TopK32()
    L.check(L.lib().f5_topk32_host(v.ctypes.data_as(ctypes.c_void_p), v.size, ctypes.byref(r)),
            "f5_topk32_host")
    return TopK32Result.from_struct(r)


def topk32_dev(d_values, n, d_ws, d_out, stream=None):
    """Device form: d_values int32[n], d_ws >= f5_topk32_ws_bytes(n) bytes,
    d_out one f5_topk32 (all device pointers as ints); enqueued on `stream`."""
    L.check(L.lib().f5_topk32_dev(d_values, n, d_ws, d_out, stream), "f5_topk32_dev")


def topk32_ws_bytes(n):
    return int(L.lib().f5_topk32_ws_bytes(int(n)))


class Sampler:
    """Temperature / top-k / top-p over a candidate set, seeded; the
    contract of sw/chat_seq.py:1776-1928.  temp == 0 is greedy and never
    draws from the generator; otherwise one ``rng.random()`` per pick
    (inverse-CDF draw), so the tokens are a pure function of the seed and
    the candidate sequence."""

    def __init__(self, temp=DEFAULT_TEMP, top_k=DEFAULT_TOP_K, top_p=DEFAULT_TOP_P, seed=None,
                 logit_exp0=-22):
        temp, top_p, top_k = float(temp), float(top_p), int(top_k)
        if temp < 0:
            raise SamplingError("temperature must be >= 0 (0 = greedy)")
        if temp > 100:
            raise SamplingError("temperature above 100 is rejected")
        if top_k < 0:
            raise SamplingError("top_k must be >= 0 (0 = no top-k cut)")
        if not 0.0 < top_p <= 1.0:
            raise SamplingError("top_p must be in (0, 1] (1.0 = off)")
        self.temp, self.top_k, self.top_p = temp, top_k, top_p
        self.logit_exp0 = int(logit_exp0)
        self.seed_given = seed is not None
        self.seed = int(seed) if seed is not None else int.from_bytes(os.urandom(8), "big") >> (64 - SEED_BITS)
        self.rng = np.random.default_rng(self.seed)
        self.n = 0
        self.n_sampled = 0

    @property
    def enabled(self):
        return self.temp > 0.0

    def reset(self):
        """Re-seed (a context reset restarts the draw sequence)."""
        self.rng = np.random.default_rng(self.seed)
        self.n = self.n_sampled = 0

    def logits(self, values, e_x):
        """Dequant: value * 2^(e_x + logit_exp0), float64 (monotone)."""
        return np.asarray(values, dtype=np.float64) * float(2.0 ** (int(e_x) + self.logit_exp0))

    def pick(self, values, indices, e_x):
        """-> (token id, info dict)."""
        t0 = time.perf_counter()
        v = np.asarray(values, dtype=np.int64)
        idx = np.asarray(indices, dtype=np.int64)
        if v.shape != idx.shape or v.ndim != 1 or v.size == 0:
            raise SamplingError("the candidate set must be two 1-D arrays of the same non-zero length")
        if np.unique(idx).size != idx.size:
            raise SamplingError("the candidate set repeats a token id")
        order = np.lexsort((idx, -v))          # value descending, index ascending
        v, idx = v[order], idx[order]
        info = {"n_cand": int(v.size), "e_x": int(e_x), "top_value": int(v[0]), "top_id": int(idx[0])}
        self.n += 1
        if not self.enabled:
            info.update(mode="greedy", rank=0, p=1.0, k_eff=1, nucleus=1,
                        sample_ms=(time.perf_counter() - t0) * 1e3)
            return int(idx[0]), info
        k = v.size if self.top_k <= 0 else min(self.top_k, v.size)
        info["k_eff"] = int(k)
        info["k_clamped"] = bool(self.top_k > v.size > 0)
        z = self.logits(v[:k], e_x) / self.temp
        z -= z.max()
        p = np.exp(z)
        p /= p.sum()
        n = k
        if self.top_p < 1.0:
            n = int(np.searchsorted(np.cumsum(p), self.top_p, side="left")) + 1
            n = max(1, min(n, k))
            p = p[:n] / p[:n].sum()
        info["nucleus"] = int(n)
        u = float(self.rng.random())
        j = min(int(np.searchsorted(np.cumsum(p), u, side="right")), n - 1)
        self.n_sampled += 1
        info.update(mode="sampled", rank=j, p=float(p[j]), u=u, value=int(v[j]), greedy_id=int(idx[0]),
                    sample_ms=(time.perf_counter() - t0) * 1e3)
        return int(idx[j]), info

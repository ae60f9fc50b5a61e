"""RoPE cos/sin tables, built on the host exactly as the reference builds
them (ref/layer_ref.py:84-90 rope_cos_sin: float64 angles, float32 cos/sin;
ref/layer_fixed.py:1333-1337 rope_tables_q15: round to Q15, clamp to
+-32767).  The device never evaluates a transcendental for RoPE: the graph
indexes this table by the step's position."""
from __future__ import annotations

import numpy as np

from .config import ROPE_F, Geometry


def rope_tables_q15(pos, geom=None):
    """(cos_q, sin_q) int64[ROT] for one position (same expressions, same
    array shapes as the reference, so numpy takes the same code path)."""
    g = geom or Geometry()
    rot = g.ROT
    inv = 1.0 / (g.THETA ** (np.arange(0, rot, 2, dtype=np.float64) / rot))
    f = pos * inv
    emb = np.concatenate([f, f])
    cos, sin = np.cos(emb).astype(np.float32), np.sin(emb).astype(np.float32)
    return (np.clip(np.round(cos * (1 << ROPE_F)), -32767, 32767).astype(np.int64),
            np.clip(np.round(sin * (1 << ROPE_F)), -32767, 32767).astype(np.int64))


def rope_table(npos, geom=None):
    """int16 [npos][128]: cos Q15 [64] | sin Q15 [64] for positions 0..npos-1."""
    g = geom or Geometry()
    out = np.zeros((npos, 128), dtype=np.int16)
    for p in range(npos):
        c, s = rope_tables_q15(p, g)
        out[p, :g.ROT] = c
        out[p, 64:64 + g.ROT] = s
    return out

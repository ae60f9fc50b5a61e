#!/usr/bin/env python3
"""Generate the weight-artifact fixtures with the UNMODIFIED reference writer.

Run where the reference checkout exists, with the environment variable
F5_REFERENCE set to its root directory; the GPU box never runs it.
It registers a few small seeded W4 matrices (g = 128 and g = 64, K = 256 ..
4096) on the reference's ``Mach`` and calls its ``dump_weights``
(ref/gen_layer_script.py:1555-1670) with ``emb_row_bytes`` and ``rs_f`` as
the 9B generator passes them (ref/gen_model_script.py:652-667), writes a
small embedding table the way that generator does (``emb_q.tofile``), and a
second artifact holding one W8 matrix (which the W4A8 loader must refuse).
The inputs are kept in ``artifact/inputs.npz`` so the tests can rebuild
every image.

    python tests/golden/gen_artifact_golden.py
"""
from __future__ import annotations

import io
import os
import sys

import numpy as np

REF = os.environ.get("F5_REFERENCE")
if not REF or not os.path.isdir(os.path.join(REF, "ref")):
    sys.exit("set F5_REFERENCE to the root of the reference checkout (the directory holding ref/)")
HERE = os.path.dirname(os.path.abspath(__file__))
OUT = os.path.join(HERE, "artifact")
os.environ["FABLE5_MODEL"] = "9b"
sys.dont_write_bytecode = True
sys.path.insert(0, os.path.join(REF, "ref"))

import gen_layer_script as GLS   # noqa: E402  (reference)

SEED = 2026
# (nrows, K, g, e, sh)
SHAPES = [(40, 256, 128, -3, 5), (24, 512, 64, 2, 6), (16, 4096, 128, -7, 9), (8, 12288, 128, 1, 11)]
EMB = (6, 64)   # vocab, H of the small embedding table


def main():
    os.makedirs(OUT, exist_ok=True)
    rng = np.random.default_rng(SEED)
    M = GLS.Mach(io.StringIO())
    arrays = {}
    for wid, (N, K, g, e, sh) in enumerate(SHAPES):
        w4 = rng.integers(-8, 8, (N, K)).astype(np.int8)
        m = rng.integers(1, 1 << 16, (N, K // g)).astype(np.int64)
        qw = {"w4": w4, "m": m, "e": e, "sh": sh}
        if g != 128:
            qw["g"] = g
        M.wids[id(qw)] = (wid, qw)
        arrays[f"w4_{wid}"] = w4
        arrays[f"m_{wid}"] = m.astype(np.uint16)
    n = M.dump_weights(os.path.join(OUT, "tiny"), emb_row_bytes=2 * EMB[1], rs_f=GLS.RS_F)
    assert n == len(SHAPES)
    emb_q = rng.integers(-32768, 32768, EMB).astype(np.int16)
    emb_q.tofile(os.path.join(OUT, "tiny.emb.bin"))
    arrays["emb"] = emb_q
    arrays["shapes"] = np.array(SHAPES, dtype=np.int64)

    M8 = GLS.Mach(io.StringIO())
    qw8 = {"w8": rng.integers(-127, 128, (8, 256)).astype(np.int8),
           "m": rng.integers(1, 1 << 16, (8, 2)).astype(np.int64), "e": 0, "sh": 7}
    M8.wids[id(qw8)] = (0, qw8)
    M8.dump_weights(os.path.join(OUT, "tiny8"), rs_f=GLS.RS_F)
    np.savez_compressed(os.path.join(OUT, "inputs.npz"), **arrays)
    print("wrote", sorted(os.listdir(OUT)))


if __name__ == "__main__":
    main()

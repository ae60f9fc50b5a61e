"""Oracle-side assembly of the seeded synthetic model (test infrastructure).

Builds the reference-layout model (per-layer dicts of ``QMat`` + integer
vector parameters, ref/layer_fixed.py:1607-1651) from the seeded generator
in ``fable5_llm_b200.synth`` so the oracle and the CUDA path consume the same
bytes.
"""
from __future__ import annotations

import numpy as np

from fable5_llm_b200 import synth
from .oracle import GEOM_9B, QMat

I64 = np.int64


class OracleModel:
    def __init__(self, seed, geom=GEOM_9B, images=None):
        self.seed = seed
        self.geom = geom
        self.specs = synth.matrix_specs(geom)
        vec, self.ln_f_q12 = synth.vector_params(seed, geom)
        self.layers = []
        qm = {}
        for s in self.specs:
            img = images[s.mid] if images is not None else s.image(seed)
            qm[(s.layer, s.name)] = QMat(img, s.N, s.K, s.e, s.sh, s.g)
        for i, lt in enumerate(geom.layer_types):
            p = vec[i]
            qw = {"type": lt, "ln1": p["ln1"], "ln2": p["ln2"],
                  "mlp": {k: qm[(i, k)] for k in ("gate", "up", "down")}}
            if lt == "full_attention":
                qw["attn"] = {k: qm[(i, k)] for k in ("q_proj", "k_proj", "v_proj", "o_proj")}
                qw["attn"]["q_norm"] = p["q_norm"]
                qw["attn"]["k_norm"] = p["k_norm"]
            else:
                qw["dn"] = {k: qm[(i, k)] for k in ("in_qkv", "in_z", "in_b", "in_a", "out")}
                for k in ("conv_w", "dt_bias_q12", "A_q15", "norm_w_q14"):
                    qw["dn"][k] = p[k]
            self.layers.append(qw)
        self.head = qm[(-1, "head")]

    def emb_row(self, tok):
        return synth.emb_rows(self.seed, [tok], self.geom.H)[0].astype(I64)

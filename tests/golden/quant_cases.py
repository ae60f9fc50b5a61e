"""Seeded float matrices for the quantizer parity cases (shared by
gen_quant_golden.py, which runs the reference quantizers on them, and
tests/test_gpu_quant.py, which runs the GPU quantizer on the same inputs).

Each case: (name, matrix, kind, kwargs) where kind is "mse" (quant_linear_mse),
"max" (quantize_weights) or "tight" (quant_linear(mse_scale=False,
tighten_e=True)).  The inputs cover the shapes of the 9B decode path
(K = 4096 and 12288), heavy-tailed and exactly-zero groups, float64 inputs
that float32 cannot hold, per-channel salience weights and a shorter alpha
grid.
"""
import numpy as np

SEED = 20261203


def cases():
    rng = np.random.default_rng(SEED)
    out = []
    w = rng.normal(0, 0.02, (48, 4096)).astype(np.float32)
    out.append(("normal_k4096", w, "mse", {}))
    t = (rng.normal(0, 1, (12, 12288)) * np.exp(rng.normal(0, 2.5, (12, 12288)))).astype(np.float32)
    t[3, 128:256] = 0.0                       # an all-zero group (scale floor 1e-12)
    t[5, 1000] = 40.0                         # one outlier dominating its group
    out.append(("heavy_k12288", t, "mse", {}))
    f = rng.normal(0, 0.05, (16, 1024))       # float64 values float32 cannot hold
    out.append(("float64_k1024", f, "mse", {}))
    s = np.abs(rng.normal(1.0, 0.7, 2048))
    out.append(("salience_k2048", rng.normal(0, 0.03, (20, 2048)).astype(np.float32), "mse",
                {"salience": s}))
    out.append(("grid5_k1024", rng.normal(0, 1.0, (8, 1024)).astype(np.float32), "mse",
                {"nalpha": 5, "amin": 0.7}))
    out.append(("max_rule_k4096", t[:, :4096].copy(), "max", {}))
    g = rng.normal(0, 0.02, (10, 1024)).astype(np.float32)
    g[0, 0] = 0.9                             # one large group: every other scale is far below it
    out.append(("tighten_k1024", g, "tight", {}))
    return out

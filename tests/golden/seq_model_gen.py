"""The random model of the reference's token-stream generator, rebuilt from
its seed without the reference (test input generation).

Restates the draw order of ref/gen_token_script.py:139-181 (per layer
init_layer_weights, then ln_f, the LM head, the embedding and the prompt
token) and of ref/layer_ref.py:107-166 (per layer ln1, ln2, the MLP gate /
up / down, then the attention q/k/v/o projections and q/k norms or the
DeltaNet in_qkv / in_z / in_b / in_a projections, conv taps, A_log,
norm_w and out projection; dt_bias is ones and draws nothing), with
numpy.random.default_rng(seed) and the reference's float32 casts, so the
float weights are bit-identical to the generator's.  tests/golden/seq9b
holds that generator run's stream and metadata, tests/golden/seq9b_ref.npz
its image digests and vectors, against which the GPU quantizer and the GPU
decode are checked.
"""
import numpy as np

f32 = np.float32
H, NQ, NKV, HD, FFN = 4096, 16, 4, 256, 12288
LNH, LNKH, LDK, LDV, CONV_K = 32, 16, 128, 128, 4
CONV_DIM = 2 * LNKH * LDK + LNH * LDV
LVD = LNH * LDV
RS_F = 7
LEGACY_TYPES = ["linear_attention", "full_attention"]


def _mlp(rng):
    s = 0.02
    return {"gate": rng.normal(0, s, (FFN, H)).astype(f32),
            "up": rng.normal(0, s, (FFN, H)).astype(f32),
            "down": rng.normal(0, s, (H, FFN)).astype(f32)}


def _attn(rng):
    s = 0.02
    return {"q_proj": rng.normal(0, s, (NQ * HD * 2, H)).astype(f32),
            "k_proj": rng.normal(0, s, (NKV * HD, H)).astype(f32),
            "v_proj": rng.normal(0, s, (NKV * HD, H)).astype(f32),
            "o_proj": rng.normal(0, s, (H, NQ * HD)).astype(f32),
            "q_norm": rng.normal(0, 0.1, HD).astype(f32),
            "k_norm": rng.normal(0, 0.1, HD).astype(f32)}


def _deltanet(rng):
    s = 0.02
    return {"in_qkv": rng.normal(0, s, (CONV_DIM, H)).astype(f32),
            "in_z": rng.normal(0, s, (LVD, H)).astype(f32),
            "in_b": rng.normal(0, s, (LNH, H)).astype(f32),
            "in_a": rng.normal(0, s, (LNH, H)).astype(f32),
            "conv_w": rng.normal(0, 0.3, (CONV_DIM, CONV_K)).astype(f32),
            "dt_bias": np.ones(LNH, dtype=f32),
            "A_log": np.log(rng.uniform(0.5, 8, LNH)).astype(f32),
            "norm_w": (1 + rng.normal(0, 0.1, LDV)).astype(f32),
            "out": rng.normal(0, s, (H, LVD)).astype(f32)}


def layer(rng, lt, out_scale=1.0):
    w = {"ln1": rng.normal(0, 0.1, H).astype(f32), "ln2": rng.normal(0, 0.1, H).astype(f32),
         "mlp": _mlp(rng), "type": lt}
    if lt == "full_attention":
        w["attn"] = _attn(rng)
    else:
        w["dn"] = _deltanet(rng)
    if out_scale != 1.0:
        w["mlp"]["down"] = (w["mlp"]["down"] * out_scale).astype(f32)
        key, sub = ("attn", "o_proj") if lt == "full_attention" else ("dn", "out")
        w[key][sub] = (w[key][sub] * out_scale).astype(f32)
    return w


def token_model(seed, layer_types=None, vocab=8192):
    """-> dict(layers=[float layer dicts], ln_f_q14, head (float64 [vocab, H]),
    emb_q (int16-range int64 [vocab, H]), prompt)."""
    layer_types = list(layer_types or LEGACY_TYPES)
    rng = np.random.default_rng(seed)
    out_scale = 1.0 if len(layer_types) == 2 else 1.0 / np.sqrt(2.0 * len(layer_types))
    layers = [layer(rng, lt, out_scale) for lt in layer_types]
    ln_f = np.clip(np.round(rng.normal(0, 0.5, H) * (1 << 14)), -32768, 32767).astype(np.int64)
    head = rng.normal(0, 1.0, (vocab, H)) / np.sqrt(H)
    emb = np.clip(np.round(rng.normal(0, 1, (vocab, H)) * (1 << RS_F)), -32768, 32767).astype(np.int64)
    tok = int(rng.integers(0, vocab))
    return {"layers": layers, "ln_f_q14": ln_f, "head": head, "emb_q": emb, "prompt": tok,
            "types": layer_types}

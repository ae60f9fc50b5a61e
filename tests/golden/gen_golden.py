#!/usr/bin/env python3
"""Generate the committed golden fixtures from the UNMODIFIED reference.

Run where the reference checkout exists, with the environment variable
F5_REFERENCE set to its root directory; the GPU box never runs it.
It reads the reference's own committed golden vectors (tb/vec_s1..s4 matvec
vectors, tb/vectors/s1..s4 unit-block vectors, the LUT ROM images) and runs
the reference's Python model (ref/w4a8_ref.py, ref/fixedpoint.py,
ref/layer_fixed.py) with FABLE5_MODEL=9b on seeded inputs, storing inputs and
outputs as small .npz files next to this script.

    python tests/golden/gen_golden.py            # unit + layer + reduced model
    python tests/golden/gen_golden.py --full     # + full 32-layer 9B model steps
    python tests/golden/gen_golden.py --only model32   # only those

Large exhaustive domains (e.g. silu over the whole 21-bit port) are stored as
sha256 digests of the int64 output plus a strided sample.
"""
from __future__ import annotations

import argparse
import hashlib
import os
import sys
import time

import numpy as np

REF = os.environ.get("F5_REFERENCE")
if not REF or not os.path.isdir(os.path.join(REF, "ref")):
    sys.exit("set F5_REFERENCE to the root of the reference checkout (the directory holding ref/)")
HERE = os.path.dirname(os.path.abspath(__file__))
REPO = os.path.dirname(os.path.dirname(HERE))
os.environ["FABLE5_MODEL"] = "9b"
os.environ["PYTHONDONTWRITEBYTECODE"] = "1"
sys.dont_write_bytecode = True
sys.path.insert(0, os.path.join(REF, "ref"))
sys.path.insert(0, REPO)

import fixedpoint as FP          # noqa: E402  (reference)
import layer_fixed as LF         # noqa: E402  (reference)
import layer_ref as LR           # noqa: E402  (reference)
import w4a8_ref as W             # noqa: E402  (reference)

from fable5_llm_b200 import synth  # noqa: E402

I64 = np.int64
SEED = 2026


def digest(a):
    return hashlib.sha256(np.ascontiguousarray(np.asarray(a, dtype=I64)).tobytes()).hexdigest()


def read_hex(path, width):
    vals = [int(l.strip(), 16) for l in open(path) if l.strip()]
    a = np.array(vals, dtype=object)
    sign = 1 << (width - 1)
    return np.array([(v ^ sign) - sign if width < 64 else v for v in vals], dtype=I64) if vals else np.zeros(0, I64)


def read_hex_u(path):
    return [int(l.strip(), 16) for l in open(path) if l.strip()]


# ---------------------------------------------------------------------------
def gen_tb_matvec():
    out = {}
    for s in range(1, 5):
        d = os.path.join(REF, "tb", f"vec_s{s}")
        K, NG, SH, N, BPR = [int(v) for v in open(os.path.join(d, "params.txt")).read().split()]
        words = read_hex_u(os.path.join(d, "x8.hex"))
        xb = b"".join(w.to_bytes(4, "little") for w in words)[:K]
        beats = read_hex_u(os.path.join(d, "beats.hex"))
        img = b"".join(b.to_bytes(64, "little") for b in beats)
        y32 = read_hex(os.path.join(d, "y32.hex"), 32)
        out[f"s{s}_params"] = np.array([K, NG, SH, N, BPR], dtype=I64)
        out[f"s{s}_x8"] = np.frombuffer(xb, dtype=np.int8).copy()
        out[f"s{s}_img"] = np.frombuffer(img, dtype=np.uint8).copy()
        out[f"s{s}_y32"] = y32.astype(np.int32)
    np.savez_compressed(os.path.join(HERE, "tb_matvec.npz"), **out)
    print("tb_matvec.npz", len(out))


LAYER_FILES = {  # name -> width (ref/gen_layer_vectors.py:9-16)
    "rmsnorm_x16": 16, "rmsnorm_w14": 16, "rmsnorm_y16": 16,
    "rope_x16": 16, "rope_cos": 16, "rope_sin": 16, "rope_y16": 16,
    "l2norm_x16": 16, "l2norm_y16": 16,
    "conv_win": 16, "conv_w": 16, "conv_y": 16,
    "attn_q": 16, "attn_k8": 8, "attn_ke": 8, "attn_v8": 8, "attn_ve": 8, "attn_p": 16,
    "attn_acc": 32,
    "dn_sin": 16, "dn_q": 16, "dn_k": 16, "dn_v": 16, "dn_sout": 16, "dn_o": 32,
    "gate_b": 16, "gate_a": 16, "gate_A": 18, "gate_dt": 16, "gate_beta": 16, "gate_decay": 16,
    "alu_dynq8_x": 16, "alu_dynq8_y": 16, "alu_dynq8_e": 16, "alu_shift32_v": 32,
    "alu_shift32_y": 16, "alu_scale_x": 16, "alu_scale_y": 16, "alu_emul_a": 16,
    "alu_emul_b": 16, "alu_emul_y": 16, "alu_add_y": 16, "alu_silu16_y": 16,
    "alu_silu32_y": 16, "alu_sigm16_y": 16, "alu_emul32_y": 16, "alu_shift32w_y": 32,
}


def gen_tb_layer():
    out = {}
    for s in range(1, 5):
        d = os.path.join(REF, "tb", "vectors", f"s{s}")
        for name, width in LAYER_FILES.items():
            p = os.path.join(d, name + ".hex")
            if os.path.exists(p):
                out[f"s{s}_{name}"] = read_hex(p, width)
        gates = open(os.path.join(d, "dn_gates.txt")).read().split()
        out[f"s{s}_dn_gates"] = np.array([int(v) for v in gates], dtype=I64)
    roms = {}
    rd = os.path.join(REF, "tb", "vectors", "s1", "roms")
    for name, width in (("rsqrt", 16), ("recip", 16), ("exp2", 18), ("sigmoid", 16), ("softplus", 17)):
        roms[name] = read_hex(os.path.join(rd, f"{name}_rom.hex"), 64)   # unsigned tables
    np.savez_compressed(os.path.join(HERE, "tb_layer.npz"), **out)
    np.savez_compressed(os.path.join(HERE, "roms.npz"), **roms)
    print("tb_layer.npz", len(out), "roms.npz", len(roms))


# ---------------------------------------------------------------------------
def gen_prims():
    rng = np.random.default_rng(SEED)
    out = {}
    # rshift_round KATs + random
    v = np.concatenate([np.array([5, -5, 4, -4, 3, -3, 0, 1, -1, 2, -2, 7, -7], dtype=I64),
                        rng.integers(-(1 << 40), 1 << 40, 3000)])
    s = rng.integers(-8, 41, v.size)
    s[:13] = 1
    out["rshr_v"], out["rshr_s"] = v, s
    out["rshr_y"] = np.array([int(W.rshift_round(I64(int(a)), int(b))) for a, b in zip(v, s)], dtype=I64)
    # dyn_quant_i8
    xs = np.concatenate([rng.integers(-32768, 32768, (300, 64)),
                         np.array([[0] * 64, [127] * 64, [-127] * 64, [128] * 64, [-128] * 64,
                                   [32767] * 64, [-32768] * 64, [255] * 64, [-255] * 64])]).astype(I64)
    out["dq_x"] = xs
    r = [FP.dyn_quant_i8(x) for x in xs]
    out["dq_x8"] = np.stack([a.astype(I64) for a, _ in r])
    out["dq_e"] = np.array([e for _, e in r], dtype=I64)
    # rsqrt_q / recip_q
    vv = np.concatenate([rng.integers(1, 1 << 48, 3000), np.array([1, 2, 3, 4, (1 << 30), (1 << 31) - 1,
                         (1 << 31), (1 << 32) - 1, (1 << 32), (1 << 47) + 12345], dtype=I64)])
    pp = np.concatenate([rng.integers(0, 48, 3000), np.array([0, 1, 2, 33, 30, 26, 16, 7, 0, 40], dtype=I64)])
    out["rs_v"], out["rs_p"] = vv, pp
    rs = [FP.rsqrt_q(int(a), int(b)) for a, b in zip(vv, pp)]
    out["rs_r"] = np.array([a for a, _ in rs], dtype=I64)
    out["rs_e"] = np.array([b for _, b in rs], dtype=I64)
    rc = [FP.recip_q(int(a), int(b)) for a, b in zip(vv, pp)]
    out["rc_r"] = np.array([a for a, _ in rc], dtype=I64)
    out["rc_e"] = np.array([b for _, b in rc], dtype=I64)
    # exhaustive LUT-function domains (digest + strided sample)
    doms = {
        "sigmoid": (FP.sigmoid_q, np.arange(-(1 << 17) - 64, (1 << 17) + 64, dtype=I64)),
        "softplus": (FP.softplus_q, np.arange(-(1 << 17) - 64, (1 << 17) + 64, dtype=I64)),
        "silu": (FP.silu_q, np.arange(-(1 << 20), 1 << 20, dtype=I64)),
        "exp_neg": (FP.exp_neg_q, -np.arange(0, 1 << 21, dtype=I64)),
        "exp2_frac": (FP.exp2_frac_q16, np.arange(0, 1 << 16, dtype=I64)),
    }
    for name, (fn, dom) in doms.items():
        t = time.time()
        y = np.array([int(fn(int(x))) for x in dom], dtype=I64)
        out[f"{name}_lo"], out[f"{name}_n"] = np.array(dom[0]), np.array(dom.size)
        out[f"{name}_sign"] = np.array(-1 if name == "exp_neg" else 1)
        out[f"{name}_digest"] = np.array(digest(y))
        out[f"{name}_sample"] = y[::97]
        print(f"  {name}: {dom.size} values in {time.time() - t:.1f}s")
    # exp_neg far tail (very negative)
    xt = -rng.integers(1 << 21, 1 << 40, 2000)
    out["expt_x"] = xt
    out["expt_y"] = np.array([FP.exp_neg_q(int(x)) for x in xt], dtype=I64)
    # bf_shift / attn_o_shift
    m = np.concatenate([np.arange(0, 70000, dtype=I64), rng.integers(0, 1 << 40, 4000),
                        (np.int64(1) << np.arange(0, 40)) - 1, (np.int64(1) << np.arange(0, 40))])
    out["bf_m"] = m
    out["bf_k"] = np.array([LF.bf_shift(int(a)) for a in m], dtype=I64)
    # dn_norm_scale / eps_norm_scale on random head blocks
    nb = 600
    scales = 10.0 ** rng.uniform(-1, 6, nb)
    blocks = np.round(rng.normal(0, 1, (nb, 128)) * scales[:, None]).astype(I64)
    blocks[0] = 0
    blocks[1, :] = 0
    blocks[1, 5] = 16384
    out["nb_o32"] = blocks
    ks = np.array([LF.dn_o_shift(b, note=False) for b in blocks], dtype=I64)
    out["nb_k"] = ks
    out["nb_m_float"] = np.array([LF.dn_norm_scale(b, int(k), note=False) for b, k in zip(blocks, ks)], dtype=I64)
    o16 = np.stack([LF.clip16(W.rshift_round(b, int(k))) for b, k in zip(blocks, ks)])
    out["nb_o16"] = o16
    out["nb_m_eps"] = np.array([LF.eps_norm_scale(o, int(k), note=False) for o, k in zip(o16, ks)], dtype=I64)
    # rmsnorm / l2norm
    for tag, n, in_f, one_plus, sd in (("rn4096", 4096, 7, True, 3.0), ("rn4096p", 4096, 7, False, 3.0),
                                       ("rn256", 256, 8, True, 1.0), ("rn128s", 128, 8, True, 0.01)):
        X = np.round(rng.normal(0, sd, (20, n)) * (1 << in_f)).astype(I64)
        X[0] = 0
        if one_plus:
            Wt = np.round(rng.normal(0, 0.1, n) * (1 << 14)).astype(I64)
        else:
            Wt = np.round((1 + rng.normal(0, 0.1, n)) * (1 << 12)).astype(I64)
        out[f"{tag}_x"], out[f"{tag}_w"] = X, Wt
        out[f"{tag}_y"] = np.stack([LF.rmsnorm_fx(x, Wt, in_f, one_plus) for x in X])
        out[f"{tag}_meta"] = np.array([n, in_f, int(one_plus)], dtype=I64)
    X = np.round(rng.normal(0, 1.5, (40, 128)) * (1 << 8)).astype(I64)
    X[0] = 0
    out["l2_x"] = X
    out["l2_y"] = np.stack([LF.l2norm_fx(x, 8, 14) for x in X])
    # rope tables and rope_fx
    pos = np.arange(0, 4096, dtype=I64)
    tabs = [LF.rope_tables_q15(int(p)) for p in pos]
    cos = np.stack([c for c, _ in tabs])
    sin = np.stack([s_ for _, s_ in tabs])
    out["rope_cos_digest"], out["rope_sin_digest"] = np.array(digest(cos)), np.array(digest(sin))
    out["rope_cos_sample"], out["rope_sin_sample"] = cos[::37], sin[::37]
    extra = np.array([65535, 100000, 1 << 20], dtype=I64)
    out["rope_extra_pos"] = extra
    out["rope_extra_cos"] = np.stack([LF.rope_tables_q15(int(p))[0] for p in extra])
    out["rope_extra_sin"] = np.stack([LF.rope_tables_q15(int(p))[1] for p in extra])
    Xr = np.round(rng.normal(0, 1, (20, 256)) * (1 << 8)).astype(I64)
    pr = rng.integers(0, 4096, 20)
    out["ropefx_x"], out["ropefx_pos"] = Xr, pr
    out["ropefx_y"] = np.stack([LF.rope_fx(x, *LF.rope_tables_q15(int(p))) for x, p in zip(Xr, pr)])
    np.savez_compressed(os.path.join(HERE, "ref_prims.npz"), **out)
    print("ref_prims.npz", len(out))


# ---------------------------------------------------------------------------
def ref_qmat(spec, seed):
    img = spec.image(seed)
    w4, m = W.unpack_ddr_rows(img.tobytes(), spec.N, spec.K, spec.g)
    return {"w4": w4, "m": m, "e": spec.e, "sh": spec.sh, "g": spec.g}


def ref_layer(seed, geom_types, i, specs, vec):
    lt = geom_types[i]
    mats = {s.name: ref_qmat(s, seed) for s in specs if s.layer == i}
    p = vec[i]
    qw = {"type": lt, "ln1": p["ln1"], "ln2": p["ln2"],
          "mlp": {k: mats[k] for k in ("gate", "up", "down")}}
    if lt == "full_attention":
        qw["attn"] = {k: mats[k] for k in ("q_proj", "k_proj", "v_proj", "o_proj")}
        qw["attn"]["q_norm"], qw["attn"]["k_norm"] = p["q_norm"], p["k_norm"]
    else:
        qw["dn"] = {k: mats[k] for k in ("in_qkv", "in_z", "in_b", "in_a", "out")}
        for k in ("conv_w", "dt_bias_q12", "A_q15", "norm_w_q14"):
            qw["dn"][k] = p[k]
    return qw


class Geom:
    def __init__(self, n_layers, vocab):
        self.n_layers, self.vocab = n_layers, vocab
        self.layer_types = [("full_attention" if i % 4 == 3 else "linear_attention") for i in range(n_layers)]
        for k in ("H", "NQ", "NKV", "HD", "FFN", "LNH", "LNKH", "LDK", "LDV", "CONV_DIM", "LVD"):
            setattr(self, k, getattr(LR, k))
        self.CONV_K = LR.CONV_K


def gen_layers():
    """One DN layer (both gated-norm modes) and one attention layer at 9B."""
    g = Geom(4, 4096)
    specs = synth.matrix_specs(g)
    vec, _ = synth.vector_params(SEED, g)
    out = {}
    nsteps = 4
    xs = np.stack([synth.emb_rows(SEED, [t], g.H)[0].astype(I64) * 1 for t in (11, 22, 33, 44, 55)])
    out["x_in"] = xs[:nsteps]
    for mode in ("float", "eps"):
        LF.SEQ_NORM = mode == "eps"
        qw = ref_layer(SEED, g.layer_types, 0, specs, vec)
        cache = LF.new_cache_fx(qw["type"])
        ys, ks = [], []
        for t in range(nsteps):
            ys.append(LF.layer_decode_fx(xs[t], qw, cache, t))
            ks.append(list(cache["dn_o_shift"]))
        out[f"dn_{mode}_y"] = np.stack(ys)
        out[f"dn_{mode}_k"] = np.array(ks, dtype=I64)
        out[f"dn_{mode}_S_digest"] = np.array(digest(cache["S"]))
        out[f"dn_{mode}_S_sample"] = cache["S"][:, ::17, ::13].astype(I64)
        out[f"dn_{mode}_conv"] = cache["conv"].astype(I64)
        out[f"dn_{mode}_sat"] = np.array(cache.get("sat", 0))
        print(f"  dn layer ({mode}) done")
    LF.SEQ_NORM = False
    qw = ref_layer(SEED, g.layer_types, 3, specs, vec)
    cache = LF.new_cache_fx(qw["type"])
    ys, kas = [], []
    for t in range(nsteps):
        ys.append(LF.layer_decode_fx(xs[t], qw, cache, t + 5))   # pos != T on purpose
        kas.append(cache["attn_o_shift"])
    out["attn_y"] = np.stack(ys)
    out["attn_ka"] = np.array(kas, dtype=I64)
    out["attn_k8"] = np.array([[k8 for k8, _ in row] for row in cache["k"]], dtype=I64)
    out["attn_ke"] = np.array([[ke for _, ke in row] for row in cache["k"]], dtype=I64)
    out["attn_v8"] = np.array([[v8 for v8, _ in row] for row in cache["v"]], dtype=I64)
    out["attn_ve"] = np.array([[ve for _, ve in row] for row in cache["v"]], dtype=I64)
    np.savez_compressed(os.path.join(HERE, "ref_layers.npz"), **out)
    print("ref_layers.npz", len(out))


def run_model(g, toks, tag):
    """FxRunner.step sequence (ref/fidelity_check.py:423-448) on the
    synthetic model, with the reference's own functions."""
    specs = synth.matrix_specs(g)
    vec, ln_f = synth.vector_params(SEED, g)
    head_spec = [s for s in specs if s.name == "head"][0]
    caches = [LF.new_cache_fx(t) for t in g.layer_types]
    out_toks, layer_x, ymax = [], [], []
    layers = [ref_layer(SEED, g.layer_types, i, specs, vec) for i in range(g.n_layers)]
    for t, tok in enumerate(toks):
        t0 = time.time()
        x = synth.emb_rows(SEED, [tok], g.H)[0].astype(I64)
        lx = []
        for i, qw in enumerate(layers):
            x = LF.layer_decode_fx(x, qw, caches[i], t)
            lx.append(x.astype(np.int16))
        xn = LF.rmsnorm_fx(x, ln_f, LF.RS_F, False)
        x8, _ = FP.dyn_quant_i8(xn)
        ys = []
        for r0 in range(0, g.vocab, 8192):
            r1 = min(r0 + 8192, g.vocab)
            img = head_spec.image(SEED, r0, r1)
            w4, m = W.unpack_ddr_rows(img.tobytes(), r1 - r0, g.H)
            ys.append(W.matvec_y32(w4, m, head_spec.sh, x8).astype(I64))
        y = np.concatenate(ys)
        out_toks.append(int(np.argmax(y)))
        ymax.append(int(y.max()))
        layer_x.append(np.stack(lx))
        print(f"  {tag} step {t}: tok {tok} -> {out_toks[-1]} ({time.time() - t0:.1f}s)", flush=True)
    return {f"{tag}_in": np.array(toks, dtype=I64), f"{tag}_out": np.array(out_toks, dtype=I64),
            f"{tag}_ymax": np.array(ymax, dtype=I64), f"{tag}_layer_x": np.stack(layer_x)}


def gen_model():
    g = Geom(4, 4096)
    out = run_model(g, [17, 901, 4000, 3, 17, 256], "m4")
    np.savez_compressed(os.path.join(HERE, "ref_model4.npz"), **out)
    print("ref_model4.npz")


def gen_model32():
    """The full 32-layer 9B model with the 248,320-row head for three host
    tokens (about four minutes per step through the reference)."""
    g = Geom(32, 248320)
    out = run_model(g, [1234, 248319, 77], "m32")
    np.savez_compressed(os.path.join(HERE, "ref_model32.npz"), **out)
    print("ref_model32.npz")


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--full", action="store_true")
    ap.add_argument("--only", default="")
    a = ap.parse_args()
    parts = a.only.split(",") if a.only else ["tb", "prims", "layers", "model"] + (["model32"] if a.full else [])
    if "tb" in parts:
        gen_tb_matvec()
        gen_tb_layer()
    if "prims" in parts:
        gen_prims()
    if "layers" in parts:
        gen_layers()
    if "model" in parts:
        gen_model()
    if "model32" in parts:
        gen_model32()


if __name__ == "__main__":
    main()

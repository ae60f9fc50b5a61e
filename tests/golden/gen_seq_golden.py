#!/usr/bin/env python3
"""Generate the SEQ-stream fixtures from the UNMODIFIED reference.

Run where the reference checkout exists, with the environment variable
F5_REFERENCE set to its root directory; the GPU box never runs it.

1. ref/gen_token_script.py writes a 9B-geometry token stream with the SEQ
   emitter on (FABLE5_MODEL=9b SEQ_EMIT=1 SEQ_PROFILE=epsnorm), vocab 8192:
   by default seed 1, 3 tokens, the legacy 2-layer stack (one DeltaNet +
   one full-attention layer, "tok9"); --seed 2 --ntok 4 --nlayers 4 --name
   tok9l4 gives the config's first four layers (3 DeltaNet + 1 attention,
   per-layer banked state, residual projections scaled by 1/sqrt(8)).  The
   weight images (265-450 MB), embedding (64 MB) and state images
   (2 x 155 MB) stay outside the repository.
2. ref/seq_model.py --gate replays the .txt script and the .seq stream and
   must print "SEQ GATE: PASS" (tokens, banked state, state region and
   scratch bit-identical).
3. The same model is rebuilt in-process from the reference's own functions
   (layer_ref.init_layer_weights, layer_fixed.quant_layer / quant_linear, in
   the generator's RNG order) and stepped with layer_decode_fx, recording
   every layer's output; the final caches are compared with the artifact's
   final state image decoded by fable5_llm_b200.state_region (pinning that
   layout restatement).

Written: tests/golden/seq9b/<name>.{seq,seq.json,seqdata.bin,weights.json}
(the stream, its blob and metadata, the weight manifest: ~80 KB) and
tests/golden/seq9b_ref.npz (<name>_ref.npz for other names: tokens, layer
outputs, the quantized vectors, and the sha256 of every weight image, the
embedding and both state images).

    python tests/golden/gen_seq_golden.py [--artifact PREFIX] [--seed S --ntok N --nlayers L --name NAME]
"""
from __future__ import annotations

import argparse
import hashlib
import os
import shutil
import subprocess
import sys
import tempfile

import numpy as np

REF = os.environ.get("F5_REFERENCE")
if not REF or not os.path.isdir(os.path.join(REF, "ref")):
    sys.exit("set F5_REFERENCE to the root of the reference checkout (the directory holding ref/)")
HERE = os.path.dirname(os.path.abspath(__file__))
REPO = os.path.dirname(os.path.dirname(HERE))
ENV = dict(os.environ, FABLE5_MODEL="9b", SEQ_EMIT="1", SEQ_PROFILE="epsnorm", PYTHONDONTWRITEBYTECODE="1")
os.environ["FABLE5_MODEL"] = "9b"
sys.dont_write_bytecode = True
SEED, NTOK, VOCAB, NLAYERS = 1, 3, 8192, 2
NAME = "tok9"
LEGACY_TYPES = ["linear_attention", "full_attention"]


def sha_file(path):
    h = hashlib.sha256()
    with open(path, "rb") as f:
        for blk in iter(lambda: f.read(1 << 24), b""):
            h.update(blk)
    return h.hexdigest()


def make_artifact(d):
    out = os.path.join(d, NAME + ".txt")
    subprocess.run([sys.executable, os.path.join(REF, "ref", "gen_token_script.py"), out, str(SEED), str(NTOK),
                    str(VOCAB), str(NLAYERS)], env=ENV, check=True)
    return os.path.join(d, NAME)


def gate(prefix):
    r = subprocess.run([sys.executable, os.path.join(REF, "ref", "seq_model.py"), "--gate", prefix],
                       env=ENV, capture_output=True, text=True)
    print(r.stdout[-1500:])
    if r.returncode or "SEQ GATE: PASS" not in r.stdout:
        sys.exit("the reference SEQ gate did not pass")


def layer_types(nlayers):
    """ref/gen_token_script.py:90-100: the legacy pair at 2 layers, else
    the config's first nlayers types."""
    if nlayers == 2:
        return list(LEGACY_TYPES)
    import json
    cfg = json.load(open(os.path.join(REF, "ref", "qwen3_5_9b_config.json")))
    return cfg["text_config"]["layer_types"][:nlayers]


def rebuild_and_step(prefix):
    sys.path.insert(0, os.path.join(REF, "ref"))
    sys.path.insert(0, REPO)
    import json

    import fixedpoint as FP      # noqa: E402  (reference)
    import layer_fixed as LF     # noqa: E402  (reference)
    import layer_ref as LR       # noqa: E402  (reference)
    import w4a8_ref as W         # noqa: E402  (reference)
    from fable5_llm_b200.state_region import StateRegion, slots

    rng = np.random.default_rng(SEED)
    types = layer_types(NLAYERS)
    out_scale = 1.0 if NLAYERS == 2 else 1.0 / np.sqrt(2.0 * NLAYERS)
    layers = [LF.quant_layer(LR.init_layer_weights(rng, lt, out_scale=out_scale)) for lt in types]
    ln_f = np.asarray(np.clip(np.round(rng.normal(0, 0.5, LR.H) * (1 << 14)), -32768, 32767), dtype=np.int64)
    _hw = rng.normal(0, 1.0, (VOCAB, LR.H)) / np.sqrt(LR.H)
    head = LF.quant_linear(_hw)
    emb = np.asarray(np.clip(np.round(rng.normal(0, 1, (VOCAB, LR.H)) * (1 << LF.RS_F)), -32768, 32767),
                     dtype=np.int64)
    tok = int(rng.integers(0, VOCAB))
    caches = [LF.new_cache_fx(lt) for lt in types]
    toks, outs = [], []
    for t in range(NTOK):
        x = emb[tok].copy()
        step = []
        for qw, c in zip(layers, caches):
            x = LF.layer_decode_fx(x, qw, c, t)
            step.append(x.copy())
        outs.append(step)
        xn = LF.rmsnorm_fx(x, ln_f, LF.RS_F, True)
        x8, _ = FP.dyn_quant_i8(xn)
        y32 = W.matvec_y32(head["w4"], head["m"], head["sh"], x8, g=head["g"])
        tok = int(np.argmax(y32))
        toks.append(tok)
    meta = json.load(open(prefix + ".seq.json"))
    assert toks == meta["expect_tokens"], (toks, meta["expect_tokens"])
    # the final state image, decoded by this repository's layout restatement
    man = json.load(open(prefix + ".weights.json"))
    reg = StateRegion(man["state"], open(prefix + ".state_final.bin", "rb").read())
    for i, (lt, d, a) in enumerate(slots(types)):
        c = caches[i]
        if lt == "full_attention":
            k8, ke, v8, ve = reg.kv(a, NTOK)
            for t in range(NTOK):
                for h in range(4):
                    assert np.array_equal(k8[t, h], c["k"][t][h][0]) and ke[t, h] == c["k"][t][h][1]
                    assert np.array_equal(v8[t, h], c["v"][t][h][0]) and ve[t, h] == c["v"][t][h][1]
        else:
            taps, win = reg.conv(d)
            assert np.array_equal(reg.dn_state(d), c["S"]), "DN S"
            assert np.array_equal(win, c["conv"]), "conv window"
            assert np.array_equal(taps, layers[i]["dn"]["conv_w"]), "conv taps"
    print("final state image == layer_decode_fx caches (S, conv taps + window, K/V rows + exponents)")
    vec = {"ln_f": ln_f}
    for i, qw in enumerate(layers):
        vec[f"l{i}_ln1"], vec[f"l{i}_ln2"] = qw["ln1"], qw["ln2"]
        if qw["type"] == "full_attention":
            vec[f"l{i}_q_norm"], vec[f"l{i}_k_norm"] = qw["attn"]["q_norm"], qw["attn"]["k_norm"]
        else:
            d = qw["dn"]
            vec[f"l{i}_conv_w"], vec[f"l{i}_dt_bias_q12"] = d["conv_w"], d["dt_bias_q12"]
            vec[f"l{i}_A_q15"], vec[f"l{i}_norm_w_q14"] = d["A_q15"], d["norm_w_q14"]
    return toks, np.array(outs, dtype=np.int16), vec


def main():
    global SEED, NTOK, NLAYERS, NAME
    ap = argparse.ArgumentParser()
    ap.add_argument("--artifact", help="reuse an artifact written by step 1 (its prefix)")
    ap.add_argument("--seed", type=int, default=SEED)
    ap.add_argument("--ntok", type=int, default=NTOK)
    ap.add_argument("--nlayers", type=int, default=NLAYERS)
    ap.add_argument("--name", default=NAME)
    a = ap.parse_args()
    SEED, NTOK, NLAYERS, NAME = a.seed, a.ntok, a.nlayers, a.name
    td = None
    if a.artifact:
        prefix = a.artifact
    else:
        td = tempfile.mkdtemp()
        prefix = make_artifact(td)
    gate(prefix)
    toks, outs, vec = rebuild_and_step(prefix)
    dst = os.path.join(HERE, "seq9b")
    os.makedirs(dst, exist_ok=True)
    for ext in (".seq", ".seq.json", ".seqdata.bin", ".weights.json"):
        shutil.copyfile(prefix + ext, os.path.join(dst, NAME + ext))
    import json
    man = json.load(open(prefix + ".weights.json"))
    wids = sorted(int(k) for k in man if k.isdigit())
    digests = np.array([sha_file(os.path.join(os.path.dirname(prefix), man[str(w)]["file"])) for w in wids])
    ref_name = "seq9b_ref.npz" if NAME == "tok9" else f"{NAME}_ref.npz"
    np.savez_compressed(os.path.join(HERE, ref_name), tokens=np.array(toks), layer_out=outs,
                        image_sha256=digests, emb_sha256=np.array(sha_file(prefix + ".emb.bin")),
                        state_sha256=np.array(sha_file(prefix + ".state.bin")),
                        state_final_sha256=np.array(sha_file(prefix + ".state_final.bin")),
                        seed=np.array(SEED), vocab=np.array(VOCAB), nlayers=np.array(NLAYERS), **vec)
    print("tokens", toks, "->", dst)
    if td:
        shutil.rmtree(td)


if __name__ == "__main__":
    main()

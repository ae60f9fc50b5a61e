"""Replay of a SEQ artifact's decode on the GPU (the SEQ-stream
compatibility harness).

A reference generator run (ref/gen_token_script.py with the SEQ emitter)
leaves a record stream that drives the decode (``.seq`` + ``.seqdata.bin`` +
``.seq.json``), the weight images it streams (``.weights.json`` +
``_w<wid>.bin``), the embedding table (``.emb.bin``) and the DDR state
region before and after the run (``.state.bin``; the final image's sha256 is
in the manifest).  ``ref/seq_model.py gate`` replays that stream on the
reference executor; this harness runs the same decode through the GPU
engine and checks it against what the stream says:

  * geometry: the stack's layer types are read off the weight plan (wid
    order of ref/gen_layer_script.py:1522-1525 -- per DeltaNet layer 8
    images led by in_qkv / in_z, per attention layer 7 led by q_proj /
    k_proj, then the LM head);
  * weights: every image is uploaded as-is into the resident row format
    (``f5_ctx_upload_matrix``), from the artifact's files or from images the
    caller made (e.g. ``quant.quant_linear_image``);
  * constants: every per-layer vector the caller supplies must be one of the
    stream's LDC payloads (ref/seq_model.py:1125-1133) -- the stream is the
    authority on norm gains and gate constants; DeltaNet conv taps travel in
    the state image's cv blocks instead and are taken from there;
  * the run: the prompt (``prompt_fed``) and then greedy decoding until as
    many tokens as ``expect_tokens`` are emitted, through ``DecodeModel``
    (the persistent engine) in the stream's norm mode -- the "epsnorm"
    profile's EPS-NORM law for the DeltaNet gated norm, or the float law;
  * the result: the tokens, and the final state region image
    (``state_region.StateRegion.from_model``), whose sha256 the manifest
    records as ``final_sha256``.

Final norm: the token generator applies vecnorm mode 0, i.e. rmsnorm_fx with
the (1 + w) gain ln_f + 2^14 (ref/gen_token_script.py:231-235), which is the
engine's plain-gain final norm with that sum uploaded.
"""
from __future__ import annotations

import numpy as np

from . import _lib as L
from .artifact import read_embedding, read_weights
from .config import Geometry
from .seq_stream import SeqArtifact
from .state_region import StateRegion, slots

DN_NAMES = ("in_qkv", "in_z", "in_b", "in_a", "out", "gate", "up", "down")
ATTN_NAMES = ("q_proj", "k_proj", "v_proj", "o_proj", "gate", "up", "down")


def layer_types_of(plan, H=4096):
    """Layer types of the stack a weight plan streams (wid order), and the
    head's vocab."""
    plan = {int(k): v for k, v in plan.items()}
    wids = sorted(plan)
    shapes = [(int(plan[w]["nrows"]), int(plan[w]["k"])) for w in wids]
    g = Geometry(1)
    types, i = [], 0
    while i < len(shapes) - 1:
        if shapes[i] == (g.CONV_DIM, H) and i + 1 < len(shapes) and shapes[i + 1] == (g.LVD, H):
            types.append("linear_attention")
            i += len(DN_NAMES)
        elif shapes[i] == (g.NQ * g.HD * 2, H) and i + 1 < len(shapes) and shapes[i + 1] == (g.NKV * g.HD, H):
            types.append("full_attention")
            i += len(ATTN_NAMES)
        else:
            raise ValueError(f"wid {wids[i]}: shape {shapes[i]} starts no known layer")
    if i != len(shapes) - 1 or shapes[-1][1] != H:
        raise ValueError("the weight plan does not end with one LM head image")
    return types, shapes[-1][0]


def _as_i16_words(v):
    """A vector as the int16 words an LDC would carry: int16 values as they
    are, wider values as little-endian 16-bit halves."""
    a = np.asarray(v, dtype=np.int64)
    if a.min(initial=0) >= -32768 and a.max(initial=0) <= 32767:
        return a
    return np.asarray(a, dtype="<i4").view("<i2").astype(np.int64)


class SeqHarness(object):
    def __init__(self, artifact, layers, ln_f_q14, emb_q=None, images=None, norm_mode=None, state=None,
                 max_T=64):
        """artifact: SeqArtifact; layers: per layer the reference dict's
        vectors (``ln1``, ``ln2`` and ``dn`` / ``attn`` sub-dicts; matrices
        are not read); ln_f_q14: the final norm weight (Q14, before the
        1 + w); images: {wid: (uint8 image, e)} (None: the artifact's
        files); emb_q: int16 [vocab, H] (None: ``.emb.bin``); state:
        StateRegion before the run (None: ``.state.bin`` when present)."""
        self.art = artifact
        self.types, self.vocab = layer_types_of(artifact.meta["weights"])
        if len(layers) != len(self.types):
            raise ValueError(f"{len(layers)} layer dicts for a {len(self.types)}-layer stream")
        self.layers, self.ln_f = layers, np.asarray(ln_f_q14, dtype=np.int64)
        self.norm_mode = norm_mode or ("eps" if artifact.profile == "epsnorm" else "float")
        prefix = artifact.prefix
        if images is None:
            mats, meta = read_weights(prefix)
            images = {w: (m.img, m.e) for w, m in mats.items()}
        self.images = images
        if emb_q is None:
            emb_q = read_embedding(prefix, self.vocab, 4096, int(artifact.manifest.get("emb_row_bytes", 8192)))
        self.emb = emb_q
        if state is None and artifact.manifest.get("state") is not None and prefix is not None:
            try:
                state = StateRegion.load(prefix)
            except FileNotFoundError:
                state = None
        self.state0 = state
        self.max_T = max_T
        self.model = None

    def check_constants(self):
        """Every supplied vector is an LDC payload of the stream."""
        pays = [p for _, _, p in self.art.ldc_payloads() if p is not None]

        def found(v):
            w = _as_i16_words(v)
            return any(p.size == w.size and np.array_equal(p, w) for p in pays)
        missing = []
        for i, (qw, lt) in enumerate(zip(self.layers, self.types)):
            vs = {"ln1": qw["ln1"], "ln2": qw["ln2"]}
            if lt == "full_attention":
                vs.update(q_norm=qw["attn"]["q_norm"], k_norm=qw["attn"]["k_norm"])
            else:
                d = qw["dn"]
                vs.update(dt_bias_q12=d["dt_bias_q12"], A_q15=d["A_q15"], norm_w_q14=d["norm_w_q14"])
            missing += [f"layer {i} {k}" for k, v in vs.items() if not found(v)]
        if not found(self.ln_f):
            missing.append("ln_f")
        if missing:
            raise AssertionError("vectors absent from the stream's LDC payloads: " + ", ".join(missing))

    def build(self):
        from .model import DecodeModel
        g = Geometry(len(self.types), self.vocab, self.types)
        m = DecodeModel(g, max_T=self.max_T, max_pos=self.max_T, norm_mode=self.norm_mode)
        m.reset()
        wid = 0
        taps = self.state0.apply_to(m, 0) if self.state0 is not None else {}
        for i, lt in enumerate(self.types):
            for nm in (ATTN_NAMES if lt == "full_attention" else DN_NAMES):
                img, e = self.images[wid]
                p = self.art.meta["weights"][str(wid)]
                m.upload_matrix(i, m.slot_of(nm), np.asarray(img.cpu() if hasattr(img, "cpu") else img,
                                                             dtype=np.uint8),
                                int(p["nrows"]), int(p["k"]), int(e), int(p["sh"]), int(p.get("g", 128)))
                wid += 1
            qw = dict(self.layers[i])
            if lt != "full_attention" and i in taps:
                if "conv_w" in qw["dn"] and not np.array_equal(np.asarray(qw["dn"]["conv_w"]), taps[i]):
                    raise AssertionError(f"layer {i}: conv taps differ from the state image's cv block")
                qw["dn"] = dict(qw["dn"], conv_w=taps[i])
            qw["type"] = lt
            m.upload_layer_vectors(i, qw)
        img, e = self.images[wid]
        p = self.art.meta["weights"][str(wid)]
        m.upload_matrix(-1, L.S_HEAD, np.asarray(img.cpu() if hasattr(img, "cpu") else img, dtype=np.uint8),
                        int(p["nrows"]), int(p["k"]), int(e), int(p["sh"]), int(p.get("g", 128)))
        m.upload_final_norm(self.ln_f + (1 << 14))
        m.upload_embedding(self.emb)
        self.taps = {i: (taps[i] if i in taps else np.asarray(self.layers[i]["dn"]["conv_w"]))
                     for i, (lt, _, _) in enumerate(slots(self.types)) if lt != "full_attention"}
        self.model = m
        return m

    def run(self):
        """-> the emitted tokens (prompt, then greedy steps)."""
        m = self.model or self.build()
        prompt = self.art.prompt
        n = len(self.art.expect_tokens)
        toks = []
        self.residuals = []      # the final layer's output after every step
        for t in range(len(prompt) - 1):
            m.decode_step(int(prompt[t]), t)
            self.residuals.append(m.read(L.BUF_X16).astype(np.int64))
        t = len(prompt) - 1
        tok = int(prompt[-1])
        while len(toks) < n:
            tok, _ = m.decode_step(tok, t)
            self.residuals.append(m.read(L.BUF_X16).astype(np.int64))
            toks.append(int(tok))
            t += 1
        self.T = t
        return toks

    def final_state(self):
        plan = self.art.manifest["state"]
        return StateRegion.from_model(plan, self.model, self.T, self.taps)

    def close(self):
        if self.model is not None:
            self.model.close()
            self.model = None

"""Reference weight artifacts: packed row images plus ``.weights.json``.

The reference's generator writes every matrix it streams as one file
``<prefix>_w<wid>.bin`` in the packed DDR row format (``pack_ddr_rows``,
ref/w4a8_ref.py:349-370) and lists them in ``<prefix>.weights.json``
(``Mach.dump_weights``, ref/gen_layer_script.py:1555-1670); its host tools
read the manifest with ``sw/hwmap.load_weights_manifest``
(sw/hwmap.py:477-529).  The row format is the one this library keeps
resident in HBM, so an artifact loads into a ``DecodeModel`` image by image,
without unpacking or re-quantizing anything.

Manifest, per wid (a decimal string key): ``file``, ``nrows``, ``k``,
``ng`` (= k // 128), ``sh``, ``e``, ``nbeats`` (= nrows * stride / 64),
``stride``, then ``g`` only when it is not 128 and ``w8`` only when true.
Artifact-level keys: ``emb_row_bytes`` (absent: 8192) and ``rs_f`` (absent:
8, sw/hwmap.py:496-508), and the state-region keys ``state`` /
``conv_images``, which this loader leaves alone (the decode state starts at
zero here and the conv taps come with the layer vectors).

Wids are handed out in first-use order (ref/gen_layer_script.py:1522-1525)
over the first decoded token: per DeltaNet layer in_qkv, in_z, in_b, in_a,
out (ref/gen_layer_script.py:1945-2047), per attention layer q_proj, k_proj,
v_proj, o_proj (:2068-2154), then the layer's MLP gate, up, down
(:2174-2188), and after the last layer the LM head
(ref/gen_model_script.py:634).  ``wid_plan`` restates that order.

Errors follow the reference: a malformed manifest or image raises
``ValueError``; W8 images (``"w8": true``) are refused because the W4A8
decode path has no W8 rows; a manifest whose ``rs_f`` differs from this
build's residual binary point is refused, since every head logit would be
scaled by a power of two (the emit/consume tie of
ref/gen_layer_script.py:1641-1663).
"""
from __future__ import annotations

import json
import os

import numpy as np

from .config import RS_F
from .w4a8_ref import pack_ddr_rows, row_stride

RS_F_MANIFEST_DEFAULT = 8          # sw/hwmap.py:506 (a manifest without rs_f)
EMB_ROW_BYTES_DEFAULT = 8192       # sw/hwmap.py:495
META_KEYS = ("emb_row_bytes", "rs_f", "state", "conv_images")

DN_ORDER = ("in_qkv", "in_z", "in_b", "in_a", "out")
ATTN_ORDER = ("q_proj", "k_proj", "v_proj", "o_proj")
MLP_ORDER = ("gate", "up", "down")


def wid_plan(layer_types):
    """[(layer, name)] in wid order; layer -1 is the LM head ("head")."""
    plan = []
    for i, lt in enumerate(layer_types):
        own = ATTN_ORDER if lt == "full_attention" else DN_ORDER
        plan += [(i, nm) for nm in own + MLP_ORDER]
    plan.append((-1, "head"))
    return plan


class WeightImage:
    """One packed matrix: ``img`` uint8 [N, stride] plus (N, K, e, sh, g), the
    reference dict {"w4","m","e","sh","g"} in its wire form."""

    def __init__(self, img, N, K, e, sh, g=128):
        self.N, self.K, self.e, self.sh, self.g = int(N), int(K), int(e), int(sh), int(g)
        self.img = np.ascontiguousarray(img, dtype=np.uint8).reshape(self.N, row_stride(self.K, self.g))

    @classmethod
    def from_dict(cls, qw):
        N, K = np.asarray(qw["w4"]).shape
        g = int(qw.get("g", 128))
        img, _ = pack_ddr_rows(qw["w4"], qw["m"], g)
        return cls(np.frombuffer(img, dtype=np.uint8), N, K, qw["e"], qw["sh"], g)


def _as_image(m):
    if isinstance(m, WeightImage):
        return m
    if isinstance(m, dict):
        if "w8" in m:
            raise ValueError("W8 matrices have no W4A8 row image")
        return WeightImage.from_dict(m)
    return WeightImage(m.img, m.N, m.K, m.e, m.sh, getattr(m, "g", 128))


def write_weights(prefix, mats, emb_q=None, emb_row_bytes=None, rs_f=None):
    """Write ``mats`` (wid order: reference dicts or packed images) as
    ``<prefix>_w<wid>.bin`` files and ``<prefix>.weights.json`` in the
    layout of ref/gen_layer_script.py:1626-1668; ``emb_q`` (int16
    [vocab][H]) goes to ``<prefix>.emb.bin``.  Returns the number of wids."""
    man = {}
    for wid, m in enumerate(mats):
        im = _as_image(m)
        fn = f"{prefix}_w{wid}.bin"
        with open(fn, "wb") as f:
            f.write(im.img.tobytes())
        ent = {"file": os.path.basename(fn), "nrows": im.N, "k": im.K, "ng": im.K // 128, "sh": im.sh,
               "e": im.e, "nbeats": im.img.size // 64, "stride": im.img.shape[1]}
        if im.g != 128:
            ent["g"] = im.g
        man[wid] = ent
    if emb_row_bytes is not None:
        man["emb_row_bytes"] = int(emb_row_bytes)
    if rs_f is not None:
        man["rs_f"] = int(rs_f)
    elif RS_F != RS_F_MANIFEST_DEFAULT:
        raise ValueError(f"a manifest without rs_f reads as {RS_F_MANIFEST_DEFAULT}, this build's residual "
                         f"binary point is {RS_F}: pass rs_f")
    with open(f"{prefix}.weights.json", "w") as f:
        json.dump(man, f, indent=1)
    if emb_q is not None:
        np.ascontiguousarray(emb_q, dtype="<i2").tofile(f"{prefix}.emb.bin")
    return len(mats)


def read_weights(prefix):
    """Read ``<prefix>.weights.json`` and its images -> ({wid: WeightImage},
    meta with emb_row_bytes / rs_f defaulted as sw/hwmap.py does).  Every
    field is checked against the row law before any byte is trusted."""
    with open(f"{prefix}.weights.json") as f:
        man = json.load(f)
    meta = {"emb_row_bytes": int(man.get("emb_row_bytes", EMB_ROW_BYTES_DEFAULT)),
            "rs_f": int(man.get("rs_f", RS_F_MANIFEST_DEFAULT)),
            "state": man.get("state"), "conv_images": man.get("conv_images")}
    base = os.path.dirname(os.path.abspath(f"{prefix}.weights.json"))
    out = {}
    for key, ent in man.items():
        if key in META_KEYS:
            continue
        try:
            wid = int(key)
        except ValueError:
            raise ValueError(f"manifest key {key!r} is neither a wid nor a known artifact key") from None
        if ent.get("w8", False):
            raise ValueError(f"wid {wid}: W8 image; the W4A8 decode path has no W8 rows")
        N, K, g = int(ent["nrows"]), int(ent["k"]), int(ent.get("g", 128))
        if g not in (64, 128) or K % 128 or N <= 0:
            raise ValueError(f"wid {wid}: no row format for nrows={N} k={K} g={g}")
        stride = row_stride(K, g)
        if int(ent["ng"]) != K // 128 or int(ent["stride"]) != stride or int(ent["nbeats"]) * 64 != N * stride:
            raise ValueError(f"wid {wid}: ng/stride/nbeats {ent['ng']}/{ent['stride']}/{ent['nbeats']} "
                             f"do not match nrows={N} k={K} g={g} (stride {stride})")
        path = os.path.join(base, os.path.basename(ent["file"]))
        img = np.fromfile(path, dtype=np.uint8)
        if img.size != N * stride:
            raise ValueError(f"wid {wid}: {path} holds {img.size} B, the manifest says {N * stride}")
        out[wid] = WeightImage(img, N, K, int(ent["e"]), int(ent["sh"]), g)
    return out, meta


def read_embedding(prefix, vocab, H, emb_row_bytes):
    """``<prefix>.emb.bin``: int16 [vocab][H], rows emb_row_bytes apart."""
    if emb_row_bytes != 2 * H:
        raise ValueError(f"emb_row_bytes {emb_row_bytes} != 2*H = {2 * H}")
    emb = np.fromfile(f"{prefix}.emb.bin", dtype="<i2")
    if emb.size != vocab * H:
        raise ValueError(f"{prefix}.emb.bin holds {emb.size} int16, expected {vocab}*{H}")
    return emb.reshape(vocab, H)


def load_artifact(model, prefix, layers=None, ln_f_q12=None):
    """Upload a reference artifact into ``model`` (a DecodeModel): every
    matrix image by wid (``wid_plan`` over the model's layer types), and the
    embedding when ``<prefix>.emb.bin`` exists.  The per-layer integer
    vectors (norm gains, conv taps, gates) are not in the weights manifest:
    pass the reference layer dicts as ``layers`` and the final norm gain as
    ``ln_f_q12`` to upload them too."""
    mats, meta = read_weights(prefix)
    if meta["rs_f"] != RS_F:
        raise ValueError(f"artifact emitted with rs_f={meta['rs_f']}, this build's residual binary point is {RS_F}")
    g = model.geom
    plan = wid_plan(g.layer_types)
    if sorted(mats) != list(range(len(plan))):
        raise ValueError(f"artifact has wids {min(mats, default=None)}..{max(mats, default=None)} "
                         f"({len(mats)}), the model's layer types need 0..{len(plan) - 1}")
    shapes = _shapes(g)
    for wid, (layer, name) in enumerate(plan):
        im = mats[wid]
        want = (g.vocab, g.H) if name == "head" else shapes[name]
        if (im.N, im.K) != want:
            raise ValueError(f"wid {wid} ({name} of layer {layer}): {im.N}x{im.K}, the model needs "
                             f"{want[0]}x{want[1]}")
        model.upload_qmat(layer, model.slot_of(name), im)
    if os.path.exists(f"{prefix}.emb.bin"):
        model.upload_embedding(read_embedding(prefix, g.vocab, g.H, meta["emb_row_bytes"]))
    if layers is not None:
        for i, qw in enumerate(layers):
            model.upload_layer_vectors(i, qw)
    if ln_f_q12 is not None:
        model.upload_final_norm(ln_f_q12)
    return meta


def _shapes(g):
    """(rows, K) of every per-layer matrix at geometry g
    (ref/layer_fixed.py:1607-1651 over ref/layer_ref.py:25-49)."""
    return {"in_qkv": (g.CONV_DIM, g.H), "in_z": (g.LVD, g.H), "in_b": (g.LNH, g.H), "in_a": (g.LNH, g.H),
            "out": (g.H, g.LVD), "q_proj": (2 * g.NQ * g.HD, g.H), "k_proj": (g.NKV * g.HD, g.H),
            "v_proj": (g.NKV * g.HD, g.H), "o_proj": (g.H, g.NQ * g.HD), "gate": (g.FFN, g.H),
            "up": (g.FFN, g.H), "down": (g.H, g.FFN)}

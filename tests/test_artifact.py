"""Reference weight artifacts (``<prefix>.weights.json`` + ``_w<wid>.bin``).

Pinned to fixtures written by the reference's own ``Mach.dump_weights``
(ref/gen_layer_script.py:1555-1670; generator: tests/golden/
gen_artifact_golden.py): the reader must return exactly the packed images of
the seeded inputs, the writer must reproduce the reference's files byte for
byte, and malformed or foreign artifacts (W8 images, a residual binary point
other than this build's, broken strides, short files, missing wids) must be
refused before anything is uploaded.
"""
import json
import os
import shutil

import numpy as np
import pytest

import oracle as O
from fable5_llm_b200 import artifact as A
from fable5_llm_b200.config import RS_F, Geometry

FIX = os.path.join(os.path.dirname(__file__), "golden", "artifact")


def _inputs():
    z = np.load(os.path.join(FIX, "inputs.npz"))
    mats = []
    for wid, (N, K, g, e, sh) in enumerate(z["shapes"].tolist()):
        qw = {"w4": z[f"w4_{wid}"].astype(np.int64), "m": z[f"m_{wid}"].astype(np.int64), "e": e, "sh": sh}
        if g != 128:
            qw["g"] = g
        mats.append(qw)
    return mats, z["emb"]


def test_reader_returns_the_reference_images():
    mats, emb = _inputs()
    imgs, meta = A.read_weights(os.path.join(FIX, "tiny"))
    assert sorted(imgs) == list(range(len(mats)))
    assert meta["rs_f"] == RS_F and meta["emb_row_bytes"] == 2 * emb.shape[1]
    for wid, qw in enumerate(mats):
        im = imgs[wid]
        g = qw.get("g", 128)
        want, stride = O.pack_ddr_rows(qw["w4"], qw["m"], g)
        assert (im.N, im.K, im.g, im.e, im.sh) == (*qw["w4"].shape, g, qw["e"], qw["sh"])
        assert im.img.shape == (im.N, stride)
        assert im.img.tobytes() == bytes(want)
        w4, m = O.unpack_ddr_rows(im.img, im.N, im.K, g)
        assert np.array_equal(w4, qw["w4"]) and np.array_equal(m, qw["m"])
    got = A.read_embedding(os.path.join(FIX, "tiny"), emb.shape[0], emb.shape[1], meta["emb_row_bytes"])
    assert np.array_equal(got, emb)


def test_writer_reproduces_the_reference_bytes(tmp_path):
    mats, emb = _inputs()
    pre = str(tmp_path / "tiny")
    assert A.write_weights(pre, mats, emb_q=emb, emb_row_bytes=2 * emb.shape[1], rs_f=RS_F) == len(mats)
    for name in sorted(os.listdir(FIX)):
        if name.startswith("tiny") and not name.startswith("tiny8"):
            with open(os.path.join(FIX, name), "rb") as f, open(tmp_path / name, "rb") as g:
                assert f.read() == g.read(), name


def test_w8_artifact_is_refused():
    with pytest.raises(ValueError, match="W8"):
        A.read_weights(os.path.join(FIX, "tiny8"))


def _copy(tmp_path, edit=None, truncate=None):
    for name in os.listdir(FIX):
        if name.startswith("tiny") and not name.startswith("tiny8"):
            shutil.copy(os.path.join(FIX, name), tmp_path / name)
    if edit:
        man = json.load(open(tmp_path / "tiny.weights.json"))
        edit(man)
        json.dump(man, open(tmp_path / "tiny.weights.json", "w"), indent=1)
    if truncate:
        p = tmp_path / truncate
        p.write_bytes(p.read_bytes()[:-64])
    return str(tmp_path / "tiny")


@pytest.mark.parametrize("case", ["stride", "ng", "nbeats", "short", "key", "g"])
def test_malformed_manifest_is_refused(tmp_path, case):
    edits = {"stride": lambda m: m["0"].update(stride=256), "ng": lambda m: m["1"].update(ng=8),
             "nbeats": lambda m: m["2"].update(nbeats=1), "key": lambda m: m.update(extra=1),
             "g": lambda m: m["0"].update(g=32)}
    pre = _copy(tmp_path, edit=edits.get(case), truncate="tiny_w3.bin" if case == "short" else None)
    with pytest.raises(ValueError):
        A.read_weights(pre)


def test_missing_rs_f_reads_as_the_reference_default(tmp_path):
    pre = _copy(tmp_path, edit=lambda m: m.pop("rs_f"))
    _, meta = A.read_weights(pre)
    assert meta["rs_f"] == A.RS_F_MANIFEST_DEFAULT == 8
    mats, _ = _inputs()
    with pytest.raises(ValueError, match="rs_f"):
        A.write_weights(str(tmp_path / "x"), mats)     # this build's RS_F is not the default


def test_wid_plan_at_9b():
    g = Geometry()
    plan = A.wid_plan(g.layer_types)
    assert len(plan) == 249 and plan[-1] == (-1, "head")
    assert plan[:8] == [(0, n) for n in ("in_qkv", "in_z", "in_b", "in_a", "out", "gate", "up", "down")]
    first_attn = [p for p in plan if p[0] == 3]
    assert first_attn == [(3, n) for n in ("q_proj", "k_proj", "v_proj", "o_proj", "gate", "up", "down")]
    sh = A._shapes(g)
    total = sum(((g.vocab, g.H) if n == "head" else sh[n])[0] * O.row_stride(((g.vocab, g.H) if n == "head"
                                                                                 else sh[n])[1])
                for _, n in plan)
    assert total == 4_091_805_696


class _Geom:
    """A small stand-in geometry (every K a multiple of 128)."""
    H, LVD, CONV_DIM, LNH, NQ, HD, NKV, FFN = 128, 128, 256, 4, 1, 128, 1, 256
    vocab = 10
    layer_types = ["linear_attention", "full_attention"]


class _Model:
    def __init__(self):
        self.geom = _Geom()
        self.mats, self.emb, self.vec, self.lnf = [], None, [], None

    slot_of = staticmethod(lambda name: name)

    def upload_qmat(self, layer, slot, im):
        self.mats.append((layer, slot, im.N, im.K, im.e, im.sh, im.img.tobytes()))

    def upload_embedding(self, emb):
        self.emb = emb

    def upload_layer_vectors(self, i, qw):
        self.vec.append(i)

    def upload_final_norm(self, v):
        self.lnf = v


def _small_artifact(tmp_path, rs_f=RS_F, drop_last=False):
    g = _Geom()
    sh = A._shapes(g)
    rng = np.random.default_rng(3)
    plan = A.wid_plan(g.layer_types)
    mats = []
    for wid, (layer, name) in enumerate(plan):
        N, K = (g.vocab, g.H) if name == "head" else sh[name]
        mats.append({"w4": rng.integers(-8, 8, (N, K)), "m": rng.integers(1, 1 << 16, (N, K // 128)),
                     "e": wid - 9, "sh": wid % 13})
    emb = rng.integers(-3000, 3000, (g.vocab, g.H)).astype(np.int16)
    pre = str(tmp_path / "small")
    A.write_weights(pre, mats[:-1] if drop_last else mats, emb_q=emb, emb_row_bytes=2 * g.H, rs_f=rs_f)
    return pre, plan, mats, emb


def test_load_artifact_maps_wids_to_layer_slots(tmp_path):
    pre, plan, mats, emb = _small_artifact(tmp_path)
    m = _Model()
    A.load_artifact(m, pre, layers=[{}, {}], ln_f_q12=np.arange(4))
    assert [(x[0], x[1]) for x in m.mats] == plan
    for x, qw in zip(m.mats, mats):
        want, _ = O.pack_ddr_rows(qw["w4"], qw["m"])
        assert x[2:6] == (*qw["w4"].shape, qw["e"], qw["sh"]) and x[6] == bytes(want)
    assert np.array_equal(m.emb, emb) and m.vec == [0, 1] and m.lnf is not None


def test_load_artifact_refuses_foreign_artifacts(tmp_path):
    pre, *_ = _small_artifact(tmp_path, rs_f=RS_F + 1)
    with pytest.raises(ValueError, match="rs_f"):
        A.load_artifact(_Model(), pre)
    pre, *_ = _small_artifact(tmp_path, drop_last=True)
    with pytest.raises(ValueError, match="wids"):
        A.load_artifact(_Model(), pre)
    m = _Model()
    m.geom.vocab = 11
    pre, *_ = _small_artifact(tmp_path)
    with pytest.raises(ValueError, match="head"):
        A.load_artifact(m, pre)

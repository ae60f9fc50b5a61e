"""GPU parity of the reference-API drop-ins (fable5_llm_b200.w4a8_ref,
fixedpoint, layer_fixed and runner.FxRunner) called the way the
reference's own callers call ref/w4a8_ref.py, ref/fixedpoint.py,
ref/layer_fixed.py and ref/fidelity_check.py:FxRunner: reference-layout
dicts ({"w4","m","e","sh","g"} matrices, layer dicts, cache dicts / lists),
checked bit for bit against the unmodified reference's outputs (committed
fixtures) and the oracle."""
import gc
import hashlib

import numpy as np
import pytest

import oracle as O
from fable5_llm_b200 import fixedpoint as FP
from fable5_llm_b200 import layer_fixed as LF
from fable5_llm_b200 import synth
from fable5_llm_b200 import w4a8_ref as W
from fable5_llm_b200.runner import FxRunner
from oracle.model import OracleModel

pytestmark = pytest.mark.gpu
I64 = np.int64
SEED = 2026


def digest(a):
    return hashlib.sha256(np.ascontiguousarray(np.asarray(a, dtype=I64)).tobytes()).hexdigest()


def ref_dict(qw):
    """An OracleModel layer (QMat matrices) as the reference's layer dict:
    every matrix as {"w4", "m", "e", "sh", "g"} (ref/layer_fixed.py:1111)."""
    out = {}
    for k, v in qw.items():
        if isinstance(v, dict):
            out[k] = ref_dict(v)
        elif isinstance(v, O.QMat):
            out[k] = v.to_dict()
        else:
            out[k] = v
    return out


@pytest.fixture(scope="module")
def om4():
    return OracleModel(SEED, O.Geometry(4, 4096))


@pytest.fixture(autouse=True, scope="module")
def _free_layer_contexts():
    yield
    LF.clear_layer_cache()


@pytest.mark.parametrize("s", [1, 2, 3, 4])
def test_matvec_y32_tb_vectors(golden, s):
    """ref/w4a8_ref.py:254-289 on the reference's own tb/vec_s* vectors,
    called with unpacked w4 / m arrays like the reference's callers."""
    d = golden("tb_matvec")
    K, NG, SH, N, BPR = [int(v) for v in d[f"s{s}_params"]]
    w4, m = W.unpack_ddr_rows(d[f"s{s}_img"].tobytes(), N, K)
    y = W.matvec_y32(w4, m, SH, d[f"s{s}_x8"])
    assert y.dtype == np.int32
    assert np.array_equal(y, d[f"s{s}_y32"])


def test_matvec_y32_overflow_asserts():
    """The reference asserts |y32| < 2^31 (ref/w4a8_ref.py:288)."""
    K = 4096
    w4 = np.full((4, K), -8, dtype=np.int8)
    m = np.full((4, K // 128), 65535, dtype=np.uint16)
    x8 = np.full(K, -127, dtype=np.int8)
    with pytest.raises(AssertionError):
        W.matvec_y32(w4, m, 0, x8)


def test_fixedpoint_vs_reference(golden):
    d = golden("ref_prims")
    for i in range(0, d["dq_x"].shape[0], 7):
        x8, e = FP.dyn_quant_i8(d["dq_x"][i])
        assert np.array_equal(x8.astype(I64), d["dq_x8"][i]) and e == int(d["dq_e"][i])
    for i in range(0, d["rs_v"].size, 37):
        assert FP.rsqrt_q(int(d["rs_v"][i]), int(d["rs_p"][i])) == (int(d["rs_r"][i]), int(d["rs_e"][i]))
        assert FP.recip_q(int(d["rs_v"][i]), int(d["rs_p"][i])) == (int(d["rc_r"][i]), int(d["rc_e"][i]))
    x = np.arange(-(1 << 17), 1 << 17, 97, dtype=I64)
    assert np.array_equal(FP.sigmoid_q(x), O.sigmoid_q(x))
    assert np.array_equal(FP.softplus_q(x), O.softplus_q(x))
    assert np.array_equal(FP.silu_q(x), O.silu_q(x))
    assert np.array_equal(FP.exp_neg_q(-np.abs(x)), O.exp_neg_q(-np.abs(x)))
    assert FP.sigmoid_q(123) == int(O.sigmoid_q(np.array([123]))[0])     # scalar in, int out


def test_matvec_to_and_rmsnorm(om4):
    rng = np.random.default_rng(5)
    x16 = np.clip(np.round(rng.normal(0, 1, 4096) * 128), -32768, 32767).astype(I64)
    qw = om4.layers[0]
    xn = LF.rmsnorm_fx(x16, qw["ln1"], LF.RS_F, True)
    assert np.array_equal(xn, O.rmsnorm_fx(x16, qw["ln1"], O.RS_F, True))
    for name, in_f, out_f in (("gate", LF.RS_F, 12), ("up", LF.RS_F, LF.RS_F)):
        y = LF.matvec_to(qw["mlp"][name].to_dict(), xn, in_f, out_f)
        assert np.array_equal(y, O.matvec_to(qw["mlp"][name], xn, in_f, out_f)), name


@pytest.mark.parametrize("mode", ["float", "eps"])
def test_layer_decode_fx_deltanet(golden, om4, mode):
    """A DeltaNet layer dict with the reference's cache dict: outputs,
    dn_o_shift, the state and the conv window equal the reference's."""
    d = golden("ref_layers")
    LF.SEQ_NORM = mode == "eps"
    try:
        qw = ref_dict(om4.layers[0])
        cache = LF.new_cache_fx(qw["type"])
        for t in range(d["x_in"].shape[0]):
            y = LF.layer_decode_fx(d["x_in"][t], qw, cache, t)
            assert np.array_equal(y, d[f"dn_{mode}_y"][t]), f"step {t}"
            assert cache["dn_o_shift"] == [int(v) for v in d[f"dn_{mode}_k"][t]]
        assert digest(cache["S"]) == str(d[f"dn_{mode}_S_digest"])
        assert np.array_equal(cache["conv"], d[f"dn_{mode}_conv"])
        LF.release_layer(qw)
    finally:
        LF.SEQ_NORM = False


def test_layer_decode_fx_attention(golden, om4):
    """An attention layer dict with the reference's list cache (pos != T)."""
    d = golden("ref_layers")
    qw = ref_dict(om4.layers[3])
    cache = LF.new_cache_fx(qw["type"])
    n = d["x_in"].shape[0]
    for t in range(n):
        y = LF.layer_decode_fx(d["x_in"][t], qw, cache, t + 5)
        assert np.array_equal(y, d["attn_y"][t]), f"step {t}"
        assert cache["attn_o_shift"] == int(d["attn_ka"][t])
    assert len(cache["k"]) == n and len(cache["v"]) == n
    for t in range(n):
        for h in range(4):
            k8, ke = cache["k"][t][h]
            v8, ve = cache["v"][t][h]
            assert np.array_equal(k8.astype(I64), d["attn_k8"][t][h]) and ke == d["attn_ke"][t][h]
            assert np.array_equal(v8.astype(I64), d["attn_v8"][t][h]) and ve == d["attn_ve"][t][h]


def test_layer_context_cache_never_serves_old_weights():
    """layer_decode_fx keeps a GPU context per layer dict.  Dicts created
    and freed in a loop (their ids may be reused) must each run with their
    own weights, and replacing a matrix inside a live dict must be seen."""
    geom = O.Geometry(4, 4096)
    x = synth.emb_rows(SEED, [77], 4096)[0].astype(I64)
    for seed in (11, 12, 13):
        om = OracleModel(seed, geom)
        qw = ref_dict(om.layers[1])
        cache = LF.new_cache_fx(qw["type"])
        y = LF.layer_decode_fx(x, qw, cache, 0)
        ref = O.layer_decode_fx(x, om.layers[1], O.DNCache(geom), 0, geom)
        assert np.array_equal(y, ref), f"seed {seed}"
        del qw, cache, om
        gc.collect()
    # a matrix replaced inside a live dict
    a, b = OracleModel(21, geom), OracleModel(22, geom)
    qw = ref_dict(a.layers[1])
    LF.layer_decode_fx(x, qw, LF.new_cache_fx(qw["type"]), 0)
    qw["mlp"]["down"] = b.layers[1]["mlp"]["down"].to_dict()
    mixed = dict(a.layers[1])
    mixed["mlp"] = dict(a.layers[1]["mlp"])
    mixed["mlp"]["down"] = b.layers[1]["mlp"]["down"]
    y = LF.layer_decode_fx(x, qw, LF.new_cache_fx(qw["type"]), 0)
    assert np.array_equal(y, O.layer_decode_fx(x, mixed, O.DNCache(geom), 0, geom))
    assert len(LF._CTX) <= LF.MAX_LAYER_CTX


def test_fxrunner_vs_reference(golden, om4):
    """FxRunner built from reference-layout dicts (the upload path a real
    reference caller takes) matches the reference's FxRunner-sequence run:
    every argmax token, max logit and layer output; resid_max / resid_clip
    equal the reference's counters over the same run; caches come back in
    the reference layout and equal the oracle's."""
    d = golden("ref_model4")
    g = O.Geometry(4, 4096)
    layers = [ref_dict(qw) for qw in om4.layers]
    emb = synth.emb_rows(SEED, range(g.vocab), g.H)
    r = FxRunner(layers, g.layer_types, emb, om4.head.to_dict(), om4.ln_f_q12, max_T=64)
    orr = O.OracleRunner(om4, max_T=64)
    for t, tok in enumerate(d["m4_in"]):
        y = r.step(int(tok), t)
        assert y.dtype == np.int64 and y.shape == (g.vocab,)
        assert int(np.argmax(y)) == int(d["m4_out"][t]) and int(y.max()) == int(d["m4_ymax"][t])
        orr.step(int(tok), t)
    x = d["m4_layer_x"].astype(I64)
    assert r.resid_max == int(np.abs(x).max()) == orr.resid_max
    assert r.resid_clip == int(((x >= 32767) | (x <= -32768)).sum()) == orr.resid_clip
    caches = r.caches
    T = len(d["m4_in"])
    for i, lt in enumerate(g.layer_types):
        c = orr.caches[i]
        if lt == "full_attention":
            assert len(caches[i]["k"]) == T
            for t in range(T):
                for h in range(4):
                    assert np.array_equal(caches[i]["k"][t][h][0], c.k8[h, t]) and caches[i]["k"][t][h][1] == c.ke[h, t]
                    assert np.array_equal(caches[i]["v"][t][h][0], c.v8[h, t]) and caches[i]["v"][t][h][1] == c.ve[h, t]
        else:
            assert np.array_equal(caches[i]["S"], c.S) and np.array_equal(caches[i]["conv"], c.conv)
    r.reset()
    assert r.resid_max == 0 and r.resid_clip == 0
    y = r.step(int(d["m4_in"][0]), 0)
    assert int(np.argmax(y)) == int(d["m4_out"][0])
    r.model.close()


def test_state_images_reference_layout(om4):
    """f5_state_save / f5_state_load images are the reference cache layout:
    after a few steps they equal the oracle's caches byte for byte, and a
    context loaded from them continues identically."""
    from fable5_llm_b200.model import DecodeModel
    from fable5_llm_b200.config import Geometry
    g = O.Geometry(4, 4096)
    m = DecodeModel(Geometry(4, 4096), max_T=64)
    m.load_synthetic(SEED)
    m.reset()
    orr = O.OracleRunner(om4, max_T=64)
    tok = 33
    for t in range(5):
        tok, _ = m.decode_step(tok, t)
        orr.step(33 if t == 0 else prev, t)
        prev = tok
    imgs = [m.state_image(i) for i in range(4)]
    for i, lt in enumerate(g.layer_types):
        c = orr.caches[i]
        if lt == "full_attention":
            T = 5
            ref = np.concatenate([c.k8[:, :T].transpose(1, 0, 2).reshape(-1), c.ke[:, :T].T.reshape(-1),
                                  c.v8[:, :T].transpose(1, 0, 2).reshape(-1), c.ve[:, :T].T.reshape(-1)])
            assert np.array_equal(imgs[i].view(np.int8), ref.astype(np.int8))
        else:
            ref = np.concatenate([c.S.astype(np.int16).reshape(-1).view(np.uint8),
                                  c.conv.astype(I64).reshape(-1).view(np.uint8)])
            assert np.array_equal(imgs[i], ref)
    nxt = m.decode_step(tok, 5)
    m.reset()
    for i in range(4):
        m.load_state_image(i, imgs[i], 5)
    m.set_position(5, 5)
    assert m.decode_step(tok, 5) == nxt
    m.close()

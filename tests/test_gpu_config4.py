"""Config 4 as specified: the full 32-layer 9B model (24 DeltaNet + 8
attention layers, 248,320-row LM head) at context 2048 decoding 64 greedy
tokens, every token, logit vector, final residual and every layer's state
compared with the oracle; and the same model's first steps from context 0
against the unmodified reference's own FxRunner-sequence run
(tests/golden/ref_model32.npz: tokens, max logits and all 32 layer outputs).

The context is filled on the GPU (2048 seeded random ids, one bit-exact step
each -- the reference would need ~69 h for it), then the oracle loads that
state, and both continue greedily."""
import os

import numpy as np
import pytest

import oracle as O
from fable5_llm_b200 import _lib as L
from fable5_llm_b200 import synth
from fable5_llm_b200.config import Geometry
from fable5_llm_b200.model import DecodeModel
from oracle.model import OracleModel

pytestmark = [pytest.mark.gpu, pytest.mark.slow]
I64 = np.int64
SEED = 2026
GOLDEN = os.path.join(os.path.dirname(os.path.abspath(__file__)), "golden")


@pytest.fixture(scope="module")
def oracle9b():
    return OracleModel(SEED, O.GEOM_9B)


def _load_gpu_state_into(r, m, T):
    for i, lt in enumerate(m.geom.layer_types):
        c = r.caches[i]
        if lt == "full_attention":
            for nm, buf in (("k8", L.BUF_K8), ("ke", L.BUF_KE), ("v8", L.BUF_V8), ("ve", L.BUF_VE)):
                getattr(c, nm)[...] = m.read(buf, i).reshape(getattr(c, nm).shape)
            c.T = T
        else:
            st = m.get_dn_state(i, T)
            c.conv[...] = st["conv"]
            c.S[...] = st["S"]


def _compare_all_state(m, r, T, t_lo):
    """Every DeltaNet layer's S and conv window; every attention layer's
    K/V rows and exponents from t_lo to T."""
    for i, lt in enumerate(m.geom.layer_types):
        c = r.caches[i]
        if lt == "full_attention":
            assert c.T == T
            for nm, buf in (("k8", L.BUF_K8), ("ke", L.BUF_KE), ("v8", L.BUF_V8), ("ve", L.BUF_VE)):
                g = m.read(buf, i).reshape(getattr(c, nm).shape)
                assert np.array_equal(g[:, t_lo:T], getattr(c, nm)[:, t_lo:T]), f"layer {i} {nm}"
        else:
            st = m.get_dn_state(i, T)
            assert np.array_equal(st["S"], c.S), f"layer {i} S"
            assert np.array_equal(st["conv"], c.conv), f"layer {i} conv"


def test_config4_context2048_64_tokens(oracle9b):
    T0, n = 2048, 64
    m = DecodeModel(Geometry(), max_T=T0 + n + 16, max_pos=T0 + n + 16)
    m.load_synthetic(SEED)
    m.reset()
    prompt = np.random.default_rng(SEED).integers(0, m.geom.vocab, T0)
    m.prefill(prompt)
    tok, mv = m.sync()
    assert m.position() == (T0, T0)
    r = O.OracleRunner(oracle9b, max_T=T0 + n + 16)
    _load_gpu_state_into(r, m, T0)
    m.set_logits(True)
    # the prompt's last step is redone by neither side: both continue from
    # the GPU's argmax after the prompt
    st0 = m.stats()
    for k in range(n):
        t = T0 + k
        nt, mv = m.decode_step(tok, t)
        ref_tok, y = r.step(tok, t)
        assert np.array_equal(m.logits(), y), f"step {t}: logits"
        assert nt == ref_tok and mv == int(y.max()), f"step {t}: token {nt} != {ref_tok}"
        assert np.array_equal(m.read(L.BUF_X16).astype(I64), r.layer_out[-1]), f"step {t}: residual"
        if k in (0, n // 2, n - 1):
            _compare_all_state(m, r, t + 1, T0)
        tok = nt
    st1 = m.stats()
    # the saturation counters over the 64 compared steps equal the oracle's
    assert st1["resid_clip"] - st0["resid_clip"] == r.resid_clip
    assert st1["resid_max"] >= r.resid_max
    m.close()


@pytest.mark.skipif(not os.path.exists(os.path.join(GOLDEN, "ref_model32.npz")), reason="no ref_model32 fixture")
def test_full_9b_vs_reference_fixture(golden):
    """The unmodified reference's 32-layer run from context 0: every emitted
    token and max logit (persistent engine), and every layer's output (one
    layer at a time through f5_layer_step, the layer_decode_fx entry)."""
    d = golden("ref_model32")
    m = DecodeModel(Geometry(), max_T=64)
    m.load_synthetic(SEED)
    m.reset()
    for t, tok in enumerate(d["m32_in"]):
        nt, mv = m.decode_step(int(tok), t)
        assert nt == int(d["m32_out"][t]) and mv == int(d["m32_ymax"][t]), f"step {t}"
        assert np.array_equal(m.read(L.BUF_X16), d["m32_layer_x"][t][-1]), f"step {t}: residual"
    stats = m.stats()
    x = d["m32_layer_x"].astype(I64)
    assert stats["resid_max"] == int(np.abs(x).max())
    assert stats["resid_clip"] == int(((x >= 32767) | (x <= -32768)).sum())
    m.reset()
    for t, tok in enumerate(d["m32_in"]):
        x16 = synth.emb_rows(SEED, [int(tok)], 4096)[0]
        for i in range(32):
            x16 = m.layer_step(i, x16, t, t)
            assert np.array_equal(x16, d["m32_layer_x"][t][i].astype(I64)), f"step {t} layer {i}"
    m.close()

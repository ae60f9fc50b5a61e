"""GPU decode-step parity: single layers, the reduced model and the full
32-layer 9B model against the unmodified reference's outputs (fixtures) and
the oracle, bit-exact in every token, logit and state word."""
import hashlib

import numpy as np
import pytest

import oracle as O
from fable5_llm_b200 import _lib as L
from fable5_llm_b200.config import Geometry
from fable5_llm_b200.model import DecodeModel
from oracle.model import OracleModel

pytestmark = pytest.mark.gpu
I64 = np.int64
SEED = 2026


def digest(a):
    return hashlib.sha256(np.ascontiguousarray(np.asarray(a, dtype=I64)).tobytes()).hexdigest()


@pytest.fixture(scope="module")
def model4():
    m = DecodeModel(Geometry(4, 4096), max_T=128)
    m.load_synthetic(SEED)
    return m


@pytest.fixture(params=["persistent", "graph"])
def engine(request):
    """Both decode engines (one persistent cooperative launch per step, or
    the per-op kernel chain as a CUDA graph) must be bit-exact."""
    return request.param


@pytest.fixture(scope="module")
def model4_eps():
    m = DecodeModel(Geometry(4, 4096), max_T=128, norm_mode="eps")
    m.load_synthetic(SEED)
    return m


@pytest.mark.parametrize("mode", ["float", "eps"])
def test_dn_layer_vs_reference(golden, model4, model4_eps, mode):
    d = golden("ref_layers")
    m = model4 if mode == "float" else model4_eps
    m.reset()
    for t in range(d["x_in"].shape[0]):
        y = m.layer_step(0, d["x_in"][t], t, t)
        assert np.array_equal(y, d[f"dn_{mode}_y"][t]), f"step {t}"
        assert np.array_equal(m.read(L.BUF_DN_KH, 0).astype(I64), d[f"dn_{mode}_k"][t])
    T = d["x_in"].shape[0]
    st = m.get_dn_state(0, T)
    assert digest(st["S"]) == str(d[f"dn_{mode}_S_digest"])
    assert np.array_equal(st["conv"], d[f"dn_{mode}_conv"])
    assert m.stats()["dn_sat"] == int(d[f"dn_{mode}_sat"])   # the reference's state["sat"]


def test_attn_layer_vs_reference(golden, model4):
    d = golden("ref_layers")
    m = model4
    m.reset()
    n = d["x_in"].shape[0]
    for t in range(n):
        y = m.layer_step(3, d["x_in"][t], t, t + 5)
        assert np.array_equal(y, d["attn_y"][t]), f"step {t}"
        assert int(m.read(L.BUF_KA, 3)[0]) == int(d["attn_ka"][t])
    kv = m.get_kv(3, n)
    for t in range(n):
        for h in range(4):
            assert np.array_equal(kv["k"][t][h][0].astype(I64), d["attn_k8"][t][h])
            assert kv["k"][t][h][1] == d["attn_ke"][t][h]
            assert np.array_equal(kv["v"][t][h][0].astype(I64), d["attn_v8"][t][h])
            assert kv["v"][t][h][1] == d["attn_ve"][t][h]


def test_default_engine_is_persistent(model4):
    assert model4.engine() == "persistent"


def test_model4_vs_reference(golden, model4, engine):
    """The reduced model (3 DeltaNet + 1 attention layer, 4096-row head):
    every emitted token, max logit and the final residual equal the
    reference's FxRunner-sequence run."""
    d = golden("ref_model4")
    m = model4
    m.set_engine(engine)
    m.reset()
    for t, tok in enumerate(d["m4_in"]):
        nt, mv = m.decode_step(int(tok), t)
        assert nt == int(d["m4_out"][t]), f"step {t}: token {nt} != {int(d['m4_out'][t])}"
        assert mv == int(d["m4_ymax"][t])
        assert np.array_equal(m.read(L.BUF_X16).astype(I64), d["m4_layer_x"][t][-1].astype(I64))


def _compare_states(m, r, T):
    for i, lt in enumerate(m.geom.layer_types):
        c = r.caches[i]
        if lt == "full_attention":
            kv = m.get_kv(i, T)
            assert c.T == T
            for t in (0, T // 2, T - 1):
                for h in range(4):
                    assert np.array_equal(kv["k"][t][h][0], c.k8[h, t]) and kv["k"][t][h][1] == c.ke[h, t]
                    assert np.array_equal(kv["v"][t][h][0], c.v8[h, t]) and kv["v"][t][h][1] == c.ve[h, t]
        else:
            st = m.get_dn_state(i, T)
            assert np.array_equal(st["S"], c.S), f"layer {i} S"
            assert np.array_equal(st["conv"], c.conv), f"layer {i} conv"


@pytest.mark.parametrize("mode", ["float", "eps"])
def test_model4_vs_oracle_logits_and_state(model4, model4_eps, mode, engine):
    m = model4 if mode == "float" else model4_eps
    m.set_engine(engine)
    m.reset()
    m.set_logits(True)
    g = m.geom
    r = O.OracleRunner(OracleModel(SEED, O.Geometry(4, 4096)), max_T=128, norm_mode=mode)
    toks = [5, 4095, 77, 1000, 3, 3, 2048]
    for t, tok in enumerate(toks):
        nt, mv = m.decode_step(tok, t)
        ref_tok, y = r.step(tok, t)
        assert np.array_equal(m.logits(), y)
        assert nt == ref_tok and mv == int(y.max())
    _compare_states(m, r, len(toks))
    m.set_logits(False)


def test_greedy_device_loop_matches_host_steps(model4, engine):
    """f5_decode_launch (tokens fed back on the device) == host-fed steps."""
    m = model4
    m.set_engine(engine)
    m.reset()
    toks, tok = [], 17
    for t in range(6):
        tok, _ = m.decode_step(tok, t)
        toks.append(tok)
    m.reset()
    m.decode_step(17, 0)
    m.decode_launch(5)
    last, _ = m.sync()
    assert last == toks[-1]
    assert m.position() == (6, 6)


def test_traced_step_is_a_greedy_step(model4):
    """The traced instance of the persistent kernel (f5_ctx_trace_step, the
    same source with its marks compiled in) runs the same greedy step as the
    step kernel, and every CTA's op marks are present and ordered."""
    m = model4
    m.set_engine("persistent")
    m.reset()
    toks, tok = [], 17
    for t in range(6):
        tok, _ = m.decode_step(tok, t)
        toks.append(tok)
    m.reset()
    m.decode_step(17, 0)
    t, kinds = m.trace_step()
    m.decode_launch(4)
    last, _ = m.sync()
    assert last == toks[-1]
    assert m.position() == (6, 6)
    assert t.shape[1] == len(kinds)
    assert (t[:, :, 0] >= 0).all() and (t[:, :, 1] >= t[:, :, 0]).all()


def test_state_save_load_roundtrip(model4, tmp_path):
    m = model4
    m.reset()
    tok = 9
    for t in range(5):
        tok, _ = m.decode_step(tok, t)
    p = str(tmp_path / "st.npz")
    m.save_state(p, 5)
    ref_next = m.decode_step(tok, 5)
    m.reset()
    assert m.load_state(p) == 5
    assert m.decode_step(tok, 5) == ref_next


def test_attention_long_context_vs_oracle(model4, engine):
    """Context 2048: the GPU fills the caches (bit-exact step by step), the
    oracle loads that state and both decode further steps."""
    m = model4
    T = 2048
    big = DecodeModel(Geometry(4, 4096), max_T=T + 8)
    big.set_engine(engine)
    big.load_synthetic(SEED)
    big.reset()
    rng = np.random.default_rng(7)
    prompt = rng.integers(0, 4096, T)
    big.decode_step(int(prompt[0]), 0)
    for t in range(1, T):
        big.decode_step(int(prompt[t]), t)
    r = O.OracleRunner(OracleModel(SEED, O.Geometry(4, 4096)), max_T=big.max_T)
    for i, lt in enumerate(big.geom.layer_types):
        if lt == "full_attention":
            c = r.caches[i]
            for nm, buf in (("k8", L.BUF_K8), ("ke", L.BUF_KE), ("v8", L.BUF_V8), ("ve", L.BUF_VE)):
                a = big.read(buf, i)
                getattr(c, nm)[...] = a.reshape(getattr(c, nm).shape)
            c.T = T
        else:
            st = big.get_dn_state(i, T)
            r.caches[i].conv[...] = st["conv"]
            r.caches[i].S[...] = st["S"]
    big.set_logits(True)
    tok = 123
    for t in range(T, T + 3):
        nt, _ = big.decode_step(tok, t)
        ref_tok, y = r.step(tok, t)
        assert np.array_equal(big.logits(), y), f"step {t}"
        assert nt == ref_tok
        tok = nt
    big.close()
    del m


@pytest.mark.parametrize("T0", [4990, 6100])
def test_attention_random_cache_multi_fill_vs_oracle(T0):
    """Random int8 K/V caches at context ~5k-6k: each persistent CTA's token
    chunk spans several 64-row shared-memory fills; both engines and the
    oracle decode from the same state."""
    geom = Geometry(4, 4096)
    rng = np.random.default_rng(T0)
    big = DecodeModel(geom, max_T=6144)
    big.load_synthetic(SEED)
    r = O.OracleRunner(OracleModel(SEED, O.Geometry(4, 4096)), max_T=big.max_T)
    for i, lt in enumerate(geom.layer_types):
        if lt == "full_attention":
            c = r.caches[i]
            c.k8[...] = rng.integers(-127, 128, c.k8.shape)
            c.v8[...] = rng.integers(-127, 128, c.v8.shape)
            c.ke[...] = rng.integers(-8, 1, c.ke.shape)
            c.ve[...] = rng.integers(-8, 1, c.ve.shape)
            c.T = T0
    outs = {}
    for eng in ("persistent", "graph"):
        big.set_engine(eng)
        big.reset()
        for i, lt in enumerate(geom.layer_types):
            if lt == "full_attention":
                c = r.caches[i]
                for nm, buf in (("k8", L.BUF_K8), ("ke", L.BUF_KE), ("v8", L.BUF_V8), ("ve", L.BUF_VE)):
                    big.write(buf, i, np.ascontiguousarray(getattr(c, nm), dtype=np.int8))
        big.set_position(T0, T0)
        big.set_logits(True)
        res = []
        tok = 321
        for t in range(T0, T0 + 2):
            nt, _ = big.decode_step(tok, t)
            res.append((nt, big.logits().copy()))
            tok = nt
        outs[eng] = res
    tok = 321
    for k, t in enumerate(range(T0, T0 + 2)):
        ref_tok, y = r.step(tok, t)
        for eng in outs:
            assert np.array_equal(outs[eng][k][1], y), f"{eng} step {t}"
            assert outs[eng][k][0] == ref_tok
        tok = ref_tok
    big.close()


@pytest.mark.slow
def test_full_9b_vs_oracle():
    """The full 32-layer 9B model with the 248,320-row head: tokens, logits
    and every layer's state after several steps, in both engines."""
    m = DecodeModel(Geometry(), max_T=64)
    m.load_synthetic(SEED)
    m.set_logits(True)
    r = O.OracleRunner(OracleModel(SEED, O.GEOM_9B), max_T=64)
    ref = []
    tok = 1234
    for t in range(3):
        ref_tok, y = r.step(tok, t)
        ref.append((tok, ref_tok, y))
        tok = ref_tok
    for eng in ("persistent", "graph"):
        m.set_engine(eng)
        m.reset()
        for t, (tok, ref_tok, y) in enumerate(ref):
            nt, mv = m.decode_step(tok, t)
            assert np.array_equal(m.logits(), y), f"{eng} step {t}"
            assert nt == ref_tok and mv == int(y.max())
        _compare_states(m, r, 3)
    m.close()


def test_prefill_matches_host_steps(model4, engine):
    """A device-fed prompt (f5_decode_prefill) leaves the same state, logit
    and next token as the same tokens fed one host step at a time, and the
    greedy continuation from it is the same."""
    m = model4
    m.set_engine(engine)
    toks = [17, 901, 4000, 3, 17, 256, 9]
    m.reset()
    for t, tok in enumerate(toks):
        nt, mv = m.decode_step(tok, t)
    x_ref = m.read(L.BUF_X16)
    m.decode_launch(3)
    cont_ref = m.sync()
    m.reset()
    m.prefill(toks)
    assert m.sync() == (nt, mv)
    assert np.array_equal(m.read(L.BUF_X16), x_ref)
    assert m.position() == (len(toks), len(toks))
    m.decode_launch(3)
    assert m.sync() == cont_ref

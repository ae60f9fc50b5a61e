"""Layer-major prompt prefill (f5_bctx_prefill) against sequential decode
steps of the single-sequence engine, which is pinned to the reference: the
argmax after the prompt, its y32 logit and every state word (DeltaNet
states, conv windows, block-float shifts, K/V rows and exponents) are
bit-identical, other sequences of the batch are untouched, and decoding
continues identically afterwards."""
import numpy as np
import pytest

from fable5_llm_b200 import _lib as L
from fable5_llm_b200.batch import BatchModel
from fable5_llm_b200.config import Geometry
from fable5_llm_b200.model import DecodeModel

pytestmark = pytest.mark.gpu
SEED = 2026


def states(read, geom, T):
    st = {}
    for i, lt in enumerate(geom.layer_types):
        if lt == "full_attention":
            for b in (L.BUF_K8, L.BUF_V8):
                st[(i, b)] = read(b, i).reshape(geom.NKV, -1, geom.HD)[:, :T]
            for b in (L.BUF_KE, L.BUF_VE):
                st[(i, b)] = read(b, i).reshape(geom.NKV, -1)[:, :T]
        else:
            for b in (L.BUF_DN_S, L.BUF_DN_CONV, L.BUF_DN_KH):
                st[(i, b)] = read(b, i)
    return st


def run_decode(m, toks, T0=0):
    m.reset()
    m.set_position(T0, T0)
    out = None
    for t, tok in enumerate(toks):
        out = m.decode_step(int(tok), T0 + t)
    return out


@pytest.mark.parametrize("B,n,seq", [(16, 40, 3), (8, 5, 0), (32, 64, 31)])
def test_prefill_matches_decode_steps(B, n, seq):
    m = DecodeModel(Geometry(4, 4096), max_T=128)
    m.load_synthetic(SEED)
    rng = np.random.default_rng(n + B)
    prompt = rng.integers(0, m.geom.vocab, n)
    ref = run_decode(m, prompt)
    s_ref = states(lambda w, i: m.read(w, i), m.geom, n)
    bm = BatchModel(m, B, max_T=128)
    bm.reset()
    got = bm.prefill(seq, prompt)
    assert got == ref, "argmax after the prompt"
    assert bm.position(seq) == (n, n)
    s_got = states(lambda w, i: bm.read(seq, w, i), m.geom, n)
    for k in s_ref:
        assert np.array_equal(s_ref[k], s_got[k]), f"state {k}"
    other = (seq + 1) % B
    assert bm.position(other) == (0, 0)
    for k, v in states(lambda w, i: bm.read(other, w, i), m.geom, 1).items():
        assert not np.any(v), f"sequence {other} touched: {k}"
    # the next step of the prefilled sequence continues the decode run
    toks = np.zeros(B, dtype=np.int32)
    toks[seq] = got[0]
    nt, mv = bm.step(toks)
    assert (int(nt[seq]), int(mv[seq])) == m.decode_step(int(got[0]), n)
    bm.close()
    m.close()


def test_prefill_after_context_and_refusals():
    """A second prompt appended to an existing context; out-of-range input."""
    m = DecodeModel(Geometry(4, 4096), max_T=96)
    m.load_synthetic(SEED)
    rng = np.random.default_rng(5)
    a, b = rng.integers(0, m.geom.vocab, 20), rng.integers(0, m.geom.vocab, 23)
    ref = run_decode(m, np.concatenate([a, b]))
    bm = BatchModel(m, 16, max_T=96)
    bm.reset()
    bm.prefill(2, a)
    assert bm.prefill(2, b) == ref
    s_ref = states(lambda w, i: m.read(w, i), m.geom, 43)
    s_got = states(lambda w, i: bm.read(2, w, i), m.geom, 43)
    for k in s_ref:
        assert np.array_equal(s_ref[k], s_got[k]), f"state {k}"
    with pytest.raises(L.F5Error):
        bm.prefill(2, [m.geom.vocab])
    with pytest.raises(L.F5Error):
        bm.prefill(2, rng.integers(0, m.geom.vocab, 60))   # 43 + 60 > max_T
    bm.close()
    m.close()


@pytest.mark.slow
def test_prefill_full_9b():
    """The 32-layer 9B model: a 100-token prompt prefilled in chunks of 64."""
    m = DecodeModel(Geometry(), max_T=128)
    m.load_synthetic(SEED)
    prompt = np.random.default_rng(9).integers(0, m.geom.vocab, 100)
    ref = run_decode(m, prompt)
    s_ref = states(lambda w, i: m.read(w, i), m.geom, 100)
    bm = BatchModel(m, 64, max_T=128)
    bm.reset()
    assert bm.prefill(0, prompt) == ref
    s_got = states(lambda w, i: bm.read(0, w, i), m.geom, 100)
    for k in s_ref:
        assert np.array_equal(s_ref[k], s_got[k]), f"state {k}"
    bm.close()
    m.close()

"""TOPK-32 capture on the GPU (f5_topk32_*, f5_ctx_topk) against the
reference's own cases and the oracle restatement, bit-exact in the list,
the count, both sticky overflow flags and the AMAX32 winner."""
import numpy as np
import pytest

import oracle as O
from oracle import topk as OT
from fable5_llm_b200 import sampling as S
from fable5_llm_b200 import synth
from fable5_llm_b200.config import RS_F, Geometry
from fable5_llm_b200.model import DecodeModel

pytestmark = pytest.mark.gpu
SEED = 2026


def check(r, exp, mask=None):
    idx = r.indices if mask is None else (r.indices & mask)
    assert r.count == exp["count"]
    assert np.array_equal(r.values, exp["val"])
    assert np.array_equal(idx, exp["idx"])
    assert (r.ovf_lit, r.ovf_disp) == (exp["ovf_lit"], exp["ovf_disp"])
    am = r.amax_idx if mask is None else r.amax_idx & mask
    assert (am, r.amax_val) == (exp["amax_idx"], exp["amax_val"])


def test_reference_cases(golden):
    """The 19 cases of tb/scripts/gen_topk_cases.py: the GPU scans the
    elements pushed since the last fresh command (its index = position; the
    unit's 18-bit counter is the position modulo 2^18)."""
    d = golden("topk_cases")
    for i, name in enumerate(d["names"]):
        seq = OT.flatten_after_fresh(d[f"{i}_elems"], [tuple(int(x) for x in c) for c in d[f"{i}_cmds"]])
        meta = [int(x) for x in d[f"{i}_meta"]]
        exp = {"count": meta[0], "val": d[f"{i}_val"], "idx": d[f"{i}_idx"], "ovf_lit": meta[1],
               "ovf_disp": meta[2], "amax_idx": meta[3], "amax_val": meta[4]}
        r = S.topk32(seq)
        assert r.n == seq.size, name
        check(r, exp, mask=OT.IDXM)


def _arrays():
    rng = np.random.default_rng(7)
    n = 248320   # the LM head's rows
    yield "empty", np.zeros(0, np.int32)
    for k in (1, 31, 32, 33, 2047, 2048, 2049, 4097):
        yield f"rand{k}", rng.integers(-2**31, 2**31, size=k, dtype=np.int64).astype(np.int32)
    yield "head_rand", rng.integers(-2**31, 2**31, size=n, dtype=np.int64).astype(np.int32)
    yield "head_logits", np.round(rng.normal(0, 2**20, size=n)).astype(np.int32)
    yield "head_alphabet", rng.choice(rng.integers(-2**31, 2**31, size=7), size=n).astype(np.int32)
    yield "ascending", np.arange(-n // 2, n - n // 2, dtype=np.int32)
    yield "descending", np.arange(n, 0, -1, dtype=np.int32)
    yield "constant", np.full(n, 12345, np.int32)
    rails = rng.integers(-1000, 1000, size=n).astype(np.int32)
    rails[rng.choice(n, 40, replace=False)] = 2**31 - 1
    rails[rng.choice(n, 40, replace=False)] = -2**31
    yield "rails", rails
    # the boundary value repeats late in the scan, after the list filled
    late = rng.integers(0, 1000, size=n).astype(np.int32)
    late[1000:1040] = 5000
    late[200000:200010] = 5000
    yield "late_ties", late


@pytest.mark.parametrize("name,vals", list(_arrays()), ids=[a for a, _ in _arrays()])
def test_against_oracle(name, vals):
    exp = OT.topk32(vals)
    check(S.topk32(vals), exp)


def test_decode_step_topk_and_sampling(golden):
    """On the reduced model: after each step the capture's entry 0 is the
    emitted greedy token, every entry is that row's logit, the list equals
    the oracle's over the stored logits, and e_x is the DYNQ8 exponent of
    rmsnorm_fx(final residual, ln_f) (the reference's head prologue)."""
    d = golden("ref_model4")
    g = Geometry(4, 4096)
    m = DecodeModel(g, max_T=128)
    m.load_synthetic(SEED)
    _, ln_f = synth.vector_params(SEED, g)
    m.set_logits(True)
    m.reset()
    for t, tok in enumerate(d["m4_in"]):
        nt, mv = m.decode_step(int(tok), t)
        r = m.topk()
        lg = m.logits()
        assert r.indices[0] == nt and r.values[0] == mv
        assert np.array_equal(r.values, lg[r.indices].astype(np.int64))
        check(r, OT.topk32(lg))
        x = d["m4_layer_x"][t][-1].astype(np.int64)
        _, e_x = O.dyn_quant_i8(O.rmsnorm_fx(x, ln_f, RS_F, False))
        assert r.e_x == e_x
    # a seeded sampled continuation is reproducible and draws from the list
    toks = []
    for rep in range(2):
        m.reset()
        s = S.Sampler(temp=0.9, top_k=16, seed=99, logit_exp0=m.head_logit_exp0())
        tok, seq = 17, []
        for t in range(4):
            tok, info = m.sample_step(tok, t, s)
            assert info["mode"] == "sampled" and tok in m.topk().indices[:16]
            seq.append(tok)
        toks.append(seq)
    assert toks[0] == toks[1]

"""SEQ artifact reader, state-region layout and the seed restatement of the
reference generator's model, on the CPU, against the unmodified reference's
9B token-stream run (tests/golden/seq9b: its stream, blob, metadata and
weight manifest; tests/golden/seq9b_ref.npz: its tokens, vectors and
digests; both made by tests/golden/gen_seq_golden.py, whose run also passed
the reference's own SEQ gate)."""
import hashlib
import os
import sys

import numpy as np
import pytest

from fable5_llm_b200 import quant as Q
from fable5_llm_b200.seq_harness import SeqHarness, layer_types_of
from fable5_llm_b200.seq_stream import (OP_MVGO, SeqArtifact, SeqFormatError, decode_mvgo,
                                        unpack_stream)
from fable5_llm_b200.seq_weights import DDRWeights
from fable5_llm_b200.state_region import StateRegion, slots

HERE = os.path.dirname(os.path.abspath(__file__))
PREFIX = os.path.join(HERE, "golden", "seq9b", "tok9")
sys.path.insert(0, os.path.join(HERE, "golden"))
import seq_model_gen as GEN  # noqa: E402

# (stream name, reference fixture) of every committed SEQ artifact
ARTIFACTS = [(n, f) for n, f in (("tok9", "seq9b_ref"), ("tok9l4", "tok9l4_ref"))
             if os.path.exists(os.path.join(HERE, "golden", "seq9b", n + ".seq"))]


def ref_layers(d, types):
    """The reference's per-layer vectors from a fixture, as layer dicts."""
    out = []
    for i, lt in enumerate(types):
        qw = {"ln1": d[f"l{i}_ln1"], "ln2": d[f"l{i}_ln2"], "type": lt}
        if lt == "full_attention":
            qw["attn"] = {"q_norm": d[f"l{i}_q_norm"], "k_norm": d[f"l{i}_k_norm"]}
        else:
            qw["dn"] = {"dt_bias_q12": d[f"l{i}_dt_bias_q12"], "A_q15": d[f"l{i}_A_q15"],
                        "norm_w_q14": d[f"l{i}_norm_w_q14"], "conv_w": d[f"l{i}_conv_w"]}
        out.append(qw)
    return out


@pytest.fixture(scope="module")
def art():
    return SeqArtifact.load(PREFIX)


def test_stream_reads_and_matches_its_metadata(art):
    assert art.histogram() == art.meta["opcode_histogram"]
    assert len(art.recs) == art.meta["nrec"] == 1965
    assert art.profile == "epsnorm" and art.meta["loop_structurally_safe"]
    assert art.prompt == [5983] and art.expect_tokens == [2380, 6362, 5836]


def test_stream_checksums_refuse_corruption(art):
    bad = bytearray(art.stream)
    bad[100] ^= 1
    with pytest.raises(SeqFormatError):
        SeqArtifact(art.meta, bytes(bad), art.blob)
    with pytest.raises(SeqFormatError):
        SeqArtifact(art.meta, art.stream, art.blob[:-2])
    with pytest.raises(SeqFormatError):
        unpack_stream(art.stream[:-3])


def test_every_mvgo_resolves_against_the_plan(art):
    mv = art.check_mvgo_plan()
    assert len(mv) == 50
    plan = art.weight_plan
    rows = {}
    for _, wid, r0, n, sh, ng in mv:
        p = plan[wid]
        assert 0 <= r0 and r0 + n <= p["nrows"] and (sh, ng) == (p["sh"], p["ng"])
        rows.setdefault(wid, set()).update(range(r0, r0 + n))
    # the looped body streams every row of every image once per token
    assert sorted(rows) == list(range(16))
    assert all(len(rows[w]) == plan[w]["nrows"] for w in rows)


def test_mvgo_refusals(art):
    W = DDRWeights(art.meta["weights"], art.meta)
    i, d = art.mvgos()[0]
    with pytest.raises(AssertionError):
        W._lookup(d["wbase"] + 1)             # not row-aligned
    with pytest.raises(AssertionError):
        W._lookup(0)                          # below the weight region
    r = art.recs[i]
    r2 = type(r)(OP_MVGO, r.flags | 0x1, r.target, r.imm32, r.addr_lo, r.len_or_addr_hi)
    with pytest.raises(SeqFormatError):
        decode_mvgo(r2)                       # MVGO cannot use indirection


def test_layer_types_from_the_weight_plan(art):
    assert layer_types_of(art.meta["weights"]) == (["linear_attention", "full_attention"], 8192)


@pytest.mark.parametrize("name,fx", ARTIFACTS)
def test_stream_constants_are_the_reference_vectors(name, fx, golden):
    d = golden(fx)
    a = SeqArtifact.load(os.path.join(HERE, "golden", "seq9b", name))
    types, _ = layer_types_of(a.meta["weights"])
    layers = ref_layers(d, types)
    h = SeqHarness(a, layers, d["ln_f"], emb_q=np.zeros((1, 1)), images={})
    h.check_constants()
    ia = types.index("full_attention")
    layers[ia]["attn"]["q_norm"] = layers[ia]["attn"]["q_norm"] + 1
    with pytest.raises(AssertionError):
        h.check_constants()


@pytest.mark.parametrize("name,fx", ARTIFACTS)
def test_every_artifact_reads_and_resolves(name, fx, golden):
    a = SeqArtifact.load(os.path.join(HERE, "golden", "seq9b", name))
    d = golden(fx)
    assert a.histogram() == a.meta["opcode_histogram"]
    assert a.expect_tokens == [int(t) for t in d["tokens"]]
    plan = a.weight_plan
    rows = {}
    for _, wid, r0, n, sh, ng in a.check_mvgo_plan():
        rows.setdefault(wid, set()).update(range(r0, r0 + n))
    assert sorted(rows) == sorted(plan) and all(len(rows[w]) == plan[w]["nrows"] for w in rows)
    types, vocab = layer_types_of(a.meta["weights"])
    assert len(types) == (int(d["nlayers"]) if "nlayers" in d else 2)


def test_state_region_round_trip(art):
    plan = art.manifest["state"]
    reg = StateRegion(plan)
    rng = np.random.default_rng(3)
    S = rng.integers(-32768, 32768, (32, 128, 128)).astype(np.int16)
    taps = rng.integers(-32768, 32768, (8192, 4))
    win = rng.integers(-32768, 32768, (8192, 3))
    kv = [rng.integers(-128, 128, s).astype(np.int8) for s in ((5, 4, 256), (5, 4), (5, 4, 256), (5, 4))]
    reg.put_dn_state(2, S)
    reg.put_conv(2, taps, win)
    reg.put_kv(1, *kv)
    assert np.array_equal(reg.dn_state(2), S)
    t2, w2 = reg.conv(2)
    assert np.array_equal(t2, taps) and np.array_equal(w2, win)
    for a, b in zip(reg.kv(1, 5), kv):
        assert np.array_equal(a, b)
    # the block addresses of the reference layout (sw/hwmap.py:621-628)
    assert plan["kv"] - plan["dn"] == 24 << 20 and plan["cv"] - plan["kv"] == 64 << 21
    assert plan["end"] - plan["cv"] == 24 << 17
    assert slots(["linear_attention"] * 3 + ["full_attention"]) == [
        ("linear_attention", 0, None), ("linear_attention", 1, None), ("linear_attention", 2, None),
        ("full_attention", None, 0)]


@pytest.mark.slow
@pytest.mark.parametrize("name,fx", ARTIFACTS)
def test_seed_restatement_matches_the_reference_generator(name, fx, golden):
    """The float model rebuilt from the generator's seed gives the
    reference's quantized vectors, embedding table (sha256) and prompt."""
    d = golden(fx)
    a = SeqArtifact.load(os.path.join(HERE, "golden", "seq9b", name))
    types, vocab = layer_types_of(a.meta["weights"])
    m = GEN.token_model(int(d["seed"]), types, vocab=int(d["vocab"]))
    ref = ref_layers(d, types)
    for i, wf in enumerate(m["layers"]):
        v = Q.layer_vectors(wf)
        assert np.array_equal(v["ln1"], ref[i]["ln1"]) and np.array_equal(v["ln2"], ref[i]["ln2"]), f"layer {i}"
        sub = "attn" if wf["type"] == "full_attention" else "dn"
        for k, want in ref[i][sub].items():
            assert np.array_equal(v[sub][k], want), f"layer {i} {k}"
    assert np.array_equal(m["ln_f_q14"], d["ln_f"])
    emb = np.ascontiguousarray(m["emb_q"].astype("<i2"))
    assert hashlib.sha256(emb.tobytes()).hexdigest() == str(d["emb_sha256"])
    assert [m["prompt"]] == a.prompt

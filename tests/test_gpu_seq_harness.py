"""The SEQ-stream harness on the GPU, against the unmodified reference's
9B token-stream run (tests/golden/seq9b, tests/golden/seq9b_ref.npz; the
run passed the reference's own SEQ gate when the fixtures were made).

The model is rebuilt from the generator's seed (tests/golden/seq_model_gen.py)
and quantized by the GPU checkpoint quantizer; then
  * every weight image is byte-identical to the reference artifact's
    (sha256 of each ``_w<wid>.bin``);
  * every MVGO record of the stream, run through the GPU DDRWeights engine
    on a seeded x8, equals the oracle's matvec_y32 over the same rows;
  * the decode the stream encodes, run by SeqHarness on the persistent
    engine in the stream's EPS-NORM mode and in the float mode, emits the
    stream's expect_tokens, with every step's final residual equal to
    layer_decode_fx's, and leaves a state region image whose sha256 is the
    reference executor's final one.
When F5_SEQ_ARTIFACT names a full artifact prefix (the generator's files,
e.g. from tests/golden/gen_seq_golden.py), the harness also runs from those
files directly."""
import hashlib
import os
import sys

import numpy as np
import pytest

import oracle as O
from fable5_llm_b200 import quant as Q
from fable5_llm_b200.artifact import wid_plan
from fable5_llm_b200.seq_harness import ATTN_NAMES, DN_NAMES, SeqHarness, layer_types_of
from fable5_llm_b200.seq_stream import SeqArtifact
from fable5_llm_b200.seq_weights import DDRWeights

HERE = os.path.dirname(os.path.abspath(__file__))
sys.path.insert(0, os.path.join(HERE, "golden"))
import seq_model_gen as GEN  # noqa: E402

pytestmark = [pytest.mark.gpu, pytest.mark.slow]

# (stream name, reference fixture) of every committed SEQ artifact: the
# legacy DeltaNet + attention pair, and the config's first four layers
ARTIFACTS = [(n, f) for n, f in (("tok9", "seq9b_ref"), ("tok9l4", "tok9l4_ref"))
             if os.path.exists(os.path.join(HERE, "golden", "seq9b", n + ".seq"))]


@pytest.fixture(scope="module", params=ARTIFACTS, ids=[a[0] for a in ARTIFACTS])
def rebuilt(request, golden):
    """(artifact, reference fixture, vectors per layer, {wid: (device image, e)}, model)."""
    name, fx = request.param
    d = golden(fx)
    art = SeqArtifact.load(os.path.join(HERE, "golden", "seq9b", name))
    types, _ = layer_types_of(art.meta["weights"])
    m = GEN.token_model(int(d["seed"]), types, vocab=int(d["vocab"]))
    images, vecs, wid = {}, [], 0
    for wf in m["layers"]:
        vecs.append(Q.layer_vectors(wf))
        own = wf["attn"] if wf["type"] == "full_attention" else wf["dn"]
        for nm in (ATTN_NAMES if wf["type"] == "full_attention" else DN_NAMES):
            W = wf["mlp"][nm] if nm in ("gate", "up", "down") else own[nm]
            img, N, K, e, sh = Q.quant_linear_image(W)
            images[wid] = (img, e)
            wid += 1
    img, N, K, e, sh = Q.quant_linear_image(m["head"])
    images[wid] = (img, e)
    return art, d, vecs, images, m


def test_gpu_quantizer_reproduces_every_reference_image(rebuilt):
    art, d, _, images, m = rebuilt
    plan = wid_plan(m["types"])
    assert len(images) == len(plan) == len(d["image_sha256"])
    for wid in range(len(plan)):
        img, e = images[wid]
        got = hashlib.sha256(img.cpu().numpy().tobytes()).hexdigest()
        assert got == str(d["image_sha256"][wid]), f"wid {wid} {plan[wid]}"
        assert e == art.manifest[str(wid)]["e"], f"wid {wid}: e"


def test_every_mvgo_on_the_gpu_engine(rebuilt):
    art, _, _, images, _ = rebuilt
    W = DDRWeights.from_images({w: img for w, (img, _) in images.items()}, art.meta["weights"], art.meta)
    rng = np.random.default_rng(11)
    seen = set()
    for i, wid, r0, n, sh, ng in art.check_mvgo_plan(W):
        if (wid, r0) in seen:
            continue
        seen.add((wid, r0))
        p = art.weight_plan[wid]
        x8 = rng.integers(-127, 128, p["k"]).astype(np.int8)
        y = art.mvgo_matvec(W, i, x8)
        rows = images[wid][0][r0 * p["stride"]:(r0 + n) * p["stride"]].cpu().numpy()
        w4, mm = O.unpack_ddr_rows(rows, n, p["k"])
        ref = O.matvec_y32_np(w4, mm, sh, x8)
        assert np.array_equal(y, np.asarray(ref, dtype=np.int64)), f"MVGO rec {i} (wid {wid} rows {r0}+{n})"


@pytest.mark.parametrize("norm_mode", ["eps", "float"])
def test_seq_decode_on_the_gpu(rebuilt, norm_mode):
    art, d, vecs, images, m = rebuilt
    h = SeqHarness(art, vecs, m["ln_f_q14"], emb_q=m["emb_q"], images=images, norm_mode=norm_mode)
    h.check_constants()
    try:
        toks = h.run()
        assert toks == art.expect_tokens == [int(t) for t in d["tokens"]]
        for t, x in enumerate(h.residuals):
            assert np.array_equal(x, d["layer_out"][t][-1]), f"step {t}: residual"
        reg = h.final_state()
        assert reg.sha256() == str(d["state_final_sha256"]) == art.manifest["state"]["final_sha256"]
    finally:
        h.close()


@pytest.mark.skipif(not os.environ.get("F5_SEQ_ARTIFACT"), reason="F5_SEQ_ARTIFACT (a full artifact prefix) not set")
def test_seq_decode_from_the_artifact_files(rebuilt):
    ref_art, d, vecs, _, m = rebuilt
    if os.path.basename(os.environ["F5_SEQ_ARTIFACT"]) != os.path.basename(ref_art.prefix):
        pytest.skip("F5_SEQ_ARTIFACT names another stream")
    art = SeqArtifact.load(os.environ["F5_SEQ_ARTIFACT"])
    h = SeqHarness(art, vecs, m["ln_f_q14"])
    try:
        assert h.run() == art.expect_tokens
        assert h.final_state().sha256() == art.manifest["state"]["final_sha256"]
    finally:
        h.close()

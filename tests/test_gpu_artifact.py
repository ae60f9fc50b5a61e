"""A model loaded from a reference weight artifact decodes exactly like the
same weights loaded any other way.

The seeded 4-layer model (three DeltaNet layers and one attention layer,
vocab 4096) is written as a reference artifact (``.weights.json`` plus one
``_w<wid>.bin`` image per matrix in the reference's wid order, and
``.emb.bin``), loaded through ``DecodeModel.load_artifact`` and stepped next
to the same model generated on the device: every token and every logit of
several decode steps must be equal, on both engines.
"""
import numpy as np
import pytest

import oracle as O
from fable5_llm_b200 import artifact as A
from fable5_llm_b200 import synth
from fable5_llm_b200.config import RS_F, Geometry
from fable5_llm_b200.model import DecodeModel
from oracle.model import OracleModel

pytestmark = pytest.mark.gpu
SEED = 2026


def _mats_in_wid_order(om, g):
    out = []
    for layer, name in A.wid_plan(g.layer_types):
        if name == "head":
            out.append(om.head)
            continue
        qw = om.layers[layer]
        own = qw["attn"] if qw["type"] == "full_attention" else qw["dn"]
        out.append(qw["mlp"][name] if name in A.MLP_ORDER else own[name])
    return out


@pytest.mark.parametrize("engine", ["persistent", "graph"])
def test_artifact_model_matches_device_generated_model(tmp_path, engine):
    g = Geometry(4, 4096)
    om = OracleModel(SEED, O.Geometry(4, 4096))
    pre = str(tmp_path / "m4")
    emb = synth.emb_rows(SEED, np.arange(g.vocab), g.H)
    A.write_weights(pre, _mats_in_wid_order(om, g), emb_q=emb, emb_row_bytes=2 * g.H, rs_f=RS_F)
    a = DecodeModel(g, max_T=128)
    a.load_artifact(pre, om.layers, om.ln_f_q12)
    b = DecodeModel(g, max_T=128)
    b.load_synthetic(SEED)
    try:
        for m in (a, b):
            m.set_engine(engine)
            m.reset()
            m.set_logits(True)
        assert a.head_e_sh == b.head_e_sh
        for t, tok in enumerate([5, 4095, 77, 1000, 3]):
            ra, rb = a.decode_step(tok, t), b.decode_step(tok, t)
            assert ra == rb
            assert np.array_equal(a.logits(), b.logits())
    finally:
        a.close()
        b.close()

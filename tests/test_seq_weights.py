"""The seq_model matvec-engine drop-in (fable5_llm_b200.seq_weights.DDRWeights,
replacing ref/seq_model.py:305-452): WBASE lookup and refusals on the CPU,
and on the GPU every MVGO-style call over the reference-written weight
artifact (tests/golden/artifact, dumped by the reference's own
Mach.dump_weights) equals the oracle's matvec_y32 on the same rows."""
import json
import os

import numpy as np
import pytest

import oracle as O
from fable5_llm_b200.seq_weights import DDRWeights

ART = os.path.join(os.path.dirname(os.path.abspath(__file__)), "golden", "artifact")
PREFIX = os.path.join(ART, "tiny")


def make_plan(prefix, base0=0x10000, align=4096):
    """A stream's weight plan over a manifest: images laid out one after the
    other from base0 (each base aligned), the fields SeqExec's plan carries."""
    man = json.load(open(prefix + ".weights.json"))
    plan, base = {}, base0
    for wid in sorted((int(k) for k in man if k.isdigit())):
        m = man[str(wid)]
        p = {k: m[k] for k in ("nrows", "k", "ng", "sh", "stride", "nbeats")}
        p["g"] = int(m.get("g", 128))
        p["base"] = base
        plan[wid] = p
        base += -(-m["nrows"] * m["stride"] // align) * align
    return plan


def test_lookup_and_refusals_cpu():
    plan = make_plan(PREFIX)
    W = DDRWeights(plan)
    for wid, p in plan.items():
        assert W._lookup(p["base"])[:2] == (wid, 0)
        assert W._lookup(p["base"] + 3 * p["stride"])[:2] == (wid, 3)
        assert W._lookup(p["base"] + 3 * p["stride"])[3] == p["nrows"] - 3
    first = min(p["base"] for p in plan.values())
    with pytest.raises(AssertionError):
        W._lookup(first - 64)                       # below the weight region
    p0 = plan[0]
    with pytest.raises(AssertionError):
        W._lookup(p0["base"] + 64)                  # not row-aligned
    with pytest.raises(AssertionError):
        W._lookup(p0["base"] + p0["nrows"] * p0["stride"] + 64)   # in the gap after the image
    with pytest.raises(NotImplementedError):
        DDRWeights({0: dict(p0, w8=True)})
    with pytest.raises(NotImplementedError):
        DDRWeights({0: dict(p0, base=[0, 0])}, {"weight_repack": True, "nch": 2})


@pytest.mark.gpu
def test_matvec_calls_vs_oracle():
    plan = make_plan(PREFIX)
    W = DDRWeights.from_files(PREFIX, plan)
    man = json.load(open(PREFIX + ".weights.json"))
    rng = np.random.default_rng(11)
    for wid, p in plan.items():
        img = np.fromfile(os.path.join(ART, man[str(wid)]["file"]), dtype=np.uint8).reshape(p["nrows"], p["stride"])
        K, g, sh = p["k"], p["g"], p["sh"]
        x8 = rng.integers(-127, 128, K).astype(np.int8)
        # whole image, then the MVGO chunking of a row window
        for r0, n in [(0, p["nrows"]), (1, p["nrows"] - 1), (p["nrows"] // 2, p["nrows"] - p["nrows"] // 2), (2, 3)]:
            y = W.matvec(p["base"] + r0 * p["stride"], n, sh, p["ng"], g, x8)
            ref = O.matvec_img(img[r0:r0 + n], n, K, sh, x8, g).astype(np.int64)
            assert y.dtype == np.int64 and np.array_equal(y, ref), (wid, r0, n)
    p = plan[0]
    x8 = np.zeros(p["k"], dtype=np.int8)
    with pytest.raises(AssertionError):
        W.matvec(p["base"], p["nrows"] + 1, p["sh"], p["ng"], p["g"], x8)          # overruns the image
    with pytest.raises(AssertionError):
        W.matvec(p["base"], 1, p["sh"] + 1, p["ng"], p["g"], x8)                   # SHAPE != manifest
    with pytest.raises(AssertionError):
        W.matvec(p["base"], 1, p["sh"], p["ng"], p["g"], np.zeros(p["k"] + 1, np.int8))   # XWIN != K

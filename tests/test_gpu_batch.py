"""GPU parity of the batched decode path (B sequences sharing the weights):
the tcgen05 W4A8 GEMM against the oracle's matvec_y32, one sequence at a
time, bit-exact."""
import numpy as np
import pytest
import torch

import oracle as O
from fable5_llm_b200 import ops

pytestmark = pytest.mark.gpu


def rand_image(rng, N, K, m_lo=1, m_hi=65536):
    w4 = rng.integers(-8, 8, (N, K)).astype(np.int8)
    m = rng.integers(m_lo, m_hi, (N, K // 128)).astype(np.uint16)
    img, _ = O.pack_ddr_rows(w4, m, 128)
    return img


def check_batch(img, N, K, x8):
    sh = O.final_shift(K)
    d_img = ops.to_dev(img)
    y, err, p = ops.batch_matvec_y32(d_img, N, K, sh, ops.to_dev(x8), want_p=True)
    torch.cuda.synchronize()
    assert int(err.item()) == 0
    y, p = y.cpu().numpy(), p.cpu().numpy()
    for b in range(x8.shape[0]):
        y_ref, p_ref = O.matvec_img(img, N, K, sh, x8[b], 128, want_p=True)
        assert np.array_equal(p[b], p_ref), f"p mismatch at sequence {b}"
        assert np.array_equal(y[b], y_ref), f"y32 mismatch at sequence {b}"


@pytest.mark.parametrize("B", [1, 8, 16, 17, 32, 40, 64])
def test_batch_matvec_4096(B):
    rng = np.random.default_rng(100 + B)
    N, K = 1000, 4096          # a ragged last tile (1000 = 7 * 128 + 104)
    img = rand_image(rng, N, K)
    x8 = rng.integers(-127, 128, (B, K)).astype(np.int8)
    check_batch(img, N, K, x8)


@pytest.mark.parametrize("N,K,B", [(4096, 4096, 64), (32, 4096, 8), (4096, 12288, 32), (300, 12288, 64),
                                   (12288, 4096, 16), (2048, 1024, 8)])
def test_batch_matvec_shapes(N, K, B):
    rng = np.random.default_rng(N + K + B)
    img = rand_image(rng, N, K)
    x8 = rng.integers(-127, 128, (B, K)).astype(np.int8)
    check_batch(img, N, K, x8)


def test_batch_matvec_extremes():
    """|acc_g| and |p| at their maxima: all -8 / 7 weights, m = 65535,
    x = +-127 (and the unsigned-weight correction at its largest)."""
    for K in (4096, 12288):
        N = 256
        w4 = np.full((N, K), -8, dtype=np.int8)
        w4[1::2] = 7
        m = np.full((N, K // 128), 65535, dtype=np.uint16)
        img, _ = O.pack_ddr_rows(w4, m)
        x8 = np.empty((16, K), dtype=np.int8)
        x8[0::2], x8[1::2] = 127, -127
        x8[3] = np.where(np.arange(K) % 2 == 0, 127, -127)
        check_batch(img, N, K, x8)


# ---------------------------------------------------------------------------
# batched decode engine vs B independent single-sequence runs
# ---------------------------------------------------------------------------
from fable5_llm_b200 import _lib as L                      # noqa: E402
from fable5_llm_b200.batch import BatchModel              # noqa: E402
from fable5_llm_b200.config import Geometry               # noqa: E402
from fable5_llm_b200.model import DecodeModel             # noqa: E402

SEED = 2026


@pytest.fixture(scope="module")
def model4b():
    m = DecodeModel(Geometry(4, 4096), max_T=64)
    m.load_synthetic(SEED)
    return m


def single_run(m, toks, T0=0):
    """The single-sequence engine from a zero state: per step (next, y32)."""
    m.reset()
    m.set_position(T0, T0)
    out = []
    for t, tok in enumerate(toks):
        out.append(m.decode_step(int(tok), T0 + t))
    return out


def state_of(read, geom, layers=None):
    st = {}
    for i, lt in enumerate(geom.layer_types):
        if layers is not None and i not in layers:
            continue
        bufs = (L.BUF_K8, L.BUF_KE, L.BUF_V8, L.BUF_VE) if lt == "full_attention" else (L.BUF_DN_S, L.BUF_DN_CONV, L.BUF_DN_KH)
        for b in bufs:
            st[(i, b)] = read(b, i)
    return st


@pytest.mark.parametrize("B", [3, 17, 40])
def test_batch_engine_matches_single(model4b, B):
    """Every sequence of a batched step equals the single-sequence engine
    (which is pinned to the reference) in every token, logit and state word."""
    m = model4b
    rng = np.random.default_rng(B)
    nsteps = 3
    toks = rng.integers(0, m.geom.vocab, (B, nsteps))
    bm = BatchModel(m, B)
    bm.reset()
    got = [bm.step(toks[:, t]) for t in range(nsteps)]
    check = sorted({0, B // 2, B - 1})
    for b in check:
        ref = single_run(m, toks[b])
        for t in range(nsteps):
            assert (int(got[t][0][b]), int(got[t][1][b])) == ref[t], f"sequence {b} step {t}"
        s_ref = state_of(lambda w, i: m.read(w, i), m.geom)
        s_got = state_of(lambda w, i: bm.read(b, w, i), m.geom)
        for k in s_ref:
            assert np.array_equal(s_ref[k], s_got[k]), f"sequence {b} state {k}"
        assert bm.position(b) == (nsteps, nsteps)
    bm.close()


def test_batch_engine_greedy_loop_and_offsets(model4b):
    """Sequences at different RoPE positions, then device-fed greedy steps."""
    m = model4b
    B = 5
    bm = BatchModel(m, B)
    bm.reset()
    rng = np.random.default_rng(7)
    off = [0, 3, 11, 20, 33]
    for b in range(B):
        bm.set_position(0, off[b], b)
    pre = rng.integers(0, m.geom.vocab, (B, 5))
    for t in range(5):
        bm.step(pre[:, t])
    bm.launch(3)
    last, mv = bm.sync()
    for b in (0, 2, B - 1):
        m.reset()
        for t in range(5):
            m.decode_step(int(pre[b, t]), off[b] + t)
        m.decode_launch(3)
        assert (int(last[b]), int(mv[b])) == m.sync(), f"sequence {b}"
        assert bm.position(b) == (8, off[b] + 8)
    bm.close()


def test_batch_topk_and_sampling(model4b):
    """Per-sequence TOPK-32 capture of the batched step: each sequence's
    stored logits equal the single-sequence engine's, its capture equals the
    oracle's over them and the single engine's capture (e_x included), and
    entry 0 is the greedy token; a seeded sampled continuation of every
    sequence is reproducible."""
    from oracle import topk as OT
    from fable5_llm_b200 import sampling as S
    m = model4b
    B = 5
    rng = np.random.default_rng(3)
    toks = rng.integers(0, m.geom.vocab, (B, 3))
    bm = BatchModel(m, B)
    bm.set_logits(True)
    bm.reset()
    for t in range(3):
        nt, mv = bm.step(toks[:, t])
    caps = bm.topk()
    m.set_logits(True)
    for b in (0, 2, B - 1):
        single_run(m, toks[b])
        lg = bm.logits(b)
        assert np.array_equal(lg, m.logits()), f"sequence {b} logits"
        r, rs = caps[b], m.topk()
        exp = OT.topk32(lg)
        assert np.array_equal(r.values, exp["val"]) and np.array_equal(r.indices, exp["idx"])
        assert (r.ovf_lit, r.ovf_disp) == (exp["ovf_lit"], exp["ovf_disp"])
        assert r.indices[0] == nt[b] and r.values[0] == mv[b]
        assert np.array_equal(r.values, rs.values) and np.array_equal(r.indices, rs.indices) and r.e_x == rs.e_x
    m.set_logits(False)
    runs = []
    for rep in range(2):
        bm.reset()
        samplers = [S.Sampler(temp=0.9, top_k=16, seed=100 + b, logit_exp0=m.head_logit_exp0()) for b in range(B)]
        cur, seq = toks[:, 0], []
        for t in range(3):
            cur, info = bm.sample_step(cur, samplers)
            assert all(i["mode"] == "sampled" for i in info)
            seq.append(cur.copy())
        runs.append(np.stack(seq))
    assert np.array_equal(runs[0], runs[1])
    bm.close()

"""Pin the CPU oracle against the reference's own golden vectors and against
outputs of the unmodified reference (tests/golden/gen_golden.py)."""
import hashlib
import os

import numpy as np
import pytest

import oracle as O

I64 = np.int64


def digest(a):
    return hashlib.sha256(np.ascontiguousarray(np.asarray(a, dtype=I64)).tobytes()).hexdigest()


# ---- tb/vec_s1..s4: the reference's committed matvec vectors ----
@pytest.mark.parametrize("s", [1, 2, 3, 4])
def test_tb_matvec(golden, s):
    d = golden("tb_matvec")
    K, NG, SH, N, BPR = [int(v) for v in d[f"s{s}_params"]]
    assert O.row_stride(K) == BPR * 64
    assert O.final_shift(K) == SH
    img = d[f"s{s}_img"]
    y = O.matvec_img(img, N, K, SH, d[f"s{s}_x8"])
    assert np.array_equal(y, d[f"s{s}_y32"])
    # numpy path over the unpacked image agrees too
    w4, m = O.unpack_ddr_rows(img, N, K)
    assert np.array_equal(O.matvec_y32_np(w4, m, SH, d[f"s{s}_x8"]), d[f"s{s}_y32"])
    img2, _ = O.pack_ddr_rows(w4, m)
    assert np.array_equal(img2.reshape(-1), img)


def test_roms(golden):
    r = golden("roms")
    assert np.array_equal(O.RSQRT_LUT, r["rsqrt"])
    assert np.array_equal(O.RECIP_LUT, r["recip"])
    assert np.array_equal(O.EXP2_LUT, r["exp2"])
    assert np.array_equal(O.SIGMOID_LUT, r["sigmoid"])
    assert np.array_equal(O.SOFTPLUS_LUT, r["softplus"])


# ---- tb/vectors/s1..s4: unit-block vectors (ref/gen_layer_vectors.py) ----
@pytest.mark.parametrize("s", [1, 2, 3, 4])
def test_tb_layer_vectors(golden, s):
    d = golden("tb_layer")
    g = lambda k: d[f"s{s}_{k}"]  # noqa: E731
    # rmsnorm (1+w), N=1024 at the pinned vector fraction 8
    assert np.array_equal(O.rmsnorm_fx(g("rmsnorm_x16"), g("rmsnorm_w14"), 8, True), g("rmsnorm_y16"))
    # rope
    assert np.array_equal(O.rope_fx(g("rope_x16"), g("rope_cos"), g("rope_sin")), g("rope_y16"))
    # l2norm
    assert np.array_equal(O.l2norm_fx(g("l2norm_x16"), O.QKV_F, O.NRM_F), g("l2norm_y16"))
    # conv4 + silu (the conv shift RS_F + CW_F - 12 of the operating point the
    # vectors were emitted at: 8 at RS_F=7 (9B), 9 at RS_F=8)
    win = g("conv_win").reshape(64, 4)
    cw = g("conv_w").reshape(64, 4)
    acc = (win * cw).sum(axis=1)
    ok = False
    for shift in (8, 9):
        pre = np.clip(O.rshr(acc, shift), -(1 << 20), (1 << 20) - 1)
        if np.array_equal(O.clip16(O.silu_q(pre)), g("conv_y")):
            ok = True
    assert ok
    # attention core (T=48)
    T = 48
    qn = g("attn_q")
    k8 = g("attn_k8").reshape(T, 256)
    ke = g("attn_ke")
    v8 = g("attn_v8").reshape(T, 256)
    ve = g("attn_ve")
    s_ = O.rshr((k8 @ qn) * 2048, 15)
    sc = O.rshr_v(s_, O.QKV_F - ke - 16)
    es = O.exp_neg_q(np.minimum(sc - sc.max(), 0))
    r, re = O.recip_q(int(es.sum()), 30)
    p = np.clip(O.rshr(es * r, 30 - re + 15), 0, 1 << 15)
    assert np.array_equal(p, g("attn_p"))
    acc = O.rshr_v(p[:, None] * v8, (15 - ve - O.QKV_F)[:, None]).sum(axis=0)
    assert np.array_equal(acc, g("attn_acc"))
    # DeltaNet recurrence step
    S = g("dn_sin").reshape(128, 128)
    q, k, v = g("dn_q"), g("dn_k"), g("dn_v")
    dec, bet = [int(x) for x in g("dn_gates")]
    Sh = O.rshr(S * dec, O.GAT_F)
    kvm = O.rshr((Sh * k[:, None]).sum(axis=0), O.NRM_F)
    dl = O.rshr((v - kvm) * bet, O.GAT_F)
    Sh = O.clip16(Sh + O.rshr(k[:, None] * dl[None, :], O.NRM_F))
    assert np.array_equal(Sh.reshape(-1), g("dn_sout"))
    assert np.array_equal(O.rshr((Sh * q[:, None]).sum(axis=0), O.NRM_F), g("dn_o"))
    # gate unit
    beta = O.sigmoid_q(g("gate_b"))
    assert np.array_equal(beta, g("gate_beta"))
    sp = O.softplus_q(g("gate_a") + g("gate_dt"))
    g16 = -O.rshr((g("gate_A") & ((1 << 18) - 1)) * sp, 11)   # A is an unsigned 18-bit port
    decay = np.minimum(O.rshr(O.exp_neg_q(np.minimum(g16, 0)), 15), 32767)
    assert np.array_equal(decay, g("gate_decay"))
    # vec_alu ops
    x8, e = O.dyn_quant_i8(g("alu_dynq8_x"))
    assert np.array_equal(x8.astype(I64), g("alu_dynq8_y")) and e == int(g("alu_dynq8_e")[0])
    assert np.array_equal(O.clip16(O.rshr(g("alu_shift32_v"), 5)), g("alu_shift32_y"))
    assert np.array_equal(O.clip16(O.rshr(g("alu_scale_x") * 2896, 15)), g("alu_scale_y"))
    assert np.array_equal(O.clip16(O.rshr(g("alu_emul_a") * g("alu_emul_b"), 12)), g("alu_emul_y"))
    assert np.array_equal(O.clip16(g("alu_emul_a") + g("alu_emul_b")), g("alu_add_y"))
    assert np.array_equal(O.clip16(O.silu_q(g("alu_scale_x") << 4)), g("alu_silu16_y"))
    v20 = np.clip(g("alu_shift32_v"), -(1 << 20), (1 << 20) - 1)
    assert np.array_equal(O.clip16(O.silu_q(v20)), g("alu_silu32_y"))
    assert np.array_equal(O.sigmoid_q(g("alu_scale_x") << 4), g("alu_sigm16_y"))
    assert np.array_equal(O.clip16(O.rshr(g("alu_shift32_v") * g("alu_emul_b"), 15)), g("alu_emul32_y"))


# ---- outputs of the unmodified reference on seeded inputs ----
def test_ref_rshr_dynq(golden):
    d = golden("ref_prims")
    y = np.array([int(O.rshr(v, s)) for v, s in zip(d["rshr_v"], d["rshr_s"])])
    assert np.array_equal(y, d["rshr_y"])
    assert np.array_equal(O.rshr_v(d["rshr_v"], d["rshr_s"]), d["rshr_y"])
    for x, x8r, er in zip(d["dq_x"], d["dq_x8"], d["dq_e"]):
        x8, e = O.dyn_quant_i8(x)
        assert e == er and np.array_equal(x8.astype(I64), x8r)


def test_ref_rsqrt_recip(golden):
    d = golden("ref_prims")
    for v, p, r, e in zip(d["rs_v"], d["rs_p"], d["rs_r"], d["rs_e"]):
        assert O.rsqrt_q(int(v), int(p)) == (int(r), int(e))
    for v, p, r, e in zip(d["rs_v"], d["rs_p"], d["rc_r"], d["rc_e"]):
        assert O.recip_q(int(v), int(p)) == (int(r), int(e))


@pytest.mark.parametrize("name,fn", [("sigmoid", O.sigmoid_q), ("softplus", O.softplus_q),
                                     ("silu", O.silu_q), ("exp_neg", O.exp_neg_q),
                                     ("exp2_frac", O.exp2_frac_q16)])
def test_ref_lut_domains_exhaustive(golden, name, fn):
    d = golden("ref_prims")
    lo, n, sign = int(d[f"{name}_lo"]), int(d[f"{name}_n"]), int(d[f"{name}_sign"])
    dom = -np.arange(0, n, dtype=I64) if sign < 0 else np.arange(lo, lo + n, dtype=I64)
    y = fn(dom)
    assert np.array_equal(y[::97], d[f"{name}_sample"])
    assert digest(y) == str(d[f"{name}_digest"])


def test_ref_exp_neg_tail(golden):
    d = golden("ref_prims")
    assert np.array_equal(O.exp_neg_q(d["expt_x"]), d["expt_y"])


def test_ref_bf_shift(golden):
    d = golden("ref_prims")
    assert np.array_equal(np.array([O.bf_shift(int(m)) for m in d["bf_m"]]), d["bf_k"])


def test_ref_norm_scales(golden):
    d = golden("ref_prims")
    for o32, k, mf, o16, me in zip(d["nb_o32"], d["nb_k"], d["nb_m_float"], d["nb_o16"], d["nb_m_eps"]):
        assert O.bf_shift(int(np.abs(o32).max())) == k
        assert O.dn_norm_scale(o32, int(k)) == mf
        assert np.array_equal(O.clip16(O.rshr(o32, int(k))), o16)
        assert O.eps_norm_scale(o16, int(k)) == me


def test_ref_rmsnorm_l2norm(golden):
    d = golden("ref_prims")
    for tag in ("rn4096", "rn4096p", "rn256", "rn128s"):
        n, in_f, one_plus = [int(v) for v in d[f"{tag}_meta"]]
        for x, y in zip(d[f"{tag}_x"], d[f"{tag}_y"]):
            assert np.array_equal(O.rmsnorm_fx(x, d[f"{tag}_w"], in_f, bool(one_plus)), y)
    for x, y in zip(d["l2_x"], d["l2_y"]):
        assert np.array_equal(O.l2norm_fx(x, 8, 14), y)


def test_ref_rope(golden):
    d = golden("ref_prims")
    tabs = [O.rope_tables_q15(p) for p in range(4096)]
    cos = np.stack([c for c, _ in tabs])
    sin = np.stack([s for _, s in tabs])
    assert np.array_equal(cos[::37], d["rope_cos_sample"])
    assert np.array_equal(sin[::37], d["rope_sin_sample"])
    assert digest(cos) == str(d["rope_cos_digest"]) and digest(sin) == str(d["rope_sin_digest"])
    for p, c, s in zip(d["rope_extra_pos"], d["rope_extra_cos"], d["rope_extra_sin"]):
        cc, ss = O.rope_tables_q15(int(p))
        assert np.array_equal(cc, c) and np.array_equal(ss, s)
    for x, p, y in zip(d["ropefx_x"], d["ropefx_pos"], d["ropefx_y"]):
        assert np.array_equal(O.rope_fx(x, *O.rope_tables_q15(int(p))), y)


# ---- layer- and model-level law: oracle vs the unmodified reference ----
@pytest.fixture(scope="module")
def oracle_model4():
    from oracle.model import OracleModel
    return OracleModel(2026, O.Geometry(4, 4096))


@pytest.mark.parametrize("mode", ["float", "eps"])
def test_oracle_dn_layer_vs_reference(golden, oracle_model4, mode):
    d = golden("ref_layers")
    qw = oracle_model4.layers[0]
    st = O.DNCache()
    for t in range(d["x_in"].shape[0]):
        y = O.layer_decode_fx(d["x_in"][t], qw, st, t, norm_mode=mode)
        assert np.array_equal(y, d[f"dn_{mode}_y"][t])
        assert st.dn_o_shift == list(d[f"dn_{mode}_k"][t])
    assert digest(st.S) == str(d[f"dn_{mode}_S_digest"])
    assert np.array_equal(st.conv, d[f"dn_{mode}_conv"])


def test_oracle_attn_layer_vs_reference(golden, oracle_model4):
    d = golden("ref_layers")
    qw = oracle_model4.layers[3]
    c = O.AttnCache(16)
    for t in range(d["x_in"].shape[0]):
        y = O.layer_decode_fx(d["x_in"][t], qw, c, t + 5)
        assert np.array_equal(y, d["attn_y"][t])
        assert c.attn_o_shift == int(d["attn_ka"][t])
    n = d["x_in"].shape[0]
    assert np.array_equal(c.k8[:, :n].transpose(1, 0, 2).astype(I64), d["attn_k8"])
    assert np.array_equal(c.ke[:, :n].T.astype(I64), d["attn_ke"])
    assert np.array_equal(c.v8[:, :n].transpose(1, 0, 2).astype(I64), d["attn_v8"])
    assert np.array_equal(c.ve[:, :n].T.astype(I64), d["attn_ve"])


def test_oracle_model4_vs_reference(golden, oracle_model4):
    d = golden("ref_model4")
    r = O.OracleRunner(oracle_model4, max_T=16)
    for t, tok in enumerate(d["m4_in"]):
        nt, y = r.step(int(tok), t)
        assert nt == int(d["m4_out"][t]) and int(y.max()) == int(d["m4_ymax"][t])
        for i, x in enumerate(r.layer_out):
            assert np.array_equal(x, d["m4_layer_x"][t][i].astype(I64)), (t, i)


@pytest.mark.skipif(not os.path.exists(os.path.join(os.path.dirname(os.path.abspath(__file__)), "golden",
                                                    "ref_model32.npz")), reason="no ref_model32 fixture")
def test_oracle_model32_vs_reference(golden):
    """The full 32-layer 9B model with the 248,320-row head: the unmodified
    reference's FxRunner-sequence run (three steps from context 0) pins the
    oracle's tokens, max logits, every layer's output and the residual
    saturation counters (ref/fidelity_check.py:416-433)."""
    from oracle.model import OracleModel
    d = golden("ref_model32")
    r = O.OracleRunner(OracleModel(2026, O.GEOM_9B), max_T=8)
    for t, tok in enumerate(d["m32_in"]):
        nt, y = r.step(int(tok), t)
        assert nt == int(d["m32_out"][t]) and int(y.max()) == int(d["m32_ymax"][t])
        for i, x in enumerate(r.layer_out):
            assert np.array_equal(x, d["m32_layer_x"][t][i].astype(I64)), (t, i)
    x = d["m32_layer_x"].astype(I64)
    assert r.resid_max == int(np.abs(x).max())
    assert r.resid_clip == int(((x >= 32767) | (x <= -32768)).sum())

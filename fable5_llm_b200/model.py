"""Host side of the resident decode model (one GPU per context).

``DecodeModel`` owns an ``f5_ctx`` (include/f5b200.h): the integer
Qwen3.5-9B weights in HBM in the reference's packed row format, the decode
state (int8 KV caches, DeltaNet conv windows and int16 states) and the
decode step (one persistent cooperative launch per token by default, or
the per-op kernel chain replayed as a CUDA graph).  All compute is in the CUDA
library; this module only moves parameters and results.
"""
from __future__ import annotations

import ctypes

import numpy as np

from . import _lib as L
from . import synth
from .config import RS_F, Geometry
from .rope import rope_table

I64 = np.int64

DN_SLOTS = {"in_qkv": L.S_IN_QKV, "in_z": L.S_IN_Z, "in_b": L.S_IN_B, "in_a": L.S_IN_A, "out": L.S_OUT}
ATTN_SLOTS = {"q_proj": L.S_Q, "k_proj": L.S_K, "v_proj": L.S_V, "o_proj": L.S_O}
MLP_SLOTS = {"gate": L.S_GATE, "up": L.S_UP, "down": L.S_DOWN}
NORM_MODES = {"float": 0, "eps": 1}


def _p(a):
    return ctypes.c_void_p(a.ctypes.data)


class DecodeModel:
    """Resident integer model on one GPU.

    geom: fable5_llm_b200.config.Geometry (9B shapes; n_layers/vocab may be
    reduced); max_T: KV capacity; norm_mode: "float" (ref/layer_fixed.py
    default) or "eps" (the seq_model EPS-NORM law)."""

    def __init__(self, geom=None, max_T=4096, norm_mode="float", device=0, world_size=1, rank=0,
                 max_pos=None):
        self.geom = geom or Geometry()
        self.max_T = (int(max_T) + 15) & ~15      # the context rounds KV capacity to 16 rows
        self.norm_mode = norm_mode
        self.device = device
        self.head_e_sh = None   # (e, sh) of the uploaded LM head
        self.lib = L.lib()
        types = "".join("A" if t == "full_attention" else "D" for t in self.geom.layer_types)
        self._types = types.encode()
        cfg = L.Config(1, self.geom.n_layers, self.geom.vocab, self.max_T, NORM_MODES[norm_mode],
                       world_size, rank, self._types)
        h = ctypes.c_void_p()
        L.check(self.lib.f5_ctx_create(ctypes.byref(cfg), device, ctypes.byref(h)), "f5_ctx_create")
        self.h = h
        npos = int(max_pos) if max_pos else self.max_T
        self.rope = rope_table(npos, self.geom)
        L.check(self.lib.f5_ctx_upload_rope(self.h, _p(self.rope), npos), "f5_ctx_upload_rope")

    def close(self):
        if getattr(self, "h", None):
            self.lib.f5_ctx_destroy(self.h)
            self.h = None

    def __del__(self):
        try:
            self.close()
        except Exception:
            pass

    # ---- weights ----
    def upload_matrix(self, layer, slot, img, N, K, e, sh, g=128):
        img = np.ascontiguousarray(img, dtype=np.uint8)
        L.check(self.lib.f5_ctx_upload_matrix(self.h, layer, slot, _p(img), N, K, g, e, sh),
                f"upload_matrix({layer},{slot})")
        if layer == -1 and slot == L.S_HEAD:
            self.head_e_sh = (int(e), int(sh))

    def upload_qmat(self, layer, slot, qm):
        """qm: the reference dict {"w4","m","e","sh","g"} or an object with
        .img/.N/.K/.e/.sh/.g (packed image)."""
        if isinstance(qm, dict):
            from .w4a8_ref import pack_ddr_rows
            img, _ = pack_ddr_rows(qm["w4"], qm["m"], qm.get("g", 128))
            N, K = qm["w4"].shape
            self.upload_matrix(layer, slot, np.frombuffer(img, dtype=np.uint8), N, K, qm["e"], qm["sh"],
                               qm.get("g", 128))
        else:
            self.upload_matrix(layer, slot, qm.img, qm.N, qm.K, qm.e, qm.sh, qm.g)

    def upload_vector(self, layer, kind, v):
        v = np.ascontiguousarray(np.asarray(v, dtype=I64).reshape(-1))
        L.check(self.lib.f5_ctx_upload_vector(self.h, layer, kind, _p(v), v.size), f"upload_vector({layer},{kind})")

    def upload_layer(self, i, qw):
        """One layer in the reference dict layout (ref/layer_fixed.py:1607-1651)."""
        for nm, sl in MLP_SLOTS.items():
            self.upload_qmat(i, sl, qw["mlp"][nm])
        own = (qw["attn"], ATTN_SLOTS) if qw["type"] == "full_attention" else (qw["dn"], DN_SLOTS)
        for nm, sl in own[1].items():
            self.upload_qmat(i, sl, own[0][nm])
        self.upload_layer_vectors(i, qw)

    def upload_layer_vectors(self, i, qw):
        """The integer vectors of one reference layer dict (norm gains, and
        conv taps / gate constants / gated-norm gain, or q/k norm gains)."""
        self.upload_vector(i, L.VEC_LN1, qw["ln1"])
        self.upload_vector(i, L.VEC_LN2, qw["ln2"])
        if qw["type"] == "full_attention":
            a = qw["attn"]
            self.upload_vector(i, L.VEC_Q_NORM, a["q_norm"])
            self.upload_vector(i, L.VEC_K_NORM, a["k_norm"])
        else:
            d = qw["dn"]
            self.upload_vector(i, L.VEC_CONV_W, d["conv_w"])
            self.upload_vector(i, L.VEC_DT_BIAS, d["dt_bias_q12"])
            self.upload_vector(i, L.VEC_A, d["A_q15"])
            self.upload_vector(i, L.VEC_NORM_W, d["norm_w_q14"])

    @staticmethod
    def slot_of(name):
        """Matrix slot of a reference matrix name ("head" for the LM head)."""
        return L.S_HEAD if name == "head" else {**DN_SLOTS, **ATTN_SLOTS, **MLP_SLOTS}[name]

    def upload_final_norm(self, ln_f_q12):
        self.upload_vector(-1, L.VEC_LN_F, ln_f_q12)

    def upload_embedding(self, emb_q):
        emb = np.ascontiguousarray(emb_q, dtype=np.int16)
        L.check(self.lib.f5_ctx_upload_embedding(self.h, _p(emb), emb.shape[0], emb.shape[1]), "upload_embedding")

    def upload_model(self, layers, emb_q, head, ln_f_q12):
        for i, qw in enumerate(layers):
            self.upload_layer(i, qw)
        self.upload_qmat(-1, L.S_HEAD, head)
        self.upload_final_norm(ln_f_q12)
        self.upload_embedding(emb_q)

    def load_artifact(self, prefix, layers=None, ln_f_q12=None):
        """A reference weight artifact (``<prefix>.weights.json``, its
        ``_w<wid>.bin`` images and ``.emb.bin``), image by image; the layer
        vectors come from the reference layer dicts (fable5_llm_b200.artifact)."""
        from . import artifact
        return artifact.load_artifact(self, prefix, layers, ln_f_q12)

    def load_synthetic(self, seed):
        """The seeded synthetic model of fable5_llm_b200.synth, generated on
        the device (weights) and the host (small vectors)."""
        g = self.geom
        for s in synth.matrix_specs(g):
            slot = L.S_HEAD if s.name == "head" else {**DN_SLOTS, **ATTN_SLOTS, **MLP_SLOTS}[s.name]
            L.check(self.lib.f5_ctx_synth_matrix(
                self.h, s.layer, slot, s.N, s.K, s.g, s.e, s.sh,
                synth.stream_key(seed, s.mid, synth.STREAM_W), synth.stream_key(seed, s.mid, synth.STREAM_M),
                int(s.symmetric)), f"synth {s.name}@{s.layer}")
            if s.name == "head":
                self.head_e_sh = (int(s.e), int(s.sh))
        vec, ln_f = synth.vector_params(seed, g)
        for i, lt in enumerate(g.layer_types):
            p = vec[i]
            self.upload_vector(i, L.VEC_LN1, p["ln1"])
            self.upload_vector(i, L.VEC_LN2, p["ln2"])
            if lt == "full_attention":
                self.upload_vector(i, L.VEC_Q_NORM, p["q_norm"])
                self.upload_vector(i, L.VEC_K_NORM, p["k_norm"])
            else:
                self.upload_vector(i, L.VEC_CONV_W, p["conv_w"])
                self.upload_vector(i, L.VEC_DT_BIAS, p["dt_bias_q12"])
                self.upload_vector(i, L.VEC_A, p["A_q15"])
                self.upload_vector(i, L.VEC_NORM_W, p["norm_w_q14"])
        self.upload_vector(-1, L.VEC_LN_F, ln_f)
        L.check(self.lib.f5_ctx_synth_embedding(self.h, synth.stream_key(seed, synth.MID_EMB, synth.STREAM_E)),
                "synth embedding")

    # ---- state ----
    def reset(self):
        L.check(self.lib.f5_ctx_reset(self.h), "reset")

    def set_position(self, T, pos):
        L.check(self.lib.f5_ctx_set_position(self.h, int(T), int(pos)), "set_position")

    def position(self):
        T, pos = ctypes.c_int(), ctypes.c_int()
        L.check(self.lib.f5_ctx_get_position(self.h, ctypes.byref(T), ctypes.byref(pos)), "get_position")
        return T.value, pos.value

    def set_logits(self, on=True):
        L.check(self.lib.f5_ctx_set_logits(self.h, int(on)), "set_logits")

    def stream_handle(self):
        sp = ctypes.c_void_p()
        L.check(self.lib.f5_ctx_stream(self.h, ctypes.byref(sp)), "f5_ctx_stream")
        return sp.value

    def prepare(self):
        L.check(self.lib.f5_ctx_prepare(self.h), "prepare")

    def set_engine(self, engine):
        """"persistent" (one cooperative launch per step) or "graph" (the
        per-op kernel chain as a CUDA graph); both are bit-exact."""
        code = {"graph": L.ENGINE_GRAPH, "persistent": L.ENGINE_PERSISTENT}[engine]
        L.check(self.lib.f5_ctx_set_engine(self.h, code), "set_engine")

    # ---- row sharding (one process / context per GPU) ----
    def ipc_handle(self):
        """This rank's 64-byte CUDA IPC handle of its dataflow buffers."""
        buf = ctypes.create_string_buffer(64)
        L.check(self.lib.f5_ctx_ipc_handle(self.h, buf, 64), "f5_ctx_ipc_handle")
        return buf.raw

    def attach_peers(self, handles):
        """All ranks' handles in rank order (this rank's own included)."""
        blob = b"".join(handles)
        assert len(blob) == 64 * len(handles)
        buf = ctypes.create_string_buffer(blob, len(blob))
        L.check(self.lib.f5_ctx_attach_peers(self.h, buf, len(handles)), "f5_ctx_attach_peers")

    def trace_step(self):
        """One persistent greedy step with per-op device timestamps ->
        (ns int64[grid, nops, 8] marks relative to the earliest start, -1
        where a CTA has no such mark (see f5_ctx_trace_step), op kinds list).
        Caches advance by one token."""
        grid, nops = ctypes.c_int(), ctypes.c_int()
        L.check(self.lib.f5_ctx_trace_step(self.h, None, 0, ctypes.byref(grid), ctypes.byref(nops)), "trace")
        out = np.zeros(grid.value * nops.value * 8, dtype=np.uint64)
        L.check(self.lib.f5_ctx_trace_step(self.h, _p(out), out.size, ctypes.byref(grid), ctypes.byref(nops)),
                "trace")
        t = out.astype(np.int64).reshape(grid.value, nops.value, 8)
        t0 = t[:, 0, 0].min()
        t = np.where(t > 0, t - t0, -1)
        kinds = ["begin"]
        for lt in self.geom.layer_types:
            core = "attn" if lt == "full_attention" else "dn"
            kinds += [f"{core}_in", core, f"{core}_out", "mlp_gate_up", "mlp_down"]
        kinds.append("head")
        assert len(kinds) == nops.value
        return t, kinds

    def engine(self):
        e = ctypes.c_int()
        L.check(self.lib.f5_ctx_get_engine(self.h, ctypes.byref(e)), "get_engine")
        return {L.ENGINE_GRAPH: "graph", L.ENGINE_PERSISTENT: "persistent"}[e.value]

    # ---- steps ----
    def decode_step(self, tok, pos):
        """One model step (FxRunner.step + argmax) -> (next token, its y32)."""
        nt, mv = ctypes.c_int(), ctypes.c_int()
        L.check(self.lib.f5_decode_step(self.h, int(tok), int(pos), ctypes.byref(nt), ctypes.byref(mv)),
                "f5_decode_step")
        return nt.value, mv.value

    def prefill(self, tokens):
        """Feed a prompt: one step per token from the current position, the
        tokens taken on the device (no host round trip between steps);
        asynchronous.  sync() then returns the argmax after the last token,
        and decode_launch continues greedily from it."""
        t = np.ascontiguousarray(np.asarray(tokens, dtype=np.int32).reshape(-1))
        L.check(self.lib.f5_decode_prefill(self.h, _p(t), int(t.size)), "f5_decode_prefill")

    def decode_launch(self, n):
        L.check(self.lib.f5_decode_launch(self.h, int(n), None), "f5_decode_launch")

    def sync(self):
        nt, mv = ctypes.c_int(), ctypes.c_int()
        L.check(self.lib.f5_ctx_sync(self.h, ctypes.byref(nt), ctypes.byref(mv)), "f5_ctx_sync")
        return nt.value, mv.value

    def time_step(self, reps=3):
        """Per-kernel-class device time of one eager step (CUDA events)."""
        out = np.zeros(8, dtype=np.float64)
        L.check(self.lib.f5_ctx_time_step(self.h, int(reps), _p(out), 8), "f5_ctx_time_step")
        keys = ("gemv_ms", "gemv_bytes", "gemv_launches", "dn_ms", "attn_ms", "other_ms", "sum_ms", "launches")
        return dict(zip(keys, out.tolist()))

    def layer_step(self, layer, x16, T, pos):
        x = np.ascontiguousarray(np.asarray(x16).astype(np.int16))
        L.check(self.lib.f5_layer_step(self.h, int(layer), _p(x), int(T), int(pos)), "f5_layer_step")
        return x.astype(I64)

    # ---- buffers ----
    _SIZES = None

    def read(self, what, layer=0, dtype=np.int16, count=None):
        g = self.geom
        sizes = {L.BUF_X16: (g.H, np.int16), L.BUF_QKV16: (g.CONV_DIM, np.int16), L.BUF_Z16: (g.LVD, np.int16),
                 L.BUF_B16: (g.LNH, np.int16), L.BUF_A16: (g.LNH, np.int16), L.BUF_ON16: (g.LVD, np.int16),
                 L.BUF_QG16: (g.NQ * g.HD * 2, np.int16), L.BUF_K16: (g.NKV * g.HD, np.int16),
                 L.BUF_V16: (g.NKV * g.HD, np.int16), L.BUF_PROD64: (g.NQ * g.HD, I64),
                 L.BUF_PROD16: (g.FFN, np.int16), L.BUF_STATS: (4, np.uint64),
                 L.BUF_DN_S: (g.LNH * g.LDK * g.LDV, np.int16), L.BUF_DN_CONV: (g.CONV_DIM * 4, np.int16),
                 L.BUF_DN_KH: (g.LNH, np.int32), L.BUF_K8: (g.NKV * self.max_T * g.HD, np.int8),
                 L.BUF_KE: (g.NKV * self.max_T, np.int8), L.BUF_V8: (g.NKV * self.max_T * g.HD, np.int8),
                 L.BUF_VE: (g.NKV * self.max_T, np.int8), L.BUF_KA: (1, np.int32),
                 L.BUF_LOGITS: (g.vocab, np.int32), L.BUF_QKVC16: (g.CONV_DIM, np.int16),
                 L.BUF_GATES: (2 * g.LNH, np.int32)}
        n, dt = sizes[what]
        out = np.empty(n, dtype=dt)
        L.check(self.lib.f5_ctx_read(self.h, what, layer, _p(out), out.nbytes), f"read({what})")
        return out

    def write(self, what, layer, arr):
        a = np.ascontiguousarray(arr)
        L.check(self.lib.f5_ctx_write(self.h, what, layer, _p(a), a.nbytes), f"write({what})")

    def logits(self):
        return self.read(L.BUF_LOGITS)

    def stats(self):
        """Saturation counters since the last reset: the DeltaNet state
        writes clipped to int16 (the reference's state["sat"] summed over
        layers), and max |x| / the count of rail values over every layer
        output (FxRunner.resid_max / resid_clip, ref/fidelity_check.py:
        416-433)."""
        s = self.read(L.BUF_STATS)
        return {"dn_sat": int(s[0]), "resid_max": int(s[1]), "resid_clip": int(s[2])}

    # ---- TOPK-32 capture and sampling (sw/chat_seq.py:1776-1928) ----
    def head_logit_exp0(self):
        """Dequant exponent of the head at e_x = 0: e + sh - 15 - RS_F
        (sw/chat_seq.py:355-357 head_logit_exp0 with this model's head)."""
        if self.head_e_sh is None:
            raise RuntimeError("head_logit_exp0: no LM head uploaded")
        e, sh = self.head_e_sh
        return e + sh - 15 - RS_F

    def topk(self):
        """The last step's TOPK-32 capture over the LM head's logits (needs
        set_logits(True) before the step) -> sampling.TopK32Result."""
        from .sampling import TopK32Result
        r = L.TopK32()
        L.check(self.lib.f5_ctx_topk(self.h, ctypes.byref(r)), "f5_ctx_topk")
        return TopK32Result.from_struct(r)

    def sample_step(self, tok, pos, sampler):
        """One decode step whose next token is drawn by `sampler`
        (sampling.Sampler, the reference's temperature / top-k / top-p
        draw over the capture list) -> (token, info)."""
        self.decode_step(tok, pos)
        r = self.topk()
        return sampler.pick(r.values, r.indices, r.e_x)

    # ---- reference-layout state I/O (ref/layer_fixed.py:1654-1666) ----
    def state_image(self, layer):
        """The layer's state in the reference cache layout (f5_state_save),
        at the context's current T, as raw bytes."""
        T, _ = self.position()
        n = self.lib.f5_state_bytes(self.h, int(layer), T)
        buf = np.empty(n, dtype=np.uint8)
        L.check(self.lib.f5_state_save(self.h, int(layer), _p(buf), n), f"state_save({layer})")
        return buf

    def load_state_image(self, layer, img, T):
        img = np.ascontiguousarray(img, dtype=np.uint8).reshape(-1)
        L.check(self.lib.f5_state_load(self.h, int(layer), _p(img), img.size, int(T)), f"state_load({layer})")

    def get_dn_state(self, layer, T):
        """-> {"conv": int64[CONV_DIM, 3] oldest first, "S": int16[LNH, LDK, LDV]}
        at T tokens (the reference's DeltaNet cache dict)."""
        g = self.geom
        T0, pos = self.position()
        if T != T0:
            self.set_position(T, pos)
        try:
            img = self.state_image(layer)
        finally:
            if T != T0:
                self.set_position(T0, pos)
        ns = g.LNH * g.LDK * g.LDV * 2
        return {"S": img[:ns].view(np.int16).reshape(g.LNH, g.LDK, g.LDV).copy(),
                "conv": img[ns:].view(I64).reshape(g.CONV_DIM, 3).copy()}

    def set_dn_state(self, layer, T, cache):
        g = self.geom
        S = np.ascontiguousarray(np.asarray(cache["S"]).astype(np.int16)).reshape(-1).view(np.uint8)
        conv = np.ascontiguousarray(np.asarray(cache["conv"], dtype=I64)).reshape(-1).view(np.uint8)
        assert S.size == g.LNH * g.LDK * g.LDV * 2 and conv.size == g.CONV_DIM * 3 * 8
        self.load_state_image(layer, np.concatenate([S, conv]), T)

    def _kv_arrays(self, layer, T):
        g = self.geom
        T0, pos = self.position()
        if T != T0:
            self.set_position(T, pos)
        try:
            img = self.state_image(layer).view(np.int8)
        finally:
            if T != T0:
                self.set_position(T0, pos)
        n = T * g.NKV
        k8 = img[:n * g.HD].reshape(T, g.NKV, g.HD)
        ke = img[n * g.HD:n * (g.HD + 1)].reshape(T, g.NKV)
        v8 = img[n * (g.HD + 1):n * (2 * g.HD + 1)].reshape(T, g.NKV, g.HD)
        ve = img[n * (2 * g.HD + 1):].reshape(T, g.NKV)
        return k8, ke, v8, ve

    def get_kv(self, layer, T):
        """-> {"k": [[(k8, ke)] * NKV] * T, "v": ...} (ref/layer_fixed.py:1400-1401)"""
        g = self.geom
        k8, ke, v8, ve = self._kv_arrays(layer, T)
        return {"k": [[(k8[t, h].copy(), int(ke[t, h])) for h in range(g.NKV)] for t in range(T)],
                "v": [[(v8[t, h].copy(), int(ve[t, h])) for h in range(g.NKV)] for t in range(T)]}

    def set_kv(self, layer, cache):
        g = self.geom
        T = len(cache["k"])
        assert T <= self.max_T
        k8 = np.zeros((T, g.NKV, g.HD), dtype=np.int8)
        v8 = np.zeros_like(k8)
        ke = np.zeros((T, g.NKV), dtype=np.int8)
        ve = np.zeros_like(ke)
        for t in range(T):
            for h in range(g.NKV):
                k8[t, h], ke[t, h] = cache["k"][t][h]
                v8[t, h], ve[t, h] = cache["v"][t][h]
        self.load_state_image(layer, np.concatenate([a.reshape(-1).view(np.uint8) for a in (k8, ke, v8, ve)]), T)
        return T

    def save_state(self, path, T=None):
        """Every layer's state in the reference cache layout (.npz of the
        f5_state_save images: per DeltaNet layer S [32,128,128] int16 and
        conv [8192,3] int64; per attention layer k8/v8 [T,4,256] int8 and
        ke/ve [T,4] int8), plus T and pos."""
        T0, pos = self.position()
        if T is not None and T != T0:
            raise ValueError(f"save_state: the context holds {T0} tokens, not {T}")
        out = {"T": np.array(T0), "pos": np.array(pos)}
        for i, lt in enumerate(self.geom.layer_types):
            if lt == "full_attention":
                for nm, a in zip(("k8", "ke", "v8", "ve"), self._kv_arrays(i, T0)):
                    out[f"l{i}_{nm}"] = a
            else:
                st = self.get_dn_state(i, T0)
                out[f"l{i}_conv"], out[f"l{i}_S"] = st["conv"], st["S"]
        np.savez(path, **out)

    def load_state(self, path, pos=None):
        d = np.load(path)
        T = int(d["T"])
        for i, lt in enumerate(self.geom.layer_types):
            if lt == "full_attention":
                self.load_state_image(i, np.concatenate([np.ascontiguousarray(d[f"l{i}_{nm}"], dtype=np.int8)
                                                         .reshape(-1).view(np.uint8)
                                                         for nm in ("k8", "ke", "v8", "ve")]), T)
            else:
                self.set_dn_state(i, T, {"conv": d[f"l{i}_conv"], "S": d[f"l{i}_S"]})
        if pos is None:
            pos = int(d["pos"]) if "pos" in d else T
        self.set_position(T, T if pos is None else pos)
        return T

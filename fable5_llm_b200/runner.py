"""Drop-in for the reference's full-model integer step, FxRunner
(ref/fidelity_check.py:404-448), running on the GPU: one persistent decode
launch per step by default (``DecodeModel.set_engine`` selects the per-op
CUDA-graph engine instead; both are bit-exact)."""
from __future__ import annotations

import numpy as np

from . import layer_fixed as LF
from .config import Geometry
from .model import DecodeModel


class FxRunner:
    """Same constructor, attributes and ``step(tok, t) -> y32 logits`` as the
    reference.

    layers_q: per-layer quantized dicts (ref/layer_fixed.py:1607-1651);
    emb_q: int16 [vocab, H]; head: quantized dict; ln_f_q12: (1+w) at Q3.12.
    The DeltaNet gated-norm law follows ``layer_fixed.SEQ_NORM`` at
    construction, like the reference's module global.

    ``caches`` returns the per-layer caches in the reference layout
    (``{"k": [...], "v": [...]}`` lists of (int8[256], e) per KV head, or
    ``{"conv": int64[8192, 3], "S": int16[32, 128, 128]}``), read back from
    the device; ``resid_max`` / ``resid_clip`` are the residual saturation
    counters the reference accumulates after every layer (max |x| and the
    number of words at the int16 rails), kept on the device."""

    def __init__(self, layers_q, layer_types, emb_q, head, ln_f_q12, max_T=4096, device=0):
        self.LF = LF
        self.layers_q = layers_q
        self.types = list(layer_types)
        self.emb_q = emb_q
        self.head = head
        self.ln_f_q12 = ln_f_q12
        vocab = int(np.asarray(head["w4"]).shape[0])
        geom = Geometry(len(self.types), vocab, self.types)
        self.model = DecodeModel(geom, max_T=max_T, norm_mode="eps" if LF.SEQ_NORM else "float",
                                 device=device, max_pos=max(max_T, 4096))
        self.model.upload_model(layers_q, emb_q, head, ln_f_q12)
        self.model.set_logits(True)
        self.reset()

    def reset(self):
        self.model.reset()
        self.last_token = None

    def step(self, tok, t):
        self.last_token, _ = self.model.decode_step(int(tok), int(t))
        return self.model.logits().astype(np.int64)

    @property
    def resid_max(self):
        return self.model.stats()["resid_max"]

    @property
    def resid_clip(self):
        return self.model.stats()["resid_clip"]

    @property
    def caches(self):
        T, _ = self.model.position()
        out = []
        for i, lt in enumerate(self.types):
            if lt == "full_attention":
                out.append(self.model.get_kv(i, T))
            else:
                out.append(self.model.get_dn_state(i, T))
        return out

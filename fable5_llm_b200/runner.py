"""Drop-in for the reference's full-model integer step, FxRunner
(ref/fidelity_check.py:404-448), running the CUDA-graph decode step."""
from __future__ import annotations

import numpy as np

from . import layer_fixed as LF
from .config import Geometry
from .model import DecodeModel


class FxRunner:
    """Same constructor and ``step(tok, t) -> y32 logits`` as the reference.

    layers_q: per-layer quantized dicts (ref/layer_fixed.py:1607-1651);
    emb_q: int16 [vocab, H]; head: quantized dict; ln_f_q12: (1+w) at Q3.12.
    The DeltaNet gated-norm law follows ``layer_fixed.SEQ_NORM`` at
    construction, like the reference's module global."""

    def __init__(self, layers_q, layer_types, emb_q, head, ln_f_q12, max_T=4096, device=0):
        vocab = int(np.asarray(head["w4"]).shape[0])
        geom = Geometry(len(layer_types), vocab, list(layer_types))
        self.model = DecodeModel(geom, max_T=max_T, norm_mode="eps" if LF.SEQ_NORM else "float",
                                 device=device, max_pos=max(max_T, 4096))
        self.model.upload_model(layers_q, emb_q, head, ln_f_q12)
        self.model.set_logits(True)
        self.types = list(layer_types)
        self.reset()

    def reset(self):
        self.model.reset()
        self.last_token = None

    def step(self, tok, t):
        self.last_token, _ = self.model.decode_step(int(tok), int(t))
        return self.model.logits().astype(np.int64)

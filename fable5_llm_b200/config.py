"""Decode geometry of Qwen3.5-9B (ref/layer_ref.py:25-49 over
ref/qwen3_5_9b_config.json) and the fixed-point formats of the 9B operating
point (ref/layer_fixed.py:103-147, 404)."""

RS_F = 7
QKV_F = 8
NRM_F = 14
S_F = 13
GAT_F = 15
CW_F = 13
ROPE_F = 15
DN_NORM_F = 11


class Geometry:
    """9B layer shapes; ``n_layers``/``vocab``/``layer_types`` may be reduced
    for tests (every per-layer shape stays the 9B one)."""

    H = 4096
    NQ = 16
    NKV = 4
    HD = 256
    ROT = 64
    THETA = 10000000.0
    FFN = 12288
    LNH = 32
    LNKH = 16
    LDK = 128
    LDV = 128
    CONV_K = 4
    VREP = LNH // LNKH
    LKD = LNKH * LDK
    LVD = LNH * LDV
    CONV_DIM = 2 * LKD + LVD
    VOCAB = 248320

    def __init__(self, n_layers=32, vocab=248320, layer_types=None):
        if layer_types is None:
            layer_types = [("full_attention" if (i % 4) == 3 else "linear_attention")
                           for i in range(n_layers)]
        assert len(layer_types) == n_layers
        self.n_layers = n_layers
        self.vocab = vocab
        self.layer_types = list(layer_types)

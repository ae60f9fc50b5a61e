"""ctypes binding of ``libf5b200.so`` (the C ABI declared in include/f5b200.h).

The library is the only compute path: if it is missing the import of the
ops fails loudly -- there is no CPU fallback.
"""
from __future__ import annotations

import ctypes
import os

_HERE = os.path.dirname(os.path.abspath(__file__))
LIB_PATH = os.path.join(_HERE, "_lib", "libf5b200.so")

c_int, c_ll, c_u64, c_vp, c_size = (ctypes.c_int, ctypes.c_longlong, ctypes.c_uint64,
                                    ctypes.c_void_p, ctypes.c_size_t)

F5_OK, F5_EINVAL, F5_ECUDA, F5_ENOMEM, F5_ETIMEOUT, F5_EOVERFLOW, F5_ESTATE, F5_ENCCL = \
    0, -1, -2, -3, -4, -5, -6, -7

GM_Y32, GM_TO16, GM_TO64, GM_RESID, GM_SILU_MUL, GM_ARGMAX = range(6)
ENGINE_GRAPH, ENGINE_PERSISTENT = 0, 1
(PR_RSHR, PR_SIGMOID, PR_SOFTPLUS, PR_SILU, PR_EXP_NEG, PR_RSQRT, PR_RECIP,
 PR_BF_SHIFT, PR_DYNQ8_E, PR_DN_NORM_SCALE, PR_EPS_NORM_SCALE, PR_EXP2_FRAC) = range(12)


class F5Error(RuntimeError):
    def __init__(self, status, msg):
        super().__init__(f"f5b200 status {status}: {msg}")
        self.status = status


class TopK32(ctypes.Structure):
    """f5_topk32 (include/f5b200.h)."""
    _fields_ = [("val", ctypes.c_int32 * 32), ("idx", ctypes.c_int32 * 32), ("count", ctypes.c_int32),
                ("ovf_lit", ctypes.c_int32), ("ovf_disp", ctypes.c_int32), ("amax_idx", ctypes.c_int32),
                ("amax_val", ctypes.c_int32), ("e_x", ctypes.c_int32), ("n", ctypes.c_int32)]


class GemvSeg(ctypes.Structure):
    _fields_ = [("w", c_vp), ("w2", c_vp), ("out", c_vp), ("p_out", c_vp),
                ("rows", c_int), ("e", c_int), ("e2", c_int), ("out_f", c_int),
                ("out_f2", c_int), ("mode", c_int), ("out_row0", c_int)]


# (name, restype, argtypes) of every exported symbol, in header order
SIGNATURES = [
    ("f5_abi_version", c_int, []),
    ("f5_status_string", ctypes.c_char_p, [c_int]),
    ("f5_last_error", c_int, [ctypes.c_char_p, c_size]),
    ("f5_gemv_dev", c_int, [ctypes.POINTER(GemvSeg), c_int, c_int, c_int, c_int, c_vp, c_vp,
                            c_vp, c_vp, c_int, c_int, c_vp]),
    ("f5_rmsnorm_dynq8_dev", c_int, [c_vp, c_vp, c_int, c_int, c_int, c_vp, c_vp, c_vp, c_vp]),
    ("f5_dynq8_dev", c_int, [c_vp, c_int, c_int, c_vp, c_vp, c_vp]),
    ("f5_prim_dev", c_int, [c_int, c_vp, c_vp, c_vp, c_vp, c_int, c_int, c_int, c_vp]),
    ("f5_synth_w4_dev", c_int, [c_vp, c_ll, c_int, c_int, c_ll, c_u64, c_u64, c_int, c_vp]),
    ("f5_synth_emb_dev", c_int, [c_vp, c_ll, c_int, c_ll, c_u64, c_vp]),
    ("f5_quant_w4_scales", c_int, [c_vp, c_int, c_int, c_int, c_int, c_vp, c_int, c_vp, c_vp, c_vp, c_vp]),
    ("f5_quant_w4_pack", c_int, [c_vp, c_int, c_int, c_int, c_int, c_vp, c_int, c_vp, c_vp, c_vp, c_vp]),
    ("f5_batch_matvec_ws_bytes", c_size, [c_int, c_int, c_int]),
    ("f5_batch_trace", c_int, [c_int, c_vp, c_size]),
    ("f5_batch_matvec_y32_dev", c_int, [c_vp, c_int, c_int, c_int, c_int, c_vp, c_int, c_vp, c_vp, c_vp,
                                        c_size, c_vp, c_vp]),
    ("f5_bctx_create", c_int, [c_vp, c_int, c_int, c_vp]),
    ("f5_bctx_destroy", c_int, [c_vp]),
    ("f5_bctx_reset", c_int, [c_vp]),
    ("f5_bctx_set_position", c_int, [c_vp, c_int, c_int, c_int]),
    ("f5_bctx_get_position", c_int, [c_vp, c_int, c_vp, c_vp]),
    ("f5_bctx_step", c_int, [c_vp, c_vp, c_vp, c_vp]),
    ("f5_bctx_prefill", c_int, [c_vp, c_int, c_vp, c_int, c_vp, c_vp]),
    ("f5_bctx_launch", c_int, [c_vp, c_int]),
    ("f5_bctx_sync", c_int, [c_vp, c_vp, c_vp]),
    ("f5_bctx_stream", c_int, [c_vp, c_vp]),
    ("f5_bctx_time_step", c_int, [c_vp, c_int, c_vp, c_int]),
    ("f5_bctx_set_logits", c_int, [c_vp, c_int]),
    ("f5_bctx_topk", c_int, [c_vp, c_vp]),
    ("f5_bctx_read", c_int, [c_vp, c_int, c_int, c_int, c_vp, c_size]),
    ("f5_bctx_write", c_int, [c_vp, c_int, c_int, c_int, c_vp, c_size]),
    ("f5_matvec_y32_host", c_int, [c_vp, c_int, c_int, c_int, c_int, c_vp, c_vp, c_vp]),
    ("f5_matvec_y32_host_noalloc", c_int, [c_vp, c_int, c_int, c_int, c_int, c_vp, c_vp, c_vp]),
    ("f5_ctx_create", c_int, [c_vp, c_int, c_vp]),
    ("f5_ctx_destroy", c_int, [c_vp]),
    ("f5_ctx_upload_matrix", c_int, [c_vp, c_int, c_int, c_vp, c_int, c_int, c_int, c_int, c_int]),
    ("f5_ctx_synth_matrix", c_int, [c_vp, c_int, c_int, c_int, c_int, c_int, c_int, c_int, c_u64, c_u64,
                                    c_int]),
    ("f5_ctx_upload_vector", c_int, [c_vp, c_int, c_int, c_vp, c_int]),
    ("f5_ctx_upload_embedding", c_int, [c_vp, c_vp, c_int, c_int]),
    ("f5_ctx_synth_embedding", c_int, [c_vp, c_u64]),
    ("f5_ctx_upload_rope", c_int, [c_vp, c_vp, c_int]),
    ("f5_ctx_reset", c_int, [c_vp]),
    ("f5_ctx_set_position", c_int, [c_vp, c_int, c_int]),
    ("f5_ctx_get_position", c_int, [c_vp, c_vp, c_vp]),
    ("f5_ctx_set_logits", c_int, [c_vp, c_int]),
    ("f5_topk32_ws_bytes", c_size, [c_ll]),
    ("f5_topk32_dev", c_int, [c_vp, c_ll, c_vp, c_vp, c_vp]),
    ("f5_topk32_host", c_int, [c_vp, c_ll, c_vp]),
    ("f5_ctx_topk", c_int, [c_vp, c_vp]),
    ("f5_ctx_stream", c_int, [c_vp, c_vp]),
    ("f5_ctx_prepare", c_int, [c_vp]),
    ("f5_ctx_set_engine", c_int, [c_vp, c_int]),
    ("f5_ctx_get_engine", c_int, [c_vp, c_vp]),
    ("f5_ctx_ipc_handle", c_int, [c_vp, c_vp, c_size]),
    ("f5_ctx_attach_peers", c_int, [c_vp, c_vp, c_int]),
    ("f5_ctx_trace_step", c_int, [c_vp, c_vp, c_size, c_vp, c_vp]),
    ("f5_decode_step", c_int, [c_vp, c_int, c_int, c_vp, c_vp]),
    ("f5_decode_launch", c_int, [c_vp, c_int, c_vp]),
    ("f5_decode_prefill", c_int, [c_vp, c_vp, c_int]),
    ("f5_ctx_sync", c_int, [c_vp, c_vp, c_vp]),
    ("f5_ctx_time_step", c_int, [c_vp, c_int, c_vp, c_int]),
    ("f5_layer_step", c_int, [c_vp, c_int, c_vp, c_int, c_int]),
    ("f5_state_bytes", c_size, [c_vp, c_int, c_int]),
    ("f5_state_save", c_int, [c_vp, c_int, c_vp, c_size]),
    ("f5_state_load", c_int, [c_vp, c_int, c_vp, c_size, c_int]),
    ("f5_ctx_read", c_int, [c_vp, c_int, c_int, c_vp, c_size]),
    ("f5_ctx_write", c_int, [c_vp, c_int, c_int, c_vp, c_size]),
]

# f5_config (include/f5b200.h)
class Config(ctypes.Structure):
    _fields_ = [("abi_version", c_int), ("n_layers", c_int), ("vocab", c_int), ("max_T", c_int),
                ("norm_mode", c_int), ("world_size", c_int), ("rank", c_int),
                ("layer_types", ctypes.c_char_p)]


S_IN_QKV, S_IN_Z, S_IN_B, S_IN_A, S_OUT = 0, 1, 2, 3, 4
S_Q, S_K, S_V, S_O = 0, 1, 2, 3
S_GATE, S_UP, S_DOWN, S_HEAD = 8, 9, 10, 0
VEC_LN1, VEC_LN2, VEC_Q_NORM, VEC_K_NORM, VEC_CONV_W, VEC_DT_BIAS, VEC_A, VEC_NORM_W, VEC_LN_F = range(9)
(BUF_X16, BUF_QKV16, BUF_Z16, BUF_B16, BUF_A16, BUF_ON16, BUF_QG16, BUF_K16, BUF_V16, BUF_PROD64,
 BUF_PROD16, BUF_STATS, BUF_DN_S, BUF_DN_CONV, BUF_DN_KH, BUF_K8, BUF_KE, BUF_V8, BUF_VE, BUF_KA,
 BUF_LOGITS, BUF_QKVC16, BUF_GATES) = range(23)

_LIB = None


def lib():
    """Load the library once (raises if it has not been built)."""
    global _LIB
    if _LIB is None:
        if not os.path.exists(LIB_PATH):
            raise RuntimeError(f"CUDA library {LIB_PATH} is not built "
                               "(python -m fable5_llm_b200.build); there is no CPU fallback")
        L = ctypes.CDLL(LIB_PATH)
        for name, res, args in SIGNATURES:
            fn = getattr(L, name)
            fn.restype = res
            fn.argtypes = args
        _LIB = L
    return _LIB


def last_error():
    buf = ctypes.create_string_buffer(512)
    lib().f5_last_error(buf, 512)
    return buf.value.decode(errors="replace")


def check(status, what=""):
    if status != F5_OK:
        raise F5Error(status, f"{what}: {last_error()}")
    return status

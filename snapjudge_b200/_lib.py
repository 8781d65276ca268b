"""ctypes binding of ``lib/libsnapjudge_b200.so`` (the C ABI in include/snapjudge_b200.h).

The library is the product: there is no fallback.  Loading fails loudly when
the in-tree build is missing (run ``python snapjudge_b200/build.py`` or
``__graft_entry__.build()``).
"""
from __future__ import annotations

import ctypes as C
import os

LIB_PATH = os.path.join(os.path.dirname(os.path.abspath(__file__)), "lib",
                        "libsnapjudge_b200.so")

SJ_OK = 0
SJ_ERR_INVALID = -1
SJ_ERR_CUDA = -2
SJ_ERR_UNSUPPORTED = -3
SJ_ERR_TIMEOUT = -4
SJ_ERR_STATE = -5
SJ_PREC_BF16 = 0
SJ_PREC_FP32 = 1
SJ_PREC_FP8 = 2
SJ_PREC_FP8_TENSOR = 3
SJ_ARCH_MODERNBERT = 0
SJ_ARCH_SJMODEL = 1

# every symbol declared in include/snapjudge_b200.h
EXPORTS = ["sj_b200_version", "sj_last_error", "sj_gemm", "sj_gemm_geglu", "sj_add_ln", "sj_rope",
           "sj_attn", "sj_attn_noalloc", "sj_check_device_errors", "sj_test_attn_wait_timeout",
           "sj_quant_e4m3", "sj_gemm_e4m3", "sj_fast_create", "sj_fast_set_tensor", "sj_fast_set_heads",
           "sj_fast_commit", "sj_fast_encode", "sj_fast_embed", "sj_fast_decide", "sj_fast_forward", "sj_fast_n_act",
           "sj_fast_encode_device",
           "sj_fast_sync", "sj_fast_launch_count", "sj_fast_set_profiling", "sj_fast_profile",
           "sj_fast_reset_calibration",
           "sj_fast_last_error", "sj_fast_destroy"]

# kernel classes of sj_fast_profile (SJ_K_* in the header)
KERNEL_CLASSES = ["embed", "ln", "qkv", "attn", "wo", "geglu", "wo2", "final"]


class SnapjudgeError(RuntimeError):
    def __init__(self, code: int, msg: str):
        super().__init__(f"[{code}] {msg}")
        self.code = code


class FastConfig(C.Structure):
    _fields_ = [("hidden_size", C.c_int), ("num_hidden_layers", C.c_int),
                ("num_attention_heads", C.c_int), ("intermediate_size", C.c_int),
                ("vocab_size", C.c_int), ("max_position_embeddings", C.c_int),
                ("norm_eps", C.c_float), ("local_attention", C.c_int),
                ("layer_sliding", C.POINTER(C.c_int)), ("rope_theta_full", C.c_double),
                ("rope_theta_sliding", C.c_double), ("precision", C.c_int),
                ("device", C.c_int), ("max_tokens", C.c_int), ("arch", C.c_int)]


_LIB = None
_P = C.c_void_p
_I = C.c_int


def lib() -> C.CDLL:
    global _LIB
    if _LIB is None:
        if not os.path.exists(LIB_PATH):
            raise ImportError(f"snapjudge_b200 extension not built: {LIB_PATH} is missing "
                              "(run `python snapjudge_b200/build.py`)")
        L = C.CDLL(LIB_PATH)
        L.sj_last_error.restype = C.c_char_p
        L.sj_fast_last_error.restype = C.c_char_p
        L.sj_fast_last_error.argtypes = [_P]
        L.sj_gemm.argtypes = [_P, _P, _P, _P, _I, _I, _I, _I, _I, _P]
        L.sj_gemm_geglu.argtypes = [_P, _P, _P, _I, _I, _I, _P]
        L.sj_add_ln.argtypes = [_P, _P, _P, _P, _P, _I, _I, C.c_float, _I, _I, _P]
        L.sj_rope.argtypes = [_P, _P, _P, _P, _P, _I, _I, _I, _P]
        L.sj_attn.argtypes = [_P, _P, _P, _P, _P, _I, _I, _I, _I, _P]
        L.sj_attn_noalloc.argtypes = [_P, _P, _P, _P, _P, _I, _I, _I, _I, _P]
        L.sj_check_device_errors.argtypes = [_P]
        L.sj_test_attn_wait_timeout.argtypes = [_I]
        L.sj_test_attn_wait_timeout.restype = None
        L.sj_quant_e4m3.argtypes = [_P, C.c_int64, _I, _P, _P, _P]
        L.sj_gemm_e4m3.argtypes = [_P, _P, _P, _P, _P, _P, _I, _I, _I, _I, _I, _I, _P]
        L.sj_fast_create.argtypes = [C.POINTER(FastConfig), C.POINTER(_P)]
        L.sj_fast_set_tensor.argtypes = [_P, C.c_char_p, _P, C.POINTER(C.c_int64), _I]
        L.sj_fast_set_heads.argtypes = [_P, _I, C.POINTER(_I), C.POINTER(_I)]
        L.sj_fast_commit.argtypes = [_P]
        L.sj_fast_encode.argtypes = [_P, _P, _P, _P, _I, _P]
        L.sj_fast_decide.argtypes = [_P, _P, _P, _I, _P]
        L.sj_fast_embed.argtypes = [_P, _P, _P, _I, _P]
        L.sj_fast_forward.argtypes = [_P, _P, _P, _P, _I, _P, _P, _I, _P, _P, _P]
        L.sj_fast_n_act.argtypes = [_P]
        L.sj_fast_encode_device.argtypes = [_P, _P, _P, _P, _P, _I, _P, _P, _P]
        L.sj_fast_sync.argtypes = [_P, _P]
        L.sj_fast_launch_count.argtypes = [_P]
        L.sj_fast_set_profiling.argtypes = [_P, _I]
        L.sj_fast_reset_calibration.argtypes = [_P]
        L.sj_fast_profile.argtypes = [_P, C.POINTER(C.c_double), C.POINTER(C.c_int64), _I]
        L.sj_fast_destroy.argtypes = [_P]
        _LIB = L
    return _LIB


def check(rc: int, engine=None) -> None:
    """Raise SnapjudgeError for a non-zero status, with the library's message."""
    if rc == SJ_OK:
        return
    L = lib()
    msg = (L.sj_fast_last_error(engine) if engine else L.sj_last_error()) or b""
    raise SnapjudgeError(rc, msg.decode(errors="replace"))

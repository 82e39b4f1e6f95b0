"""ctypes binding of libsupra_attn (include/supra_attn.h).

Loading fails loudly: there is no CPU or eager fallback. If the shared library is missing the
import raises ImportError telling how to build it.
"""

from __future__ import annotations

import ctypes as C
import os

_HERE = os.path.dirname(os.path.abspath(__file__))
LIB_PATH = os.environ.get("SUPRA_ATTN_LIB", os.path.join(_HERE, "libsupra_attn.so"))

OK, EINVAL, ENOMEM, ECUDA, ETIMEOUT, EDEVICE, ESTATE = range(7)
FP32, TF32, TF32X3 = 0, 1, 2
F_DEFAULT_SCALE = 0x1
F_T5_TABLE = 0x2


class Desc(C.Structure):
    """supra_attn_desc (include/supra_attn.h)."""

    _fields_ = [
        ("q", C.c_void_p), ("k", C.c_void_p), ("v", C.c_void_p), ("out", C.c_void_p), ("bias", C.c_void_p),
        ("q_size", C.c_int64), ("k_size", C.c_int64), ("v_size", C.c_int64), ("out_size", C.c_int64),
        ("bias_size", C.c_int64),
        ("ldq", C.c_int64), ("ldk", C.c_int64), ("ldv", C.c_int64),
        ("q_off", C.c_int64), ("k_off", C.c_int64), ("v_off", C.c_int64), ("o_off", C.c_int64),
        ("Lq", C.c_int32), ("Lk", C.c_int32), ("H", C.c_int32), ("D", C.c_int32),
        ("scale", C.c_float), ("variant", C.c_int32), ("flags", C.c_uint32), ("bias_param", C.c_uint32),
    ]


class GroupNorm(C.Structure):
    """supra_attn_groupnorm (include/supra_attn.h)."""

    _fields_ = [("gamma", C.c_void_p), ("beta", C.c_void_p), ("groups", C.c_int32), ("rows_per_image", C.c_int32),
                ("eps", C.c_float), ("silu", C.c_int32)]


class LayerNorm(C.Structure):
    """supra_attn_layernorm (include/supra_attn.h)."""

    _fields_ = [("mod", C.c_void_p), ("mod_size", C.c_int64), ("shift_off", C.c_int64), ("scale_off", C.c_int64),
                ("eps", C.c_float), ("reserved", C.c_int32)]


class LinearDesc(C.Structure):
    """supra_attn_linear_desc (include/supra_attn.h)."""

    _fields_ = [
        ("x", C.c_void_p), ("w", C.c_void_p), ("bias", C.c_void_p), ("y", C.c_void_p),
        ("x_size", C.c_int64), ("w_size", C.c_int64), ("bias_size", C.c_int64), ("y_size", C.c_int64),
        ("ldx", C.c_int64), ("ldw", C.c_int64), ("ldy", C.c_int64), ("x_off", C.c_int64), ("y_off", C.c_int64),
        ("M", C.c_int32), ("N", C.c_int32), ("K", C.c_int32),
        ("variant", C.c_int32), ("flags", C.c_uint32), ("act", C.c_uint32),
        ("gn", C.POINTER(GroupNorm)), ("resid", C.c_void_p), ("resid_size", C.c_int64), ("ldr", C.c_int64),
        ("r_off", C.c_int64), ("gate", C.c_void_p), ("gate_size", C.c_int64), ("g_off", C.c_int64),
        ("ln", C.POINTER(LayerNorm)),
    ]


class ProfileEntry(C.Structure):
    _fields_ = [("name", C.c_char * 48), ("launches", C.c_int64), ("ms", C.c_double), ("flops", C.c_double),
                ("bytes", C.c_double)]


# (name, restype, argtypes) for every exported function; tests check the list against the header.
SIGNATURES = [
    ("supra_attn_create", C.c_int, [C.c_int, C.POINTER(C.c_void_p)]),
    ("supra_attn_destroy", C.c_int, [C.c_void_p]),
    ("supra_attn_set_stream", C.c_int, [C.c_void_p, C.c_void_p]),
    ("supra_attn_last_error", C.c_char_p, [C.c_void_p]),
    ("supra_attn_status_string", C.c_char_p, [C.c_int]),
    ("supra_attn_tensor_alloc", C.c_int, [C.c_void_p, C.c_int64, C.POINTER(C.c_void_p)]),
    ("supra_attn_tensor_free", C.c_int, [C.c_void_p, C.c_void_p]),
    ("supra_attn_upload", C.c_int, [C.c_void_p, C.c_void_p, C.c_void_p, C.c_int64]),
    ("supra_attn_download", C.c_int, [C.c_void_p, C.c_void_p, C.c_void_p, C.c_int64]),
    ("supra_attn_host_alloc", C.c_int, [C.c_void_p, C.c_int64, C.POINTER(C.c_void_p)]),
    ("supra_attn_host_free", C.c_int, [C.c_void_p, C.c_void_p]),
    ("supra_attn_enqueue", C.c_int, [C.c_void_p, C.POINTER(Desc)]),
    ("supra_attn_check_desc", C.c_int, [C.POINTER(Desc), C.c_char_p, C.c_int32]),
    ("supra_attn_enqueue_batch", C.c_int, [C.c_void_p, C.POINTER(Desc), C.c_int32]),
    ("supra_attn_flush", C.c_int, [C.c_void_p]),
    ("supra_attn_sync", C.c_int, [C.c_void_p, C.POINTER(C.c_int32)]),
    ("supra_attn_pending", C.c_int, [C.c_void_p, C.POINTER(C.c_int32)]),
    ("supra_attn_relative_bucket", C.c_int32, [C.c_int32, C.c_int32, C.c_int32]),
    ("supra_attn_position_bias", C.c_int,
     [C.c_void_p, C.c_void_p, C.c_int64, C.c_int32, C.c_int32, C.c_int32, C.c_int32, C.c_void_p, C.c_int64]),
    ("supra_attn_profile_enable", C.c_int, [C.c_void_p, C.c_int32]),
    ("supra_attn_profile_report", C.c_int, [C.c_void_p, C.POINTER(ProfileEntry), C.c_int32, C.POINTER(C.c_int32)]),
    ("supra_attn_profile_reset", C.c_int, [C.c_void_p]),
    ("supra_attn_launch_count", C.c_int, [C.c_void_p, C.POINTER(C.c_int64)]),
    ("supra_attn_attention_noalloc", C.c_int, [C.POINTER(Desc), C.c_void_p, C.c_char_p, C.c_int32]),
    ("supra_attn_enqueue_linear", C.c_int, [C.c_void_p, C.POINTER(LinearDesc)]),
    ("supra_attn_check_linear_desc", C.c_int, [C.POINTER(LinearDesc), C.c_char_p, C.c_int32]),
]


def _load():
    if not os.path.exists(LIB_PATH):
        raise ImportError(
            f"libsupra_attn.so not found at {LIB_PATH}; build it with "
            "`python supra2-img-web_b200/supra_attn/build.py` (needs nvcc). There is no fallback.")
    lib = C.CDLL(LIB_PATH)
    for name, res, args in SIGNATURES:
        f = getattr(lib, name)
        f.restype = res
        f.argtypes = args
    return lib


lib = _load()


class SupraAttnError(RuntimeError):
    """A non-OK status from libsupra_attn, with the context's message."""

    def __init__(self, status: int, message: str):
        self.status = status
        super().__init__(f"{lib.supra_attn_status_string(status).decode()}: {message}")


class SupraAttnValueError(SupraAttnError, ValueError):
    """EINVAL: the call was rejected synchronously (the reference throws, app/gpu/ops.js:122)."""


def check(status: int, ctx=None):
    if status == OK:
        return
    msg = lib.supra_attn_last_error(ctx).decode() if ctx else ""
    if status == EINVAL:
        raise SupraAttnValueError(status, msg)
    raise SupraAttnError(status, msg)

"""ctypes binding of libreels_lowvram.so (declared in include/reels_lowvram.h).

The library is located like the reference locates its native SentencePiece
bridge (src/models/wan21/tokenizer.jl:5-17): an environment override
(``REELS_LOWVRAM_LIBRARY``), else the in-tree build next to this file.  There
is no fallback: if the library is missing every compute call raises.
"""
from __future__ import annotations

import ctypes
import os
import threading

HERE = os.path.dirname(os.path.abspath(__file__))
LIB_NAME = "libreels_lowvram.so"

F32, F16, BF16 = 0, 1, 2
W_OUT_CONTIGUOUS, W_IN_CONTIGUOUS = 0, 1
PASS_FORWARD, PASS_BACKWARD, PASS_DROPOUT = 0, 1, 2
PATH_NONE, PATH_TENSORCORE, PATH_CUDACORE = 0, 1, 2
ACT_NONE, ACT_GELU_TANH = 0, 1
OK, EINVAL, EDEVICE = 0, -1, -2

class OptTensor(ctypes.Structure):
    """reels_opt_tensor: one parameter tensor of the optimizer step."""
    _fields_ = [("param", ctypes.c_void_p), ("grad", ctypes.c_void_p), ("m", ctypes.c_void_p),
                ("v", ctypes.c_void_p), ("master", ctypes.c_void_p), ("n", ctypes.c_int64),
                ("param_dtype", ctypes.c_int), ("decay", ctypes.c_int)]


# Every symbol the header declares, with (restype, argtypes).
_vp = ctypes.c_void_p
_i64 = ctypes.c_int64
_int = ctypes.c_int
_f = ctypes.c_float
_sz = ctypes.c_size_t
SIGNATURES = {
    "reels_lowvram_last_error": (ctypes.c_char_p, []),
    "reels_lowvram_abi_version": (_int, []),
    "reels_lowvram_last_path": (_int, []),
    "reels_q8_plan": (_int, [_i64, _i64, _i64, _int, _int, ctypes.POINTER(ctypes.c_int64)]),
    "reels_sk_plan": (_int, [_i64, _i64, _i64, _int, ctypes.POINTER(ctypes.c_int64)]),
    "reels_sk_dual_plan": (_int, [_i64, _i64, _i64, _int, ctypes.POINTER(ctypes.c_int64)]),
    "reels_lowvram_check_device_status": (_int, [_vp]),
    "reels_lowvram_profile_enable": (_int, [_int]),
    "reels_lowvram_profile_read": (_int, [ctypes.POINTER(ctypes.c_double), ctypes.POINTER(ctypes.c_int64),
                                          ctypes.POINTER(ctypes.c_double), ctypes.POINTER(ctypes.c_int64)]),
    "reels_q8_quantize": (_int, [_vp, _int, _int, _i64, _i64, _vp, _vp, _vp]),
    "reels_q8_materialize": (_int, [_vp, _vp, _int, _i64, _i64, _int, _vp, _vp]),
    "reels_q8lora_workspace_bytes": (_sz, [_i64, _i64, _i64, _i64, _int, _int]),
    "reels_q8lora_saved_bytes": (_sz, [_i64, _i64, _int]),
    "reels_q8_weight_mul": (_int, [_vp, _vp, _vp, _int, _vp, _i64, _i64, _i64, _int, _vp, _vp, _sz, _vp]),
    "reels_q8_weight_transpose_mul": (_int, [_vp, _vp, _vp, _int, _i64, _i64, _i64, _int, _vp, _vp, _sz, _vp]),
    "reels_q8lora_forward": (_int, [_vp, _vp, _vp, _int, _vp, _vp, _vp, _i64, _i64, _i64, _i64, _f, _int,
                                    _vp, _vp, _vp, _sz, _vp]),
    "reels_q8lora_backward": (_int, [_vp, _vp, _vp, _vp, _int, _vp, _vp, _vp, _i64, _i64, _i64, _i64, _f, _f,
                                     _int, _vp, _vp, _vp, _int, _vp, _sz, _vp]),
    "reels_q8lora_forward_static_ws": (_int, [_vp, _vp, _vp, _int, _vp, _vp, _vp, _i64, _i64, _i64, _i64, _f,
                                              _int, _vp, _vp, _vp]),
    "reels_q8lora_forward_act": (_int, [_vp, _vp, _vp, _int, _vp, _vp, _vp, _i64, _i64, _i64, _i64, _f, _int,
                                        _int, _vp, _vp, _vp, _vp, _sz, _vp]),
    "reels_q8lora_backward_act": (_int, [_vp, _vp, _vp, _vp, _int, _vp, _vp, _vp, _i64, _i64, _i64, _i64, _f, _f,
                                         _int, _int, _vp, _vp, _vp, _vp, _int, _vp, _sz, _vp]),
    "reels_q8lora_forward_dropout": (_int, [_vp, _vp, _vp, _int, _vp, _vp, _vp, _i64, _i64, _i64, _i64, _f, _int,
                                            _f, ctypes.c_uint64, ctypes.c_uint64, _vp, _vp, _vp, _sz, _vp]),
    "reels_q8lora_backward_dropout": (_int, [_vp, _vp, _vp, _vp, _int, _vp, _vp, _vp, _i64, _i64, _i64, _i64, _f,
                                             _f, _int, _f, ctypes.c_uint64, ctypes.c_uint64, _vp, _vp, _vp, _int, _vp,
                                             _sz, _vp]),
    "reels_dropout_mask": (_int, [_i64, _f, ctypes.c_uint64, ctypes.c_uint64, _vp, _vp]),
    "reels_layernorm_modulate": (_int, [_vp, _i64, _i64, _i64, _vp, _vp, _vp, _vp, _f, _int, _vp, _vp]),
    "reels_layernorm_modulate_workspace_bytes": (_sz, [_i64, _i64, _i64]),
    "reels_layernorm_modulate_backward": (_int, [_vp, _vp, _i64, _i64, _i64, _vp, _vp, _vp, _f, _int, _vp, _vp, _vp,
                                                 _int, _vp, _sz, _vp]),
    "reels_gated_residual": (_int, [_vp, _vp, _vp, _i64, _i64, _i64, _int, _vp, _vp]),
    "reels_gated_residual_workspace_bytes": (_sz, [_i64, _i64, _i64]),
    "reels_gated_residual_backward": (_int, [_vp, _vp, _vp, _i64, _i64, _i64, _int, _vp, _vp, _int, _vp, _sz, _vp]),
    "reels_opt_workspace_bytes": (_sz, [_int]),
    "reels_opt_prepare": (_int, [ctypes.POINTER(OptTensor), _int, _vp, _sz, _vp]),
    "reels_grad_norm_sq": (_int, [_vp, _f, _vp, _vp]),
    "reels_adamw_update": (_int, [_vp, _f, _f, _f, _f, _f, _f, _f, _f, _vp, _f, _vp]),
}

_lock = threading.Lock()
_lib = None


class NativeError(RuntimeError):
    """A native call returned a non-zero status."""

    def __init__(self, op: str, code: int, message: str):
        super().__init__(f"{op} failed ({code}): {message}")
        self.code = code


def library_path() -> str:
    configured = os.environ.get("REELS_LOWVRAM_LIBRARY", "")
    return configured or os.path.join(HERE, LIB_NAME)


def lib():
    """Load (once) and return the native library; raise if it is missing."""
    global _lib
    with _lock:
        if _lib is None:
            path = library_path()
            if not os.path.isfile(path):
                raise RuntimeError(
                    f"native low-VRAM library not found at {path}; build it with "
                    "`python -m reels_b200.build` or set REELS_LOWVRAM_LIBRARY")
            L = ctypes.CDLL(path)
            for name, (res, args) in SIGNATURES.items():
                fn = getattr(L, name)
                fn.restype = res
                fn.argtypes = args
            _lib = L
    return _lib


def check(op: str, code: int) -> None:
    if code != OK:
        msg = lib().reels_lowvram_last_error().decode(errors="replace")
        if code == EINVAL:
            raise ValueError(f"{op}: {msg}")
        raise NativeError(op, code, msg)


def last_path() -> int:
    return lib().reels_lowvram_last_path()


def profile_enable(on: bool = True) -> None:
    lib().reels_lowvram_profile_enable(1 if on else 0)


def profile_read():
    """(q8_ms, q8_launches, q8_flops, kernel_launches) since the last read."""
    ms, fl = ctypes.c_double(), ctypes.c_double()
    n, k = ctypes.c_int64(), ctypes.c_int64()
    check("profile_read", lib().reels_lowvram_profile_read(ctypes.byref(ms), ctypes.byref(n), ctypes.byref(fl),
                                                           ctypes.byref(k)))
    return ms.value, n.value, fl.value, k.value

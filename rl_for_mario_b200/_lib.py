"""ctypes binding of the C-ABI library (include/dt_attn.h).

The library is loaded from ``rl_for_mario_b200/_native/libdt_attn_sm100.so``.
There is no fallback: if the library is missing every call raises
``DTKernelUnavailable`` (build it with ``python -m rl_for_mario_b200.build``).
"""
from __future__ import annotations

import ctypes
import threading
from pathlib import Path

LIB_PATH = Path(__file__).resolve().parent / "_native" / "libdt_attn_sm100.so"

DT_OK = 0
DT_ERR_INVALID = 1
DT_ERR_UNSUPPORTED = 2
DT_ERR_CUDA = 3
DT_ERR_DEVICE = 4

DT_DTYPE_BF16 = 0
DT_DTYPE_FP16 = 1
DT_DTYPE_FP32 = 2

_P = ctypes.c_void_p
_I = ctypes.c_int
_L = ctypes.c_int64
_F = ctypes.c_float
_U = ctypes.c_uint32

# Exported symbol -> (restype, argtypes).  Kept in the order of include/dt_attn.h.
SIGNATURES = {
    "dt_version": (_I, []),
    "dt_last_error": (ctypes.c_char_p, []),
    "dt_device_status": (_I, [_P]),
    "dt_attn_prefill": (_I, [_P, _P, _P, _P, _P, _P, _I, _L, _P, _I, _I, _I, _I, _I,
                             _L, _L, _L, _L, _L, _L, _L, _L, _L, _L, _L, _L, _F, _I, _I, _P]),
    "dt_attn_decode": (_I, [_P, _P, _P, _P, _P, _P, _I, _I, _P, _I, _P, _P, _P, _P, _I, _L, _I,
                            _I, _I, _I, _I, _I, _L, _L, _L, _L, _L, _L, _L, _L, _L, _L, _L, _L,
                            _F, _I, _I, _P]),
    "dt_kv_write": (_I, [_P, _P, _P, _P, _I, _I, _P, _I, _P, _P, _P, _I, _L, _I, _I, _I, _I, _I,
                         _L, _L, _L, _L, _L, _L, _I, _I, _P]),
    "dt_rmsnorm_qkv": (_I, [_P, _L, _P, _P, _L, _I, _I, _I, _F, _I, _P]),
    "dt_rmsnorm_qkv_rope": (_I, [_P, _L, _P, _P, _L, _I, _I, _I, _F, _P, _P, _L, _I, _I, _I, _I, _I, _P]),
    "dt_rmsnorm_swiglu": (_I, [_P, _L, _P, _P, _L, _I, _I, _I, _F, _I, _P]),
    "dt_gemm_residual": (_I, [_P, _L, _P, _P, _L, _I, _I, _I, _I, _P]),
    "dt_qkv_rope": (_I, [_P, _L, _P, _P, _L, _I, _I, _I, _P, _P, _L, _I, _I, _I, _I, _I, _P]),
    "dt_frames_to_blocks": (_I, [_P, _P, _L, _I, _I, _I, _P, _I, _P]),
    "dt_rmsnorm": (_I, [_P, _L, _P, _P, _L, _I, _I, _F, _I, _P]),
    "dt_frames_conv1": (_I, [_P, _L, _I, _I, _I, _P, _P, _P, _P, _I, _I, _P]),
    "dt_encoder_conv23": (_I, [_P, _L, _P, _P, _P, _P, _P, _P, _I, _P]),
    "dt_frames_conv1_noalloc": (_I, [_P, _L, _I, _I, _I, _P, _P, _P, _I, _I, _P]),
    "dt_nes_reset": (_I, [_P, _I, _P, _I, _P, _U, _P, _U, _P]),
    "dt_nes_run_frames": (_I, [_P, _I, _I, _P, _U, _P, _U, _P]),
    "dt_nes_set_buttons": (_I, [_P, _I, _P, _P]),
    "dt_nes_set_actions": (_I, [_P, _I, _P, _P, _I, _P]),
    "dt_nes_observe": (_I, [_P, _I, _P, _P, _I, _P]),
    "dt_nes_env_update": (_I, [_P, _I, _I, _I, _P, _P, _P, _P, _P, _P, _P, _P, _P, _U, _P, _U, _P]),
}


class DTKernelUnavailable(RuntimeError):
    """The CUDA library is not built or cannot be loaded."""


class DTKernelError(RuntimeError):
    """A library call returned a nonzero status."""

    def __init__(self, fn: str, code: int, msg: str):
        super().__init__(f"{fn} failed (status {code}): {msg}")
        self.code = code


_lock = threading.Lock()
_lib = None


def load() -> ctypes.CDLL:
    """Loads the library once and declares every exported signature."""
    global _lib
    if _lib is not None:
        return _lib
    with _lock:
        if _lib is None:
            if not LIB_PATH.exists():
                raise DTKernelUnavailable(
                    f"{LIB_PATH} is missing; build it with `python -m rl_for_mario_b200.build`")
            try:
                lib = ctypes.CDLL(str(LIB_PATH))
            except OSError as e:  # pragma: no cover - depends on the machine
                raise DTKernelUnavailable(f"cannot load {LIB_PATH}: {e}") from e
            for name, (res, args) in SIGNATURES.items():
                fn = getattr(lib, name)
                fn.restype = res
                fn.argtypes = args
            _lib = lib
    return _lib


def check(fn: str, rc: int) -> None:
    if rc != DT_OK:
        msg = load().dt_last_error()
        raise DTKernelError(fn, rc, msg.decode() if msg else "")

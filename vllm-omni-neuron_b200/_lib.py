"""ctypes binding of the C ABI in ``include/vomni_b200.h`` (``libvomni_b200.so``).

The shared library is the only compute path: there is no Python or CPU fallback. If the library
is missing or the device is not an sm_100 part, calls raise instead of computing anything else.
"""

from __future__ import annotations

import ctypes
import threading
from pathlib import Path

HERE = Path(__file__).resolve().parent
LIB_PATH = HERE / "libvomni_b200.so"
HEADER = HERE.parent / "include" / "vomni_b200.h"

c_int, c_float, c_size_t, c_void_p, c_char_p = ctypes.c_int, ctypes.c_float, ctypes.c_size_t, ctypes.c_void_p, ctypes.c_char_p
P = c_void_p  # any device pointer / stream handle

# name -> (restype, argtypes); mirrors include/vomni_b200.h
SIGNATURES = {
    "vomni_abi_version": (c_int, []),
    "vomni_strerror": (c_char_p, [c_int]),
    "vomni_device_status": (c_int, [ctypes.POINTER(c_int), c_int]),
    "vomni_selftest_bounded_wait": (c_int, [ctypes.c_uint, ctypes.POINTER(c_int), P]),
    "vomni_selftest_ready_wait": (c_int, [ctypes.c_uint, c_int, ctypes.POINTER(c_int), P]),
    "vomni_selftest_exp2_poly": (c_int, [P, P, ctypes.c_longlong, P]),
    "vomni_memcpy_2d_async": (c_int, [P, c_size_t, P, c_size_t, c_size_t, c_size_t, P]),
    "vomni_cm_workspace_bytes": (c_size_t, [c_int, c_int, c_int, c_int]),
    "vomni_cm_prologue": (c_int, [P, P, c_int, c_int, c_int, c_int, P, P, P]),
    "vomni_cm_attend": (
        c_int,
        [P, P, P, c_int, c_int, c_int, c_int, c_int, c_int, c_int, c_float, P, P, P, P, c_int, P, P, P],
    ),
    "vomni_cm_attention_local": (
        c_int,
        [P, P, P, P, P, c_int, c_int, c_int, c_int, c_float, c_int, P, c_size_t, P],
    ),
    "vomni_adaln_modulate": (
        c_int,
        [P, P, P, P, P, ctypes.c_longlong, c_int, ctypes.c_longlong, c_float, c_int, c_int, c_int, c_int, P, P, P, P],
    ),
    "vomni_qkv_fp8_gemm": (c_int, [P, P, P, P, P, c_int, c_int, c_int, c_int, c_int, P, P, P]),
    "vomni_qk_norm_rope": (c_int, [P, c_int, c_int, c_int, c_int, c_int, P, c_float, P, P, P, P, P]),
    "vomni_oproj_gemm": (c_int, [P, c_int, c_int, c_int, P, P, c_int, P, P, c_int, P, P]),
    "vomni_oproj_rowquant": (c_int, [P, c_int, c_int, c_int, P, P, P]),
    "vomni_cfg_combine": (c_int, [P, P, P, ctypes.c_longlong, c_int, ctypes.c_float, P]),
    "vomni_ffn_fp8_up": (c_int, [P, P, P, P, P, c_int, c_int, c_int, P, P, P]),
    "vomni_ffn_fp8_down": (c_int, [P, P, P, P, P, P, c_int, c_int, c_int, P, P, ctypes.c_longlong, P, P]),
    "vomni_ffn_gemm": (c_int, [P, ctypes.c_longlong, c_int, P, P, c_int, c_int, P, P, ctypes.c_longlong, P, P]),
    "vomni_linear_sumsq": (c_int, [P, ctypes.c_longlong, c_int, P, P, c_int, P, c_int, P, P]),
    "vomni_qkv_unpack_rows": (c_int, [P, c_int, c_int, P, P, P]),
    "vomni_mx_packed_scales_bytes": (c_size_t, [c_int, c_int]),
    "vomni_mx_pack_scales": (c_int, [P, c_int, c_int, P, P]),
    "vomni_qkv_mx32_gemm": (c_int, [P, P, P, P, P, c_int, c_int, c_int, c_int, c_int, P, P, P]),
    "vomni_nccl_unique_id": (c_int, [P, c_size_t]),
    "vomni_ring_create": (c_int, [ctypes.POINTER(c_void_p), c_int, c_int, P, c_size_t, c_int, c_int, c_int, c_int]),
    "vomni_ring_destroy": (c_int, [P]),
    "vomni_ring_check": (c_int, [P]),
    "vomni_ring_attention": (
        c_int,
        [P, P, P, P, P, P, c_int, c_int, c_int, c_int, c_float, c_int, P],
    ),
    "vomni_ring_phase_plan": (c_int, [c_int, ctypes.POINTER(c_int), ctypes.POINTER(c_int), c_int]),
    "vomni_ring_source_rank": (c_int, [c_int, c_int, c_int]),
    "vomni_cm_prologue_strided": (c_int, [P, P, c_int, c_int, c_int, c_int, ctypes.c_longlong, ctypes.c_longlong, P, P, P]),
    "vomni_cm_attend_strided": (
        c_int,
        [P, P, P, c_int, c_int, c_int, c_int, c_int, c_int, c_int, ctypes.c_longlong, ctypes.c_longlong, c_float, P, P, P, P, c_int, P, P, P],
    ),
    "vomni_cm_attention_local_strided": (
        c_int,
        [P, P, P, P, P, c_int, c_int, c_int, c_int, ctypes.c_longlong, ctypes.c_longlong, c_float, c_int, P, c_size_t, P],
    ),
    "vomni_cm_attention_cross": (
        c_int,
        [P, P, P, P, P, c_int, c_int, c_int, c_int, c_int, ctypes.c_longlong, ctypes.c_longlong, c_float, c_int, P,
         c_size_t, P],
    ),
    "vomni_ring_attention_strided": (
        c_int,
        [P, P, P, P, P, P, c_int, c_int, c_int, c_int, ctypes.c_longlong, ctypes.c_longlong, c_float, c_int, P],
    ),
    "vomni_cm_attention_local_noalloc": (
        c_int,
        [P, P, P, P, P, c_int, c_int, c_int, c_int, c_float, c_int, P],
    ),
}

# flags (include/vomni_b200.h)
CM_ACC_IN = 1
CM_FINAL = 2
CM_OUT_DMAJOR = 4
CM_LSE = 8
CM_OVERLAP = 16

_lib = None
_lock = threading.Lock()


class VomniError(RuntimeError):
    def __init__(self, code: int, what: str):
        self.code = code
        super().__init__(f"{what} failed: {strerror(code)} (vomni status {code})")


def load():
    """Load (once) and return the ctypes library handle."""
    global _lib
    if _lib is not None:
        return _lib
    with _lock:
        if _lib is None:
            if not LIB_PATH.exists():
                raise RuntimeError(f"{LIB_PATH.name} is not built; run the package's build() first")
            lib = ctypes.CDLL(str(LIB_PATH))
            for name, (res, args) in SIGNATURES.items():
                fn = getattr(lib, name)
                fn.restype = res
                fn.argtypes = args
            _lib = lib
    return _lib


def strerror(code: int) -> str:
    return load().vomni_strerror(int(code)).decode()


def check(code: int, what: str) -> None:
    if code != 0:
        raise VomniError(code, what)


def call(name: str, *args) -> None:
    check(getattr(load(), name)(*args), name)


def device_status(clear: bool = True) -> int:
    """Synchronise and return (optionally clearing) the device status word: 0 when healthy."""
    out = c_int(0)
    check(load().vomni_device_status(ctypes.byref(out), int(clear)), "vomni_device_status")
    return out.value


def declared_symbols() -> list[str]:
    """Names of every entry point declared in include/vomni_b200.h."""
    import re

    text = HEADER.read_text()
    return re.findall(r"VOMNI_API\s+[\w\s\*]+?\b(vomni_\w+)\s*\(", text)

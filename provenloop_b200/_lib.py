"""ctypes binding of libtsgpu.so (the C ABI in include/tsgpu.h).

The library is the only compute path: if it is missing or no CUDA device is
visible, every entry point raises -- there is no CPU fallback.
"""
from __future__ import annotations

import ctypes as C
import os
import threading

import numpy as np

HERE = os.path.dirname(os.path.abspath(__file__))
# TSGPU_LIBRARY selects another build of the same ABI (e.g. an instrumented one)
LIB_PATH = os.environ.get("TSGPU_LIBRARY") or os.path.join(HERE, "libtsgpu.so")

TS_OK = 0
TS_ERR_ARG = -1
TS_ERR_OOM = -2
TS_ERR_CUDA = -3
TS_ERR_UNSUPPORTED = -4
TS_ERR_SCALE = -5
TS_ERR_STATE = -6
TS_ERR_NODEVICE = -7

_lib = None
_lock = threading.Lock()

vp = C.c_void_p
u32, u64, i32, f64, sz, cint = C.c_uint32, C.c_uint64, C.c_int32, C.c_double, C.c_size_t, C.c_int
P = C.POINTER
pvp = P(vp)

# name -> (restype, argtypes); mirrors include/tsgpu.h
SIGNATURES = {
    "ts_last_error": (C.c_char_p, []),
    "ts_version": (cint, []),
    "ts_device_count": (cint, [P(cint)]),
    "ts_launch_count": (cint, [P(u64)]),
    "ts_profile_enable": (cint, [cint]),
    "ts_profile_reset": (cint, []),
    "ts_profile_read": (cint, [C.c_char_p, P(f64), P(u64)]),
    "ts_params_custom": (cint, [u32, P(u32), u32, P(u64)]),
    "ts_host_tables": (cint, [u32, u64, P(u64), P(u64), P(f64), P(f64), P(f64), P(f64)]),
    "ts_ctx_create": (cint, [u32, cint, pvp]),
    "ts_ctx_create_custom": (cint, [u32, P(u32), u32, u32, cint, pvp]),
    "ts_ctx_create_moduli": (cint, [u32, P(u64), u32, cint, pvp]),
    "ts_ctx_destroy": (cint, [vp]),
    "ts_ctx_info": (cint, [vp, P(u32), P(u32), P(u32), P(u64)]),
    "ts_ctx_get_stream": (cint, [vp, pvp]),
    "ts_ctx_set_stream": (cint, [vp, vp]),
    "ts_ctx_reset_stream": (cint, [vp]),
    "ts_ctx_synchronize": (cint, [vp]),
    "ts_ctx_stats": (cint, [vp, P(u64)]),
    "ts_ctx_tables": (cint, [vp, u32, P(u64), P(u64), P(f64), P(f64), P(f64), P(f64)]),
    "ts_keygen": (cint, [vp, u64, pvp]),
    "ts_keygen_batch": (cint, [vp, P(u64), u32, pvp]),
    "ts_sk_destroy": (cint, [vp]),
    "ts_sk_count": (cint, [vp, P(u32)]),
    "ts_sk_export": (cint, [vp, u32, P(u64)]),
    "ts_encrypt": (cint, [vp, vp, P(f64), sz, u64, pvp]),
    "ts_encrypt_batch": (cint, [vp, vp, vp, sz, sz, sz, P(u64), P(i32), cint, pvp]),
    "ts_encrypt_stream": (cint, [vp, vp, P(f64), sz, sz, sz, u64, pvp]),
    "ts_keygen_public": (cint, [vp, vp, u32, u64, pvp]),
    "ts_pk_destroy": (cint, [vp]),
    "ts_pk_export": (cint, [vp, P(u64), P(u64)]),
    "ts_encrypt_pk": (cint, [vp, vp, vp, sz, sz, sz, P(u64), cint, pvp]),
    "ts_rescale": (cint, [vp, vp, pvp]),
    "ts_ct_destroy": (cint, [vp]),
    "ts_ct_info": (cint, [vp, P(u32), P(u32), P(f64)]),
    "ts_ct_export": (cint, [vp, u32, P(u64), P(u64)]),
    "ts_ct_import": (cint, [vp, P(u64), P(u64), u32, f64, pvp]),
    "ts_ct_select": (cint, [vp, vp, u32, pvp]),
    "ts_ct_to_bytes": (cint, [vp, C.c_char_p, sz, P(sz)]),
    "ts_ct_from_bytes": (cint, [vp, C.c_char_p, sz, u32, pvp]),
    "ts_pk_to_bytes": (cint, [vp, C.c_char_p, sz, P(sz)]),
    "ts_pk_from_bytes": (cint, [vp, C.c_char_p, sz, pvp]),
    "ts_decrypt": (cint, [vp, vp, vp, P(i32), vp, cint]),
    "ts_decrypt_noalloc": (cint, [vp, vp, vp, vp]),
    "ts_ct_pt_mul": (cint, [vp, vp, P(f64), sz, pvp]),
    "ts_encode_ntt": (cint, [vp, vp, sz, sz, sz, cint, pvp]),
    "ts_pt_destroy": (cint, [vp]),
    "ts_pt_export": (cint, [vp, u32, P(u64)]),
    "ts_ct_pt_mul_ntt": (cint, [vp, vp, vp, u32, pvp]),
    "ts_ct_add": (cint, [vp, vp, vp, pvp]),
    "ts_ct_sub": (cint, [vp, vp, vp, pvp]),
    "ts_ntt_forward": (cint, [vp, vp, sz, u32, u32]),
    "ts_ntt_inverse": (cint, [vp, vp, sz, u32, u32]),
    "ts_hadamard": (cint, [vp, vp, vp, vp, sz, u32, cint]),
    "ts_lora_load": (cint, [vp, P(C.c_float), P(C.c_float), u32, u32, u32, pvp]),
    "ts_lora_destroy": (cint, [vp]),
    "ts_lora_set_expert": (cint, [vp, vp, u32, P(C.c_float), P(C.c_float)]),
    "ts_lora_info": (cint, [vp, P(u32), P(u32), P(u32), P(u32), P(u32)]),
    "ts_lora_delta_batch": (cint, [vp, vp, vp, vp, u32, P(i32), P(i32), P(u64), vp, vp, cint]),
    "ts_dp_noise": (cint, [vp, vp, u32, u32, f64, f64, P(u64), cint]),
}


class TsError(RuntimeError):
    """Error raised from a failed libtsgpu call."""

    def __init__(self, code: int, msg: str):
        super().__init__(msg)
        self.code = code


def lib():
    """Load libtsgpu.so (built in-tree by provenloop_b200.build)."""
    global _lib
    with _lock:
        if _lib is None:
            if not os.path.exists(LIB_PATH):
                raise ImportError(
                    f"libtsgpu.so not found at {LIB_PATH}; build it with `python -m provenloop_b200.build` "
                    "(the CUDA engine has no CPU fallback)")
            L = C.CDLL(LIB_PATH)
            for name, (res, args) in SIGNATURES.items():
                f = getattr(L, name)
                f.restype = res
                f.argtypes = args
            _lib = L
    return _lib


def last_error() -> str:
    m = lib().ts_last_error()
    return m.decode() if m else ""


def check(rc: int, what: str = ""):
    """Map a TS_ERR_* status to a Python exception (lib.rs error conventions:
    unsupported degree -> ValueError; assert!-style violations -> ValueError;
    device / runtime failures -> RuntimeError)."""
    if rc == TS_OK:
        return
    msg = last_error() or f"{what} failed with status {rc}"
    if rc in (TS_ERR_ARG, TS_ERR_UNSUPPORTED, TS_ERR_SCALE):
        raise ValueError(msg)
    raise TsError(rc, msg)


def ptr(a: np.ndarray, ctype):
    return a.ctypes.data_as(P(ctype)) if a is not None else None


def device_count() -> int:
    n = C.c_int(0)
    check(lib().ts_device_count(C.byref(n)), "ts_device_count")
    return int(n.value)


def launch_count() -> int:
    v = C.c_uint64(0)
    check(lib().ts_launch_count(C.byref(v)), "ts_launch_count")
    return int(v.value)


def profile_enable(on: bool = True):
    check(lib().ts_profile_enable(1 if on else 0), "ts_profile_enable")


def profile_reset():
    check(lib().ts_profile_reset(), "ts_profile_reset")


def profile_read(kernel: str):
    """(total_ms, launches) of `kernel` since the last reset, or (0.0, 0)."""
    ms, n = C.c_double(0.0), C.c_uint64(0)
    rc = lib().ts_profile_read(kernel.encode(), C.byref(ms), C.byref(n))
    if rc != TS_OK:
        return 0.0, 0
    return float(ms.value), int(n.value)

"""ctypes binding of the C ABI declared in include/sokutou_b200.h.

The shared library is built in-tree (python -m sokutou_b200.build) and loaded from
sokutou_b200/lib/libsokutou_b200.so. There is no fallback: if the library is missing every op
raises.
"""

from __future__ import annotations

import ctypes
import os

# SOKUTOU_B200_LIB overrides the in-tree library (e.g. a build with other compile-time tuning)
LIB_PATH = os.environ.get("SOKUTOU_B200_LIB") or os.path.join(os.path.dirname(os.path.abspath(__file__)), "lib",
                                                               "libsokutou_b200.so")

SK_OK = 0
ERRORS = {-1: "SK_ERR_INVALID_ARG", -2: "SK_ERR_UNSUPPORTED", -3: "SK_ERR_CUDA", -4: "SK_ERR_DEVICE",
          -5: "SK_ERR_WORKSPACE", -6: "SK_ERR_TOO_LARGE"}
DEVICE_ERRORS = {0: "SK_DEVERR_NONE", 1: "SK_DEVERR_POS_RANGE", 2: "SK_DEVERR_TIMEOUT"}
SK_BF16, SK_F32, SK_E4M3 = 0, 1, 2
SK_DECODE_KV_STABLE = 1

# every symbol the header declares, with (restype, argtypes)
_P, _I, _F, _LL, _SZ = ctypes.c_void_p, ctypes.c_int, ctypes.c_float, ctypes.c_longlong, ctypes.c_size_t
SIGNATURES = {
    "sk_version": (_I, []),
    "sk_device_error": (_I, [ctypes.POINTER(ctypes.c_int), _I]),
    "sk_dit_attention": (_I, [_P, _P, _P, _P, _P, _P, _P, _I, _I, _I, _I, _I, _I, _LL, _LL, _I, _F, _P]),
    "sk_dit_qkv_prologue": (_I, [_P, _P, _P, _P, _P, _P, _I, _I, _I, _I, _F, _I, _P]),
    "sk_dit_gate": (_I, [_P, _P, _P, _LL, _I, _I, _I, _F, _P]),
    "sk_dit_linear": (_I, [_P, _P, _P, _I, _I, _I, _I, _P]),
    "sk_dit_linear_ex": (_I, [_P, _P, _P, _I, _I, _I, _I, _I, _P]),
    "sk_dit_linear_fp8": (_I, [_P, _P, _P, _P, _P, _I, _I, _I, _I, _P]),
    "sk_dit_attention_layer": (_I, [_P, _P, _P, _P, _P, _P, _P, _P, _P, _P, _I, _I, _I, _I, _I, _LL, _LL, _F, _I,
                                    _F, _P]),
    "sk_decode_workspace_bytes": (_SZ, [_I, _I, _I, _I, _I]),
    "sk_decode_attention": (_I, [_P, _P, _P, _F, _P, _P, _P, _P, _I, _I, _I, _I, _I, _P, _P, _SZ, _I, _P]),
    "sk_decode_attention_ex": (_I, [_P, _P, _P, _F, _P, _P, _P, _P, _I, _I, _I, _I, _I, _P, _P, _SZ, _I, _I, _P]),
    "sk_prefill_attention": (_I, [_P, _P, _P, _F, _P, _P, _P, _I, _I, _I, _I, _I, _I, _P, _P, _I, _P]),
    "sk_decode_attention_noalloc": (_I, [_P, _P, _P, _F, _P, _P, _P, _P, _I, _I, _I, _I, _I, _P, _I, _P]),
    "sk_decode_block_workspace_bytes": (_SZ, [_I, _I, _I, _I]),
    "sk_decode_attention_grouped": (_I, [_P, _I, _I, _I, _I, _I, _I, _I, _P]),
    "sk_decode_attention_block": (_I, [_P, _P, _F, _P, _P, _P, _F, _P, _P, _P, _P, _I, _I, _I, _I, _I, _P, _I, _I, _I,
                                       _P, _SZ, _I, _P]),
}



class SkDecodeRequest(ctypes.Structure):
    """include/sokutou_b200.h SkDecodeRequest (80 bytes): one request of sk_decode_attention_grouped."""
    _fields_ = [("qkv", _P), ("qn", _P), ("kn", _P), ("rope", _P), ("Kc", _P), ("Vc", _P), ("pos_ptr", _P),
                ("out", _P), ("pos_add", _I), ("eps", _F), ("reserved", _I * 2)]


assert ctypes.sizeof(SkDecodeRequest) == 80

_lib = None


class SokutouError(RuntimeError):
    pass


def lib() -> ctypes.CDLL:
    """The loaded library (loaded once). Raises if it has not been built."""
    global _lib
    if _lib is None:
        if not os.path.exists(LIB_PATH):
            raise SokutouError(f"native library missing: {LIB_PATH} (build it with `python -m sokutou_b200.build`)")
        L = ctypes.CDLL(LIB_PATH)
        for name, (res, args) in SIGNATURES.items():
            fn = getattr(L, name)
            fn.restype, fn.argtypes = res, args
        _lib = L
    return _lib


def check(rc: int, what: str) -> None:
    if rc != SK_OK:
        raise SokutouError(f"{what} failed: {ERRORS.get(rc, rc)}")

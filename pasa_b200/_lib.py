"""ctypes binding of libpasa_b200.so (the C ABI in include/pasa_b200.h).

The library is built in-tree by :mod:`pasa_b200.build`.  Importing this
module never builds; a missing library raises ``ImportError`` so that no
caller can silently run without the CUDA path.
"""
from __future__ import annotations

import ctypes
from ctypes import POINTER, c_char_p, c_double, c_float, c_int, c_int64, c_size_t, c_uint32, c_void_p
from pathlib import Path

LIB_PATH = Path(__file__).resolve().parent / "libpasa_b200.so"

# status codes (pasa_status)
OK = 0
ERR_SHAPE = 1
ERR_DTYPE = 2
ERR_ALIGN = 3
ERR_DENSITY = 4
ERR_UNSUPPORTED = 5
ERR_WORKSPACE = 6
ERR_NULL = 7
ERR_CUDA = 8
ERR_DEVICE = 9

BF16 = 0
F32 = 1

ATTN_AUTO = 0
ATTN_TCGEN05 = 1
ATTN_SIMT = 2

DEVERR_WAIT_TIMEOUT = 0x1

O_BHTD = 0
O_BTHD = 1

MODEL_HUNYUAN = 0
MODEL_WAN = 1

PEER_HANDLE_BYTES = 64

EXPORTS = (
    "pasa_abi_version", "pasa_status_string", "pasa_derive", "pasa_workspace_size", "pasa_prep",
    "pasa_select", "pasa_attn", "pasa_forward", "pasa_forward_noalloc", "pasa_place",
    "pasa_forward_host_workspace_size", "pasa_forward_host", "pasa_dense_attn",
    "pasa_dit_row_norm", "pasa_dit_qkv_rope", "pasa_forward_ex", "pasa_peer_alloc", "pasa_peer_free",
    "pasa_peer_open", "pasa_peer_close", "pasa_dit_qkv_rope_scatter", "pasa_forward_scatter",
    "pasa_sample_mse_workspace_size", "pasa_sample_mse", "pasa_forward_range_workspace_size",
    "pasa_forward_range",
)

_lib = None


def load() -> ctypes.CDLL:
    global _lib
    if _lib is not None:
        return _lib
    if not LIB_PATH.exists():
        raise ImportError(
            f"{LIB_PATH} is missing: build the CUDA library first (python -m pasa_b200.build)")
    lib = ctypes.CDLL(str(LIB_PATH))
    P = c_void_p
    sig = {
        "pasa_abi_version": (c_int, []),
        "pasa_status_string": (c_char_p, [c_int]),
        "pasa_derive": (c_int, [c_int64, c_int, c_int, c_double, POINTER(c_int64), POINTER(c_int64),
                                POINTER(c_int64)]),
        "pasa_workspace_size": (c_int, [c_int64, c_int64, c_int64, c_int, c_int, c_int, c_int, c_int64,
                                        POINTER(c_size_t)]),
        "pasa_prep": (c_int, [P, P, P, P, c_int64, c_int64, c_int64, c_int, c_int, c_int, c_int,
                              P, P, P, P, P]),
        "pasa_select": (c_int, [P, P, P, P, P, c_int64, c_int64, c_int, c_int, c_float, c_int, c_int64, P, P]),
        "pasa_attn": (c_int, [P, P, P, P, P, P, P, P, P, c_int64, c_int64, c_int, c_int, c_float, c_int64,
                              P, P, c_int]),
        "pasa_forward": (c_int, [P, P, P, P, c_int64, c_int64, c_int64, c_int, c_int, c_double, c_float, c_int,
                                 P, P, c_size_t, P, c_int]),
        "pasa_place": (c_int, [P, P, P, P, c_int64, c_int64, c_int64, c_int, c_int, c_int64, c_int64, c_int64,
                               c_int]),
        "pasa_forward_noalloc": (c_int, [P, P, P, P, c_int64, c_int64, c_int64, c_int, c_int, c_double, c_float,
                                         c_int, P, P, c_int]),
        "pasa_forward_host_workspace_size": (c_int, [c_int64, c_int64, c_int64, c_int, c_int, c_double, c_int64,
                                                     POINTER(c_size_t)]),
        "pasa_forward_host": (c_int, [P, P, P, P, c_int64, c_int64, c_int64, c_int, c_int, c_double, c_float, c_int,
                                      P, P, c_size_t, c_int64, P, POINTER(c_uint32), c_int]),
        "pasa_dense_attn": (c_int, [P, P, P, P, c_int64, c_int64, c_int, c_int, c_float, P, P]),
        "pasa_forward_ex": (c_int, [P, P, P, P, c_int64, c_int64, c_int64, c_int, c_int, c_double, c_float,
                                    c_int, P, P, c_size_t, P, c_int, c_int]),
        "pasa_peer_alloc": (c_int, [c_size_t, POINTER(c_void_p), P]),
        "pasa_peer_free": (c_int, [P]),
        "pasa_peer_open": (c_int, [P, POINTER(c_void_p)]),
        "pasa_peer_close": (c_int, [P]),
        "pasa_dit_qkv_rope_scatter": (c_int, [P, P, P, P, P, P, P, P, c_int64, c_int, c_int, c_float, P, c_int,
                                              c_int]),
        "pasa_forward_scatter": (c_int, [P, P, P, P, c_int64, c_int64, c_int, c_double, c_float, c_int, P, P,
                                         c_size_t, P, c_int, c_int64, c_int64, c_int]),
        "pasa_sample_mse_workspace_size": (c_int, [c_int64, c_int64, c_int, POINTER(c_size_t)]),
        "pasa_sample_mse": (c_int, [P, P, P, P, c_int64, c_int64, c_int64, c_int, c_int, P, c_int64, c_int,
                                    c_int64, c_int64, c_int64, P, c_size_t, P, P]),
        "pasa_forward_range_workspace_size": (c_int, [c_int64, c_int64, c_int64, c_int, c_int, c_double, c_int64,
                                                      c_int64, POINTER(c_size_t)]),
        "pasa_forward_range": (c_int, [P, P, P, P, c_int64, c_int64, c_int64, c_int, c_int, c_double, c_float,
                                       c_int, P, P, c_size_t, P, c_int, c_int64, c_int64]),
        "pasa_dit_row_norm": (c_int, [P, P, P, P, P, P, P, P, P, c_int64, c_int64, c_int, c_float, c_int, P]),
        "pasa_dit_qkv_rope": (c_int, [P, P, P, P, P, P, P, P, c_int64, c_int64, c_int, c_int, c_float, c_int,
                                      P, P, P]),
    }
    for name, (res, args) in sig.items():
        fn = getattr(lib, name)
        fn.restype = res
        fn.argtypes = args
    _lib = lib
    return lib


def status_string(code: int) -> str:
    return load().pasa_status_string(int(code)).decode()


class PasaError(RuntimeError):
    def __init__(self, fn: str, code: int):
        self.code = code
        super().__init__(f"{fn} failed: {status_string(code)} (status {code})")


def check(fn: str, code: int) -> None:
    """Map a pasa_status to the reference's error behaviour: argument
    problems raise ValueError, runtime problems RuntimeError."""
    if code == OK:
        return
    if code in (ERR_SHAPE, ERR_DTYPE, ERR_ALIGN, ERR_DENSITY, ERR_UNSUPPORTED, ERR_NULL, ERR_WORKSPACE):
        raise ValueError(f"{fn}: {status_string(code)} (status {code})")
    raise PasaError(fn, code)


def derive(T: int, density: float, block: int = 64, group: int = 32):
    nt, ng, ns = c_int64(), c_int64(), c_int64()
    check("pasa_derive", load().pasa_derive(int(T), int(block), int(group), float(density), ctypes.byref(nt),
                                            ctypes.byref(ng), ctypes.byref(ns)))
    return nt.value, ng.value, ns.value


def workspace_size(B: int, H: int, T: int, D: int, dtype: int, ns: int, block: int = 64, group: int = 32) -> int:
    n = c_size_t()
    check("pasa_workspace_size", load().pasa_workspace_size(int(B), int(H), int(T), int(D), int(dtype),
                                                            int(block), int(group), int(ns), ctypes.byref(n)))
    return n.value

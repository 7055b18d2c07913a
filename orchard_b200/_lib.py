"""ctypes binding of liborchard_b200.so (the C ABI in include/orchard_b200.h).

The library is required: importing a compute entry point without it raises. There is
no CPU fallback anywhere in the package.
"""

from __future__ import annotations

import ctypes as C
import os
import re
import threading

_PKG = os.path.dirname(os.path.abspath(__file__))
LIB_PATH = os.environ.get("ORCHARD_B200_LIB", os.path.join(_PKG, "lib", "liborchard_b200.so"))
HEADER = os.path.join(os.path.dirname(_PKG), "include", "orchard_b200.h")

F32, F16 = 0, 1


class OrchardError(RuntimeError):
    """A nonzero status from liborchard_b200."""

    def __init__(self, fn: str, status: int, msg: str):
        super().__init__(f"{fn} failed with status {status}: {msg}")
        self.status = status
        self.fn = fn


_vp, _u32, _i32, _f32, _sz = C.c_void_p, C.c_uint32, C.c_int, C.c_float, C.c_size_t
_u32p = C.POINTER(C.c_uint32)

# name -> (restype, argtypes)
_SIGS = {
    "orch_version": (_i32, []),
    "orch_status_string": (C.c_char_p, [_i32]),
    "orch_last_error": (C.c_char_p, []),
    "orch_init": (_i32, [_i32, C.c_char_p]),
    "orch_is_available": (_i32, []),
    "orch_device_name": (_i32, [C.c_char_p, _sz]),
    "orch_device_check": (_i32, [_u32p, _vp]),
    "orch_alloc": (_i32, [_sz, C.POINTER(_vp)]),
    "orch_free": (_i32, [_vp]),
    "orch_h2d": (_i32, [_vp, _vp, _sz, _vp]),
    "orch_d2h": (_i32, [_vp, _vp, _sz, _vp]),
    "orch_memset": (_i32, [_vp, _i32, _sz, _vp]),
    "orch_sync": (_i32, [_vp]),
    "orch_matmul": (_i32, [_vp, _vp, _vp, _u32, _u32, _u32, _vp]),
    "orch_matmul_simd": (_i32, [_vp, _vp, _vp, _u32, _u32, _u32, _vp]),
    "orch_rmsnorm": (_i32, [_vp, _vp, _vp, _f32, _u32, _u32, _vp]),
    "orch_rope": (_i32, [_vp, _vp, _vp, _vp, _u32, _u32, _u32, _vp]),
    "orch_gemv_q8_0": (_i32, [_vp, _vp, _vp, _vp, _u32, _u32, _vp]),
    "orch_gemv_q4_0": (_i32, [_vp, _vp, _vp, _vp, _u32, _u32, _vp]),
    "orch_gemm_q4_0": (_i32, [_vp, _vp, _vp, _vp, _u32, _u32, _u32, _vp]),
    "orch_add": (_i32, [_vp, _vp, _vp, _u32, _vp]),
    "orch_mul": (_i32, [_vp, _vp, _vp, _u32, _vp]),
    "orch_silu": (_i32, [_vp, _vp, _u32, _vp]),
    "orch_softmax": (_i32, [_vp, _vp, _u32, _u32, _vp]),
    "orch_embedding": (_i32, [_vp, _vp, _vp, _u32, _u32, _u32, _vp]),
    "orch_rmsnorm_ex": (_i32, [_vp, _i32, _vp, _i32, _vp, _i32, _f32, _u32, _u32, _vp]),
    "orch_rope_ex": (_i32, [_vp, _i32, _vp, _vp, _i32, _vp, _i32, _u32, _u32, _u32, _vp]),
    "orch_gemm_q4_0_ex": (_i32, [_vp, _vp, _vp, _i32, _vp, _i32, _u32, _u32, _u32, _vp]),
    "orch_gemm_q8_0_ex": (_i32, [_vp, _vp, _vp, _i32, _vp, _i32, _u32, _u32, _u32, _vp]),
    "orch_binary_ex": (_i32, [_i32, _vp, _vp, _vp, _i32, _u32, _vp]),
    "orch_silu_ex": (_i32, [_vp, _vp, _i32, _u32, _vp]),
    "orch_swiglu_ex": (_i32, [_vp, _vp, _vp, _i32, _u32, _vp]),
    "orch_softmax_ex": (_i32, [_vp, _i32, _vp, _i32, _u32, _u32, _vp]),
    "orch_embedding_ex": (_i32, [_vp, _vp, _i32, _vp, _i32, _u32, _u32, _u32, _vp]),
    "orch_quantize_q4_0": (_i32, [_vp, _i32, _vp, _vp, _u32, _u32, _vp]),
    "orch_quantize_q8_pc": (_i32, [_vp, _i32, _vp, _vp, _u32, _u32, _vp]),
    "orch_quantize_q8_0": (_i32, [_vp, _i32, _vp, _vp, _u32, _u32, _vp]),
    "orch_gemm_q8_pc": (_i32, [_vp, _vp, _vp, _i32, _vp, _i32, _u32, _u32, _u32, _vp]),
    "orch_lora_xa": (_i32, [_vp, _vp, _vp, _u32, _u32, _u32, _vp]),
    "orch_q4_linear_resid": (_i32, [_vp, _vp, _vp, _vp, _u32, _u32, _u32, _vp, _vp, _u32, _vp]),
    "orch_q4_linear_swiglu": (_i32, [_vp, _vp, _vp, _vp, _u32, _u32, _u32, _vp, _vp, _u32, _vp]),
    "orch_q4_qkv_rope": (_i32, [_vp, _vp, _vp, _u32, _u32, _u32, _u32, _vp, _vp, _vp, _vp, _u32,
                                _vp, _vp, _vp, _u32, _u32, _vp, _vp, _u32, _vp]),
    "orch_q4t_bytes": (_sz, [_u32, _u32]),
    "orch_q4t_pack": (_i32, [_vp, _vp, _u32, _u32, _vp, _vp]),
    "orch_q4t_gemm": (_i32, [_vp, _vp, _vp, _i32, _u32, _u32, _u32, _vp]),
    "orch_q4t_linear_resid": (_i32, [_vp, _vp, _vp, _u32, _u32, _u32, _vp, _vp, _u32, _vp]),
    "orch_q4t_linear_swiglu": (_i32, [_vp, _vp, _vp, _u32, _u32, _u32, _vp, _vp, _u32, _vp]),
    "orch_q4t_qkv_rope": (_i32, [_vp, _vp, _u32, _u32, _u32, _u32, _vp, _vp, _vp, _vp, _u32,
                                 _vp, _vp, _vp, _u32, _u32, _vp, _vp, _u32, _vp]),
    "orch_q4t_rms_qkv_rope": (_i32, [_vp, _vp, _vp, _f32, _vp, _u32, _u32, _u32, _u32, _vp, _vp, _vp, _vp, _u32,
                                     _vp, _vp, _vp, _u32, _u32, _vp]),
    "orch_q4t_rms_linear_swiglu": (_i32, [_vp, _vp, _vp, _f32, _vp, _vp, _u32, _u32, _u32, _vp]),
    "orch_gemv_max_rows": (_u32, []),
    "orch_attention_workspace_bytes": (_sz, [_u32, _u32, _u32, _u32]),
    "orch_attention_decode": (_i32, [_vp, _vp, _vp, _vp, _vp, _vp, _u32, _u32, _u32, _u32, _u32, _vp, _sz,
                                     _vp]),
    "orch_set_tc_min_m": (_i32, [_u32]),
    "orch_attention_prefill": (_i32, [_vp, _vp, _vp, _vp, _u32, _vp, _u32, _u32, _u32, _u32, _u32, _vp]),
    "orch_set_stream_k": (_i32, [_i32]),
    "orch_argmax_pairs": (_i32, [_vp, _u32, _u32, _u32, _vp, _vp]),
    "orch_argmax_merge": (_i32, [_vp, _u32, _u32, _u32, _u32, _vp, _vp]),
    "orch_sample_rows": (_i32, [_vp, _u32, _u32, C.c_float, _vp, _vp, _vp]),
    "orch_attention_noalloc_max_bytes": (_sz, []),
    "orch_attention_decode_noalloc": (_i32, [_vp, _vp, _vp, _vp, _vp, _vp, _u32, _u32, _u32, _u32, _u32, _vp]),
    "orch_argmax_rows": (_i32, [_vp, _u32, _u32, _vp, _vp]),
    "orch_embed_rows": (_i32, [_vp, _vp, _i32, _vp, _u32, _u32, _u32, _vp]),
    "orch_peer_region_bytes": (_sz, [_u32, _u32]),
    "orch_ipc_handle": (_i32, [_vp, _vp]),
    "orch_ipc_open": (_i32, [_vp, C.POINTER(_vp)]),
    "orch_ipc_close": (_i32, [_vp]),
    "orch_peer_allreduce": (_i32, [_vp, _u32, _u32, _u32, _vp, _u32, _i32, _vp]),
}

_lock = threading.Lock()
_lib = None


def header_symbols(path: str = HEADER):
    """Every function name declared in the C header."""
    text = open(path).read()
    text = re.sub(r"/\*.*?\*/", "", text, flags=re.S)
    return sorted(set(re.findall(r"\b(orch_[a-z0-9_]+)\s*\(", text)))


def lib() -> C.CDLL:
    """The loaded library with typed entry points (raises if it was not built)."""
    global _lib
    if _lib is not None:
        return _lib
    with _lock:
        if _lib is None:
            if not os.path.exists(LIB_PATH):
                raise ImportError(
                    f"liborchard_b200.so not found at {LIB_PATH}; build it with "
                    "`python -m orchard_b200.build` (there is no CPU fallback)")
            h = C.CDLL(LIB_PATH, mode=C.RTLD_GLOBAL)
            for name, (res, args) in _SIGS.items():
                f = getattr(h, name)
                f.restype = res
                f.argtypes = args
            _lib = h
    return _lib


def last_error() -> str:
    return (lib().orch_last_error() or b"").decode(errors="replace")


def call(name: str, *args) -> int:
    """Calls an int-returning entry point, raising OrchardError on a nonzero status.

    Tensor arguments are passed by device address and stay referenced for the duration of
    the call; work enqueued on a stream is ordered before any later reuse of their memory
    by the caching allocator on that stream."""
    args = tuple(a.data_ptr() if hasattr(a, "data_ptr") else a for a in args)
    rc = getattr(lib(), name)(*args)
    if rc != 0:
        raise OrchardError(name, rc, last_error())
    return rc


def ptr(t) -> int:
    """Device address of a torch tensor (or an int address)."""
    if t is None:
        return None
    if isinstance(t, int):
        return t
    return t.data_ptr()

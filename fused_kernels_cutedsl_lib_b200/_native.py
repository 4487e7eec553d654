"""ctypes binding of the C ABI in ``include/fk_b200.h`` (``_lib/libfk_b200.so``).

There is no fallback: if the shared library is missing or fails to load, every
entry point raises. Build it with ``python -m fused_kernels_cutedsl_lib_b200.build``
(``__graft_entry__.build()`` does this).
"""
from __future__ import annotations

import ctypes
import os
import threading
from pathlib import Path

# FK_LIB_PATH selects another build of the same library (A/B measurements).
LIB_PATH = Path(os.environ.get("FK_LIB_PATH") or Path(__file__).resolve().parent / "_lib" / "libfk_b200.so")

_c_int = ctypes.c_int
_c_float = ctypes.c_float
_p = ctypes.c_void_p

# name -> (restype, argtypes). Mirrors include/fk_b200.h one to one.
SIGNATURES: dict[str, tuple] = {
    "fk_last_error": (ctypes.c_char_p, []),
    "fk_version": (_c_int, []),
    "fk_num_sms": (_c_int, []),
    "fk_get_device_error": (_c_int, [ctypes.POINTER(_c_int), _c_int]),
    "fk_use_device": (_c_int, [_c_int]),
    "fk_dec_attn_chunk_tokens": (_c_int, [_c_int, _c_int]),
    "fk_dec_attn_splitkv_fwd": (
        _c_int,
        [_p, _p, _p, _p, _p, _p, _c_int, _c_int, _c_int, _c_int, _c_int, _c_int, _c_float, _p],
    ),
    "fk_dec_attn_combine": (
        _c_int,
        [_p, _p, _p, _p, _p, _c_int, _c_int, _c_int, _c_int, _c_int, _p],
    ),
    "fk_dec_attn_fwd": (
        _c_int,
        [_p, _p, _p, _p, _p, _p, _p, _p, _c_int, _c_int, _c_int, _c_int, _c_int, _c_int,
         _c_float, _p],
    ),
    "fk_linear_workspace_bytes": (_c_int, [_c_int, _c_int, _c_int, _c_int, ctypes.POINTER(ctypes.c_size_t)]),
    "fk_linear": (
        _c_int,
        [_p, _p, _p, _p, _c_int, _p, _p, _c_int, _c_int, _c_int, _c_float, _p, ctypes.c_size_t, _p],
    ),
    "fk_skinny_gemm": (_c_int, [_p, _p, _p, _c_int, _c_int, _c_int, _p, ctypes.c_size_t, _p]),
    "fk_rmsnorm_linear": (
        _c_int, [_p, _p, _p, _p, _c_int, _c_int, _c_int, _c_float, _p, ctypes.c_size_t, _p]),
    "fk_swiglu_gemm": (_c_int, [_p, _p, _p, _c_int, _c_int, _c_int, _p, ctypes.c_size_t, _p]),
    "fk_swiglu_gemm2": (_c_int, [_p, _p, _p, _p, _c_int, _c_int, _c_int, _p, ctypes.c_size_t, _p]),
    "fk_skinny_gemm_noalloc": (_c_int, [_p, _p, _p, _c_int, _c_int, _c_int, _p]),
    "fk_dec_attn_fwd_ex": (
        _c_int,
        [_p, ctypes.c_longlong, _p, _p, _p, _p, _p, _p, _p, _c_int, _c_int, _c_int, _c_int, _c_int, _c_int,
         _c_float, _p],
    ),
    "fk_kv_append": (
        _c_int,
        [_p, ctypes.c_longlong, _c_int, _c_int, _p, _p, _p, _p, _c_int, _c_int, _c_int, _c_int, _p],
    ),
    "fk_dattn1": (_c_int, [_p, _p, _p, _p, _c_int, _c_int, _c_int, _c_int, _p]),
    "fk_prefill_attn_fwd": (
        _c_int,
        [_p, _p, _p, _p, _p, _c_int, _c_int, _c_int, _c_int, _c_int, _c_int, _c_float, _p],
    ),
    "fk_linear_ex": (
        _c_int,
        [_p, _p, _p, _p, _c_int, _p, _c_int, _p, _c_int, _p, _c_int, _c_int, _c_int, _c_int, _c_float, _p,
         ctypes.c_size_t, _p],
    ),
    "fk_dec_attn_fwd_peers": (
        _c_int,
        [_p, ctypes.c_longlong, _p, _p, _p, _p, _p, _c_int, _p, _p, _p, _c_int, _c_int, _c_int, _c_int, _c_int,
         _c_int, _c_float, _p],
    ),
    "fk_peer_alloc": (_c_int, [ctypes.c_size_t, ctypes.POINTER(ctypes.c_void_p)]),
    "fk_peer_free": (_c_int, [_p]),
    "fk_ipc_handle_bytes": (_c_int, []),
    "fk_ipc_get_handle": (_c_int, [_p, _p]),
    "fk_ipc_open": (_c_int, [_p, ctypes.POINTER(ctypes.c_void_p)]),
    "fk_ipc_close": (_c_int, [_p]),
    "fk_peer_barrier": (_c_int, [_p, _p, _p, _c_int, _c_int, _p]),
    "fk_lora_linear": (
        _c_int,
        [_p, _p, _p, _p, _p, _p, _c_int, _c_int, _c_int, _c_int, _p, ctypes.c_size_t, _p],
    ),
    "fk_linear_kv_append": (
        _c_int,
        [_p, _p, _p, _p, _c_int, _c_int, _c_int, _c_float, _p, _p, _p, _p, _p, _c_int, _c_int, _c_int, _c_int,
         _c_int, _c_int, _p, ctypes.c_size_t, _p],
    ),
    "fk_dec_attn_fwd_commit": (
        _c_int,
        [_p, ctypes.c_longlong, _p, _p, _p, _p, _p, _p, _p, _p, _p, _c_int, _c_int, _c_int, _c_int, _c_int, _c_int,
         _c_int, _c_int, _c_float, _p],
    ),
    "fk_qkv_head_scatter": (_c_int, [_p, _p, _p, _p, _p, _p, _c_int, _c_int, _c_int, _c_int, _p]),
    "fk_dec_attn_fwd_paged": (
        _c_int,
        [_p, _p, _p, _p, _p, _p, _p, _p, _p, _c_int, _c_int, _c_int, _c_int, _c_int, _c_int, _c_int, _c_int,
         _c_float, _p],
    ),
    "fk_kv_append_paged": (
        _c_int,
        [_p, ctypes.c_longlong, _c_int, _c_int, _p, _p, _p, _p, _p, _c_int, _c_int, _c_int, _c_int, _c_int, _p],
    ),
    "fk_set_wait_limit_ns": (_c_int, [ctypes.c_ulonglong]),
    "fk_dec_attn_fwd_fused": (
        _c_int,
        [_p, ctypes.c_longlong, _p, _p, _p, _p, _p, _p, _p, _c_int, _p, _p, _p, _p, _c_int, _c_int, _c_int,
         _c_int, _c_int, _c_int, _c_int, _c_int, _c_float, _p],
    ),
    "fk_debug_attn_withhold_tile": (_c_int, [_c_int]),
    "fk_peer_signal": (_c_int, [_p, _p, _c_int, _c_int, _p]),
    "fk_linear_ex_wait": (
        _c_int,
        [_p, _p, _p, _p, _c_int, _p, _c_int, _p, _c_int, _p, _c_int, _c_int, _c_int, _c_int, _c_float, _p,
         ctypes.c_size_t, _p, _p, _c_int, _c_int, _p],
    ),
    "fk_kv_append_wait": (
        _c_int,
        [_p, ctypes.c_longlong, _c_int, _c_int, _p, _p, _p, _p, _c_int, _c_int, _c_int, _c_int, _p, _p, _c_int,
         _c_int, _p],
    ),
    "fk_rmsnorm_swiglu": (
        _c_int, [_p, _p, _p, _p, _c_int, _c_int, _c_int, _c_float, _p, ctypes.c_size_t, _p]),
}

_lock = threading.Lock()
_lib: ctypes.CDLL | None = None


class FKError(RuntimeError):
    """A CUDA-side failure reported by libfk_b200 (status -3 / -4)."""


def load() -> ctypes.CDLL:
    """Load libfk_b200.so once and attach the C signatures."""
    global _lib
    if _lib is not None:
        return _lib
    with _lock:
        if _lib is not None:
            return _lib
        if not LIB_PATH.exists():
            raise ImportError(
                f"{LIB_PATH} is missing: build it with "
                "`python -m fused_kernels_cutedsl_lib_b200.build` (needs nvcc)"
            )
        lib = ctypes.CDLL(str(LIB_PATH))
        for name, (res, args) in SIGNATURES.items():
            fn = getattr(lib, name)
            fn.restype = res
            fn.argtypes = args
        _lib = lib
    return _lib


def check(status: int) -> None:
    """Raise the Python exception matching a C-ABI status code."""
    if status == 0:
        return
    msg = load().fk_last_error().decode(errors="replace")
    if status == -1:
        raise ValueError(msg)
    if status == -2:
        raise NotImplementedError(msg)
    raise FKError(f"libfk_b200 status {status}: {msg}")


_tls = threading.local()


def use_device(index: int) -> None:
    """Make CUDA device `index` current for the library on this thread."""
    if getattr(_tls, "device", None) != index:
        check(load().fk_use_device(int(index)))
        _tls.device = index


def device_error(clear: bool = True) -> int:
    """Read (and by default clear) the device error word of the current device."""
    code = _c_int(0)
    check(load().fk_get_device_error(ctypes.byref(code), int(clear)))
    return code.value

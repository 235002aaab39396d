"""ctypes binding of ``libtinybatch_b200.so`` (the C ABI in include/tinybatch_b200.h).

The library is the only compute path: if it is missing or cannot be loaded
this module raises, there is no fallback.  Tensors are passed as raw device
pointers (``data_ptr()``); the current torch CUDA stream is used unless a
stream is given.
"""
from __future__ import annotations

import ctypes
from ctypes import c_float, c_int, c_size_t, c_uint, c_void_p
from pathlib import Path

import torch

_LIB_PATH = Path(__file__).resolve().parent / "_lib" / "libtinybatch_b200.so"
_lib = None

TB_OK = 0
STATUS_NAMES = {101: "pipeline barrier wait ran out", 102: "wait for a peer GPU's data ran out",
                103: "block id / position / slot out of range"}

_SIGS = {
    "tb_version": (c_int, []),
    "tb_last_error": (ctypes.c_char_p, []),
    "tb_debug_trace": (c_int, [c_void_p]),
    "tb_status": (c_int, [ctypes.POINTER(c_uint), c_int]),
    "tb_gemm_scratch_bytes": (c_size_t, [c_int, c_int, c_int, c_int]),
    "tb_gemm_max_active_clusters": (c_int, [c_int, c_int, ctypes.POINTER(c_int)]),
    "tb_linear": (c_int, [c_void_p, c_int, c_void_p, c_int, c_int, c_int, c_int,
                          c_void_p, c_int, c_int, c_float, c_float,
                          c_void_p, c_int, c_int, c_int, c_int, c_void_p, c_size_t, c_void_p]),
    "tb_linear_static_scratch": (c_int, [c_void_p, c_int, c_void_p, c_int, c_int, c_int, c_int,
                                         c_void_p, c_int, c_int, c_float, c_float,
                                         c_void_p, c_int, c_int, c_int, c_int, c_void_p]),
    "tb_qkv_rope_kv": (c_int, [c_void_p, c_int, c_void_p, c_int, c_void_p, c_int, c_int,
                               c_int, c_int, c_int, c_void_p, c_int, c_int, c_float, c_float,
                               c_void_p, c_void_p, c_int, c_void_p, c_void_p,
                               c_void_p, c_int, c_void_p, c_int, c_int, c_int,
                               c_void_p, c_size_t, c_void_p]),
    "tb_gate_up_swiglu": (c_int, [c_void_p, c_int, c_void_p, c_int, c_int, c_int, c_int,
                                  c_void_p, c_int, c_int, c_float, c_float,
                                  c_void_p, c_int, c_int, c_int, c_void_p, c_size_t, c_void_p]),
    "tb_row_linear_residual": (c_int, [c_void_p, c_int, c_void_p, c_int, c_int, c_int, c_int,
                                       c_void_p, c_int, c_void_p, c_void_p, c_int,
                                       c_void_p, c_int, c_void_p, c_void_p, c_void_p, c_int,
                                       c_int, c_int, c_void_p, c_size_t, c_void_p]),
    "tb_attention_scratch_bytes": (c_size_t, [c_int, c_int, c_int, c_int, c_int]),
    "tb_paged_attention_decode": (c_int, [c_void_p, c_int, c_void_p, c_int, c_void_p, c_int,
                                          c_int, c_int, c_int, c_int, c_void_p, c_int,
                                          c_void_p, c_void_p, c_void_p, c_void_p, c_int, c_int,
                                          c_int, c_void_p, c_size_t, c_void_p]),
    "tb_paged_attention_prefill": (c_int, [c_void_p, c_int, c_void_p, c_int, c_void_p, c_int,
                                           c_int, c_int, c_int, c_int, c_void_p, c_int,
                                           c_void_p, c_void_p, c_void_p, c_int,
                                           c_void_p, c_int, c_void_p]),
    "tb_comm_create": (c_int, [c_int, c_int, c_int, c_int, ctypes.POINTER(c_void_p), c_void_p]),
    "tb_comm_open": (c_int, [c_void_p, c_void_p]),
    "tb_comm_destroy": (c_int, [c_void_p]),
    "tb_row_linear_allreduce_residual": (c_int, [c_void_p, c_int, c_void_p, c_int, c_int, c_int,
                                                 c_int, c_void_p, c_int, c_void_p, c_void_p, c_int,
                                                 c_void_p, c_int, c_void_p, c_void_p, c_void_p,
                                                 c_int, c_void_p, c_int, c_int, c_void_p, c_int,
                                                 c_int, c_void_p]),
    "tb_embed": (c_int, [c_void_p, c_int, c_void_p, c_int, c_int, c_int, c_void_p,
                         c_void_p, c_int, c_void_p, c_int, c_void_p, c_void_p]),
    "tb_argmax": (c_int, [c_void_p, c_int, c_int, c_int, c_void_p, c_void_p]),
    "tb_argmax_vocab_parallel": (c_int, [c_void_p, c_void_p, c_int, c_int, c_int, c_int,
                                         c_void_p, c_int, c_void_p]),
}


class NativeError(RuntimeError):
    pass


def lib_path() -> Path:
    return _LIB_PATH


def exported_symbols() -> list[str]:
    return sorted(_SIGS)


def load():
    """Load the library (once).  Raises if it has not been built."""
    global _lib
    if _lib is not None:
        return _lib
    if not _LIB_PATH.exists():
        raise NativeError(f"{_LIB_PATH.name} is not built: run `python -m tinybatch_b200.build` "
                          "(the CUDA library is required; there is no CPU fallback)")
    lib = ctypes.CDLL(str(_LIB_PATH))
    for name, (res, args) in _SIGS.items():
        fn = getattr(lib, name)
        fn.restype = res
        fn.argtypes = args
    _lib = lib
    return lib


def check(rc: int, what: str) -> None:
    if rc != TB_OK:
        msg = load().tb_last_error()
        raise NativeError(f"{what} failed (code {rc}): {msg.decode() if msg else ''}")


def status(clear: bool = True) -> int:
    code = c_uint(0)
    check(load().tb_status(ctypes.byref(code), int(clear)), "tb_status")
    return code.value


def raise_on_status(what: str = "device") -> None:
    code = status(clear=True)
    if code:
        raise NativeError(f"{what}: device status {code} ({STATUS_NAMES.get(code, 'unknown')})")


def ptr(t: torch.Tensor | None) -> int | None:
    if t is None:
        return None
    if not t.is_cuda:
        raise NativeError("expected a CUDA tensor")
    return t.data_ptr()


def stream_ptr(stream: torch.cuda.Stream | None = None) -> int:
    s = stream if stream is not None else torch.cuda.current_stream()
    return s.cuda_stream

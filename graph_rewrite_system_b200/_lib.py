"""ctypes binding of ``libgrs_b200.so`` (the C ABI declared in include/grs_b200.h).

The library is loaded once, from the package directory only.  If it is
missing the import fails loudly: there is no CPU or library fallback for any
operation of this package.
"""
from __future__ import annotations

import ctypes
from pathlib import Path

import torch

LIBRARY_PATH = Path(__file__).resolve().parent / "libgrs_b200.so"

GRS_OK = 0
ERRORS = {
    -1: (RuntimeError, "paged KV cache exhausted"),
    -2: (RuntimeError, "retaining an unallocated page"),
    -3: (RuntimeError, "negative page reference count"),
    -4: (ValueError, "unsupported shape or layout"),
    -5: (RuntimeError, "CUDA launch failed"),
    -6: (RuntimeError, "free-list corruption"),
    -7: (RuntimeError, "prefix handle length/block table mismatch"),
    -8: (RuntimeError, "workspace too small"),
    -9: (ValueError, "inputs exceed the library's fixed scratch capacity"),
}

DTYPE_CODES = {torch.bfloat16: 0, torch.float32: 1}

_lib = None

c_i64 = ctypes.c_int64
c_int = ctypes.c_int
c_ptr = ctypes.c_void_p
c_f32 = ctypes.c_float

# argtypes per entry point; kept beside the header so a mismatch is obvious.
_SIGNATURES: dict[str, list] = {
    "grs_version": [],
    "grs_paged_attention": [
        c_int, c_ptr, c_i64, c_i64, c_i64,
        c_ptr, c_ptr, c_i64, c_i64, c_i64,
        c_ptr, c_i64, c_ptr,
        c_ptr, c_ptr, c_i64, c_i64, c_ptr,
        c_ptr, c_ptr, c_i64,
        c_ptr, c_i64, c_i64, c_i64,
        c_int, c_int, c_int, c_int, c_int, c_int, c_ptr,
    ],
}


def register(name: str, argtypes: list) -> None:
    """Declare an additional entry point's ctypes signature."""
    _SIGNATURES[name] = argtypes
    if _lib is not None:
        fn = getattr(_lib, name)
        fn.argtypes = argtypes
        fn.restype = c_int


def lib() -> ctypes.CDLL:
    global _lib
    if _lib is None:
        if not LIBRARY_PATH.exists():
            raise ImportError(
                f"{LIBRARY_PATH} is missing: build it with "
                "`python -m graph_rewrite_system_b200.build` (no fallback exists)"
            )
        handle = ctypes.CDLL(str(LIBRARY_PATH))
        for name, argtypes in _SIGNATURES.items():
            fn = getattr(handle, name)
            fn.argtypes = argtypes
            fn.restype = ctypes.c_char_p if name == "grs_version" else c_int
        _lib = handle
    return _lib


def exported_symbols() -> list[str]:
    return sorted(_SIGNATURES)


def check(status: int, what: str = "") -> None:
    if status != GRS_OK:
        exc, message = ERRORS.get(status, (RuntimeError, f"error {status}"))
        raise exc(f"{message}{' in ' + what if what else ''}")


def ptr(t: torch.Tensor | None) -> int | None:
    return None if t is None else t.data_ptr()


def stream_of(t: torch.Tensor) -> int:
    return torch.cuda.current_stream(t.device).cuda_stream


def require_cuda(*tensors: torch.Tensor | None) -> None:
    for t in tensors:
        if t is not None and not t.is_cuda:
            raise RuntimeError(
                "graph_rewrite_system_b200 kernels run on CUDA tensors only (no CPU fallback)"
            )

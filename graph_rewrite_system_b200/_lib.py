"""ctypes binding of ``libgrs_b200.so`` (the C ABI declared in include/grs_b200.h).

The library is loaded once, from the package directory only.  If it is
missing the import fails loudly: there is no CPU or library fallback for any
operation of this package.
"""
from __future__ import annotations

import ctypes
from pathlib import Path
import re

import torch

LIBRARY_PATH = Path(__file__).resolve().parent / "libgrs_b200.so"

GRS_OK = 0
GRS_ERR_SHAPE = -4
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
    -10: (RuntimeError, "an in-kernel wait timed out"),
    -11: (RuntimeError, "ranked records out of order"),
}

DTYPE_CODES = {torch.bfloat16: 0, torch.float32: 1}

_lib = None

c_i64 = ctypes.c_int64
c_int = ctypes.c_int
c_ptr = ctypes.c_void_p
c_f32 = ctypes.c_float

HEADER_PATH = Path(__file__).resolve().parent.parent / "include" / "grs_b200.h"

_C_TYPES = {"int": c_int, "int64_t": c_i64, "float": c_f32, "double": ctypes.c_double}


def _parse_header(text: str) -> dict[str, tuple[object, list]]:
    """(restype, argtypes) of every GRS_API declaration: pointers become
    c_void_p, scalars their ctypes type."""
    text = re.sub(r"/\*.*?\*/", " ", text, flags=re.S)
    out = {}
    for ret, name, params in re.findall(
            r"GRS_API\s+((?:const\s+)?[\w]+\s*\**)\s*(grs_\w+)\s*\(([^)]*)\)\s*;", text):
        args = []
        params = params.strip()
        if params and params != "void":
            for param in params.split(","):
                param = " ".join(param.replace("*", " * ").split())
                if "*" in param:
                    args.append(c_ptr)
                    continue
                base = param.replace("const ", "").split()[0]
                if base not in _C_TYPES:
                    raise ImportError(f"unsupported parameter type in {name}: {param}")
                args.append(_C_TYPES[base])
        ret = ret.replace("const", "").strip()
        if "*" in ret:
            restype = ctypes.c_char_p if ret.startswith("char") else c_ptr
        elif ret == "void":
            restype = None
        else:
            restype = _C_TYPES[ret.split()[0]]
        out[name] = (restype, args)
    return out


_SIGNATURES: dict[str, tuple[object, list]] = _parse_header(HEADER_PATH.read_text())


class _Bound:
    """The library's entry points with header-derived signatures; a call with
    the wrong number of arguments raises instead of reaching the C ABI."""

    def __init__(self, handle: ctypes.CDLL):
        self.handle = handle
        for name, (restype, argtypes) in _SIGNATURES.items():
            fn = getattr(handle, name)
            fn.argtypes = argtypes
            fn.restype = restype
            setattr(self, name, self._checked(name, fn, len(argtypes)))

    @staticmethod
    def _checked(name, fn, count):
        def call(*args):
            if len(args) != count:
                raise TypeError(f"{name} takes {count} arguments ({len(args)} given)")
            return fn(*args)
        call.__name__ = name
        return call


def lib() -> _Bound:
    global _lib
    if _lib is None:
        if not LIBRARY_PATH.exists():
            raise ImportError(
                f"{LIBRARY_PATH} is missing: build it with "
                "`python -m graph_rewrite_system_b200.build` (no fallback exists)"
            )
        _lib = _Bound(ctypes.CDLL(str(LIBRARY_PATH)))
    return _lib


def exported_symbols() -> list[str]:
    return sorted(_SIGNATURES)


def check(status: int, what: str = "") -> None:
    if status != GRS_OK:
        exc, message = ERRORS.get(status, (RuntimeError, f"error {status}"))
        raise exc(f"{message}{' in ' + what if what else ''}")


def ptr(t: torch.Tensor | None) -> int | None:
    return None if t is None else t.data_ptr()


_PINNED_STREAM: list[int] = []


def current_stream() -> int:
    """Raw handle of the stream pinned by an enclosing ``pinned_stream()``
    block, else of torch's current stream."""
    if _PINNED_STREAM:
        return _PINNED_STREAM[-1]
    return torch.cuda.current_stream().cuda_stream


def stream_of(t: torch.Tensor) -> int:
    if _PINNED_STREAM:
        return _PINNED_STREAM[-1]
    return torch.cuda.current_stream(t.device).cuda_stream


class pinned_stream:
    """Resolve torch's current stream once and launch every call inside the
    block on it (a beam-search level makes ~60 launches; looking the stream
    up per launch costs more host time than the launch itself)."""

    def __enter__(self):
        _PINNED_STREAM.append(torch.cuda.current_stream().cuda_stream)
        return self

    def __exit__(self, *exc):
        _PINNED_STREAM.pop()


def require_cuda(*tensors: torch.Tensor | None) -> None:
    for t in tensors:
        if t is not None and not t.is_cuda:
            raise RuntimeError(
                "graph_rewrite_system_b200 kernels run on CUDA tensors only (no CPU fallback)"
            )

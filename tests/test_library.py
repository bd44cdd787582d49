"""The C-ABI library loads and exports every entry point the header declares
(no kernel is launched: this runs on CPU)."""
from __future__ import annotations

import ctypes
import re

from conftest import ROOT


def declared_entry_points() -> list[str]:
    names = []
    for header in (ROOT / "include").glob("*.h"):
        text = header.read_text()
        names += re.findall(r"GRS_API\s+[\w\s\*]+?\b(grs_\w+)\s*\(", text)
    return sorted(set(names))


def test_header_declares_entry_points():
    names = declared_entry_points()
    assert "grs_paged_attention" in names and "grs_cache_append" in names
    assert "grs_proposals_rank" in names


def test_library_exports_every_declared_symbol():
    from graph_rewrite_system_b200 import build as build_mod

    build_mod.build()
    lib = ctypes.CDLL(str(build_mod.LIBRARY))
    missing = [n for n in declared_entry_points() if not hasattr(lib, n)]
    assert not missing, f"not exported: {missing}"


def test_python_bindings_cover_header():
    from graph_rewrite_system_b200 import _lib
    import graph_rewrite_system_b200.paged_attention  # noqa: F401
    import graph_rewrite_system_b200.paged_cache  # noqa: F401
    import graph_rewrite_system_b200.gpu_proposals  # noqa: F401
    import graph_rewrite_system_b200.kernels  # noqa: F401

    bound = set(_lib.exported_symbols())
    missing = [n for n in declared_entry_points() if n not in bound]
    assert not missing, f"no ctypes binding for: {missing}"
    lib = _lib.lib()
    assert lib.grs_version().startswith(b"grs_b200")


def test_cpu_tensors_rejected():
    import pytest
    import torch
    from graph_rewrite_system_b200.paged_attention import paged_attention

    q = torch.zeros(1, 1, 1, 32)
    kc = torch.zeros(1, 4, 1, 32)
    with pytest.raises(RuntimeError, match="CUDA"):
        paged_attention(q, kc, kc, torch.zeros(1, 1, dtype=torch.int32),
                        torch.zeros(1, dtype=torch.int32))

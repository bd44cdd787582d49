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
    """Every declaration is bound with a signature parsed from the header, and
    a call with the wrong argument count is refused before reaching C."""
    import pytest
    from graph_rewrite_system_b200 import _lib
    import graph_rewrite_system_b200.rollout  # noqa: F401  (imports every host module)

    bound = set(_lib.exported_symbols())
    assert bound == set(declared_entry_points())
    assert len(_lib._SIGNATURES["grs_topology_materialize"][1]) == 47
    lib = _lib.lib()
    assert lib.grs_version().startswith(b"grs_b200")
    with pytest.raises(TypeError):
        lib.grs_cache_init(0, 0, 0, 0, 1)


def test_cpu_tensors_rejected():
    import pytest
    import torch
    from graph_rewrite_system_b200.paged_attention import paged_attention

    q = torch.zeros(1, 1, 1, 32)
    kc = torch.zeros(1, 4, 1, 32)
    with pytest.raises(RuntimeError, match="CUDA"):
        paged_attention(q, kc, kc, torch.zeros(1, 1, dtype=torch.int32),
                        torch.zeros(1, dtype=torch.int32))

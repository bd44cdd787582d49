"""CPU oracle for the beam-search decode path (test infrastructure only).

This package restates, in plain NumPy and CPU PyTorch (fp32), the reference's
algorithms for every stage of the hot path, each function citing the
reference file:line it follows.  It is the checker: only ``tests/``,
``__graft_entry__.smoke()`` and ``bench.py``'s CPU-baseline / reference legs
import it.  The product path (``graph_rewrite_system_b200``) never imports it.

Parity of the restatement itself is pinned by ``tests/golden/*.npz``: vectors
produced by running the reference's own Python code on seeded inputs
(``tests/golden/make_golden.py``), checked in ``tests/test_oracle_golden.py``.
"""

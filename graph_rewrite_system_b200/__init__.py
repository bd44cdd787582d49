"""B200-native (sm_100a) beam-search decode path of the Quartz rewrite world model.

Drop-in replacements for the reference's hot-path modules, backed by
hand-written CUDA kernels in ``libgrs_b200.so`` (C ABI: include/grs_b200.h):

* ``paged_attention``  - paged decode / readout attention (paged_attention.py)
* ``paged_cache``      - PagedKVCache fork / COW / append / release (paged_cache.py)
* ``gpu_proposals``    - expansion and bounded ranking (gpu_proposals.py)

Importing a submodule that launches kernels loads the library; a missing
library raises ImportError (there is no CPU fallback).
"""

__all__ = ["paged_attention", "paged_cache", "gpu_proposals", "synthetic", "types"]

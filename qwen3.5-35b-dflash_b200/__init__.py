"""B200-native block-verify path for the Qwen3.5-MoE DFlash target.

Python name: ``qwen35_dflash_b200`` (the directory name is not an identifier; see
``__graft_entry__.load_package``).  Submodules:

* ``lib``        — ctypes binding of the C-ABI library ``libqw_b200.so`` (no fallback)
* ``fused_ops``  — drop-in adapter module for the reference's ``ModuleFusedOps``
* ``w4``         — W4A16 packing into the kernels' stream format
* ``engine``     — device-resident weights, paged KV / GDN state banks, block verify
* ``session``    — prefill / verify / commit semantics over the engine
"""
from __future__ import annotations

import importlib

__all__ = ["config", "synthetic", "lib", "fused_ops", "w4", "engine", "session", "build"]


def __getattr__(name):
    if name in __all__:
        return importlib.import_module(f"{__name__}.{name}")
    raise AttributeError(name)

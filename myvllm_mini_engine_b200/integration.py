"""Rebind the reference engine's paged-KV entry points to this package.

``install(mini_engine)`` patches an already imported ``mini_engine`` package
(the reference engine) so that its model, cache, batch and scheduler code calls
the sm_100a implementations here.  It covers names bound with ``from ...
import`` as well as module attributes:

* ``mini_engine.kernels.paged.paged_attention``            (paged.py:8)
* ``mini_engine.kernels.data.write_kv_cache[_batch|_slots]`` (data.py:39, 67, 84)
* ``mini_engine.kernels.prefill.paged_prefill_attention``  (prefill.py:61)
* the same names imported by ``mini_engine.model.native_qwen3`` (:13-18)
* ``PrefillBatch`` in ``mini_engine.engine.batch`` / ``.engine`` / ``.engine.runtime``
* ``BlockManager`` in ``mini_engine.cache.block_manager`` / ``.cache`` /
  ``.cache.prefix_cache`` / ``.engine.scheduler`` / ``.model.native_runner``

Out-of-scope ops (embedding, RoPE, norms, GEMMs, sampling) are left alone.
Returns the list of rebound ``module.name`` strings.
"""

from __future__ import annotations

import importlib
import sys

from .cache.block_manager import BlockManager
from .engine.batch import PrefillBatch
from .kernels.data import write_kv_cache, write_kv_cache_batch, write_kv_cache_slots
from .kernels.paged import paged_attention
from .kernels.prefill import paged_prefill_attention

REPLACEMENTS = {
    "kernels.paged": {"paged_attention": paged_attention},
    "kernels.data": {"write_kv_cache": write_kv_cache, "write_kv_cache_batch": write_kv_cache_batch,
                     "write_kv_cache_slots": write_kv_cache_slots},
    "kernels.prefill": {"paged_prefill_attention": paged_prefill_attention},
    "model.native_qwen3": {"paged_attention": paged_attention, "write_kv_cache_batch": write_kv_cache_batch,
                           "write_kv_cache_slots": write_kv_cache_slots,
                           "paged_prefill_attention": paged_prefill_attention},
    "engine.batch": {"PrefillBatch": PrefillBatch},
    "engine": {"PrefillBatch": PrefillBatch},
    "engine.runtime": {"PrefillBatch": PrefillBatch},
    "cache.block_manager": {"BlockManager": BlockManager},
    "cache": {"BlockManager": BlockManager},
    "cache.prefix_cache": {"BlockManager": BlockManager},
    "engine.scheduler": {"BlockManager": BlockManager},
    "model.native_runner": {"BlockManager": BlockManager},
}


def install(package) -> list[str]:
    """Patch the reference package object (or its name) in place."""
    if isinstance(package, str):
        package = importlib.import_module(package)
    root = package.__name__
    patched = []
    for suffix, names in REPLACEMENTS.items():
        full = f"{root}.{suffix}"
        try:
            module = sys.modules.get(full) or importlib.import_module(full)
        except ImportError:
            continue  # optional parts (e.g. the model needs transformers) may be absent
        for name, value in names.items():
            if hasattr(module, name):
                setattr(module, name, value)
                patched.append(f"{full}.{name}")
    return patched

"""Drop this package into an imported reference engine (``mini_engine``).

``install(mini_engine)`` rebinds, inside the already imported reference
package, the CUDA backend of every paged-KV entry point to the sm_100a
implementation here, and adds copy-on-write to the reference's allocator and
pool.  It covers names bound with ``from ... import`` as well as module
attributes:

* ``paged_attention``                       (kernels/paged.py:8)
* ``write_kv_cache[_batch|_slots]``         (kernels/data.py:39, 67, 84)
* ``paged_prefill_attention``               (kernels/prefill.py:61)
* the same names imported by ``model/native_qwen3.py`` (:13-18)
* ``PrefillBatch`` in ``engine.batch`` / ``engine`` / ``engine.runtime``
  (device-side metadata: one host-to-device copy and one kernel)
* ``BlockManager.copy_on_write`` / ``BlockManager.prepare_write`` (new methods
  on the reference class; ``cache/cow.py``) and ``KVCachePool.copy_blocks``
  (new; the device copy of the forked pages over every layer);
* with ``fuse_decode_append`` (default), ``Attention.forward_decode_batch``
  (model/native_qwen3.py:179-197) on the CUDA data and decode backends: its
  KV append and paged decode become one launch
  (``kernels.paged_attention_with_append``); other backends run the
  reference method unchanged.

Each rebound op keeps the reference's signature and default ``backend``.  A
call with a CUDA backend ("cuda", and for decode "cuda_baseline" /
"cuda_vector128") runs the kernels here; any other backend (the reference's
"torch" path) still runs the reference's own function, unchanged, so a model
built with ``data_backend="torch"`` and ``decode_backend="cuda"`` keeps working.
The allocator, scheduler, prefix cache, model and runtime stay the reference's.
Returns the list of rebound ``module.name`` strings.
"""

from __future__ import annotations

import functools
import importlib
import sys

from .cache.cow import copy_on_write, prepare_write
from .engine.batch import PrefillBatch
from .kernels import data as _data
from .kernels.paged import CUDA_BACKENDS, paged_attention, paged_attention_with_append
from .kernels.prefill import paged_prefill_attention

# op name -> (module of its definition in the reference, our implementation, backends routed to ours)
OPS = {
    "paged_attention": ("kernels.paged", paged_attention, CUDA_BACKENDS),
    "write_kv_cache": ("kernels.data", _data.write_kv_cache, ("cuda",)),
    "write_kv_cache_batch": ("kernels.data", _data.write_kv_cache_batch, ("cuda",)),
    "write_kv_cache_slots": ("kernels.data", _data.write_kv_cache_slots, ("cuda",)),
    "paged_prefill_attention": ("kernels.prefill", paged_prefill_attention, ("cuda",)),
}
# modules that bind the ops with ``from ... import``
IMPORTERS = ("model.native_qwen3",)
BATCH_MODULES = ("engine.batch", "engine", "engine.runtime")


def _routed(reference_op, ours, cuda_backends):
    """The reference op with its CUDA backends answered by ``ours``; same signature and defaults."""
    if getattr(reference_op, "__minikv_ours__", None) is ours:
        return reference_op  # already installed
    default = reference_op.__kwdefaults__.get("backend") if reference_op.__kwdefaults__ else None

    @functools.wraps(reference_op)
    def op(*args, backend=default, **kwargs):
        if backend in cuda_backends:
            return ours(*args, backend=backend, **kwargs)
        return reference_op(*args, backend=backend, **kwargs)

    op.__minikv_ours__ = ours
    op.__minikv_reference__ = reference_op
    return op


def _module(root, suffix):
    name = f"{root}.{suffix}"
    try:
        return sys.modules.get(name) or importlib.import_module(name)
    except ImportError:
        return None  # optional parts (e.g. the model needs transformers) may be absent


def _pool_copy_blocks(self, pairs) -> None:
    """Copy-on-write ``(src, dst)`` page pairs over every layer of this pool's K and V tensors."""
    _data.copy_blocks(self.key, self.value, pairs)


def _fused_decode_batch(reference_method):
    """``Attention.forward_decode_batch`` whose KV append and decode run as one kernel on the CUDA backends.

    The steps before the attention are the reference's own (its projection,
    q/k norms and the RoPE op its module binds); only the two calls at
    native_qwen3.py:188-196 are replaced by ``paged_attention_with_append``,
    which writes the same rows and returns the same attention.
    """
    if getattr(reference_method, "__minikv_reference__", None) is not None:
        return reference_method  # already installed

    @functools.wraps(reference_method)
    def forward_decode_batch(self, x, cos, sin, cache, block_tables, positions, layer, decode_backend):
        if self.data_backend != "cuda" or decode_backend not in CUDA_BACKENDS:
            return reference_method(self, x, cos, sin, cache, block_tables, positions, layer, decode_backend)
        rope = sys.modules[type(self).__module__].apply_rope_backend
        q, k, v = self._project_qkv(x)
        q, k = rope(self.q_norm(q), self.k_norm(k), cos, sin, backend="cuda", validate=False)
        attention = paged_attention_with_append(q, cache.key[layer], cache.value[layer], block_tables, positions,
                                                k, v, cache.shape.block_size, validate=False)
        return self.o_proj(attention.reshape(x.shape[0], -1))

    forward_decode_batch.__minikv_reference__ = reference_method
    return forward_decode_batch


def install(package, *, fuse_decode_append: bool = True) -> list[str]:
    """Patch the reference package object (or its name) in place; idempotent."""
    if isinstance(package, str):
        package = importlib.import_module(package)
    root = package.__name__
    patched = []
    routed = {}
    for name, (home, ours, backends) in OPS.items():
        module = _module(root, home)
        if module is None or not hasattr(module, name):
            continue
        routed[name] = _routed(getattr(module, name), ours, backends)
        setattr(module, name, routed[name])
        patched.append(f"{root}.{home}.{name}")
    for suffix in IMPORTERS:
        module = _module(root, suffix)
        for name, op in routed.items():
            if module is not None and hasattr(module, name):
                setattr(module, name, op)
                patched.append(f"{root}.{suffix}.{name}")
    for suffix in BATCH_MODULES:
        module = _module(root, suffix)
        if module is not None and hasattr(module, "PrefillBatch"):
            module.PrefillBatch = PrefillBatch
            patched.append(f"{root}.{suffix}.PrefillBatch")
    allocator = _module(root, "cache.block_manager")
    if allocator is not None:
        allocator.BlockManager.copy_on_write = copy_on_write
        allocator.BlockManager.prepare_write = prepare_write
        patched += [f"{root}.cache.block_manager.BlockManager.{n}" for n in ("copy_on_write", "prepare_write")]
    model = _module(root, "model.native_qwen3")
    if fuse_decode_append and model is not None and hasattr(model, "Attention"):
        model.Attention.forward_decode_batch = _fused_decode_batch(model.Attention.forward_decode_batch)
        patched.append(f"{root}.model.native_qwen3.Attention.forward_decode_batch")
    pools = _module(root, "cache.kv_cache")
    if pools is not None:
        pools.KVCachePool.copy_blocks = _pool_copy_blocks
        patched.append(f"{root}.cache.kv_cache.KVCachePool.copy_blocks")
    return patched

"""Operator API of the paged-KV hot path (mirrors ``mini_engine/kernels``)."""

from .data import copy_blocks, write_kv_cache, write_kv_cache_batch, write_kv_cache_slots
from .fp8 import (paged_attention_fp8, paged_attention_fp8_with_append, paged_prefill_attention_fp8,
                  write_kv_cache_slots_fp8)
from .paged import paged_attention, paged_attention_with_append
from .prefill import paged_prefill_attention

__all__ = ["copy_blocks", "paged_attention", "paged_attention_with_append", "paged_attention_fp8", "paged_attention_fp8_with_append", "paged_prefill_attention", "paged_prefill_attention_fp8", "write_kv_cache",
           "write_kv_cache_batch", "write_kv_cache_slots", "write_kv_cache_slots_fp8"]

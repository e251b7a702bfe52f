"""The drop-in installer rebinds every paged-KV name the reference engine uses.

Needs a copy of the reference engine under baseline/_ref (build container
only); skipped elsewhere.  No kernel runs: only name binding is checked.
"""

import sys
from pathlib import Path

import pytest

REF = Path(__file__).resolve().parents[1] / "baseline" / "_ref"


@pytest.mark.skipif(not (REF / "mini_engine").is_dir(), reason="reference copy not present")
def test_install_rebinds_reference_entry_points():
    sys.path.insert(0, str(REF))
    try:
        import mini_engine
        import mini_engine.model.native_qwen3 as nq
        from myvllm_mini_engine_b200 import integration, kernels
        from myvllm_mini_engine_b200.cache import BlockManager
        from myvllm_mini_engine_b200.engine import PrefillBatch

        patched = integration.install(mini_engine)
        assert nq.paged_attention is kernels.paged_attention
        assert nq.write_kv_cache_batch is kernels.write_kv_cache_batch
        assert nq.write_kv_cache_slots is kernels.write_kv_cache_slots
        assert nq.paged_prefill_attention is kernels.paged_prefill_attention
        import mini_engine.kernels.data as data
        import mini_engine.engine.batch as batch
        import mini_engine.engine.scheduler as scheduler
        assert data.write_kv_cache is kernels.write_kv_cache
        assert batch.PrefillBatch is PrefillBatch and scheduler.BlockManager is BlockManager
        assert len(patched) >= 14
    finally:
        sys.path.remove(str(REF))
        for name in [n for n in sys.modules if n == "mini_engine" or n.startswith("mini_engine.")]:
            del sys.modules[name]

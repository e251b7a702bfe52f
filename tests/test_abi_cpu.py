"""C-ABI library: loads, exports every declared symbol, rejects bad shapes (no GPU needed)."""

import ctypes
import re
from pathlib import Path

import pytest

from myvllm_mini_engine_b200 import _lib

HEADER = Path(__file__).resolve().parents[1] / "include" / "minikv.h"


def declared_symbols():
    text = re.sub(r"/\*.*?\*/", "", HEADER.read_text(), flags=re.S)
    return sorted(set(re.findall(r"\b(minikv_\w+)\s*\(", text)))


def test_library_exports_every_header_symbol():
    lib = _lib.load()
    names = declared_symbols()
    assert len(names) >= 13
    for name in names:
        assert hasattr(lib, name), name
    assert set(names) == set(_lib.SIGNATURES), "ctypes signatures must cover the header exactly"
    assert lib.minikv_abi_version() == 1


def test_decode_argument_errors_surface_as_codes_and_messages():
    lib = _lib.load()
    null = ctypes.c_void_p(16)
    args = [null] * 6 + [null, 1 << 20]
    # q_heads not divisible by kv_heads
    rc = lib.minikv_paged_decode(*args, 2, 6, 4, 128, 10, 16, 4, _lib.BF16, None)
    assert rc == _lib.EINVAL and "GQA" in lib.minikv_last_error().decode()
    rc = lib.minikv_paged_decode(*args, 2, 8, 4, 100, 10, 16, 4, _lib.BF16, None)
    assert rc == _lib.EINVAL and "head_dim" in lib.minikv_last_error().decode()
    rc = lib.minikv_paged_decode(*args, 2, 8, 4, 128, 10, 16, 1 << 17, _lib.BF16, None)
    assert rc == _lib.EINVAL and "1M tokens" in lib.minikv_last_error().decode()
    rc = lib.minikv_paged_decode(*args, 0, 8, 4, 128, 10, 16, 4, _lib.BF16, None)
    assert rc == _lib.EINVAL and "empty" in lib.minikv_last_error().decode()
    rc = lib.minikv_paged_decode(*args, 2, 8, 4, 128, 10, 16, 4, 7, None)
    assert rc == _lib.EINVAL


def test_workspace_queries_are_shape_only():
    lib = _lib.load()
    a = lib.minikv_paged_decode_workspace_bytes(32, 16, 8, 128, 4096, 16, 128, _lib.BF16)
    b = lib.minikv_paged_decode_workspace_bytes(32, 16, 8, 128, 4096, 16, 128, _lib.BF16)
    assert a == b > 0
    assert lib.minikv_paged_decode_workspace_bytes(32, 16, 8, 100, 4096, 16, 128, _lib.BF16) == -1
    assert lib.minikv_paged_prefill_workspace_bytes(2048, 16, 16, 8, 128, 1000, 16, 72, 128, _lib.BF16) >= 0


def test_kv_write_argument_errors():
    lib = _lib.load()
    p = ctypes.c_void_p(16)
    # row of 3 heads x 5 dims x 2 bytes is not a 16-byte multiple
    rc = lib.minikv_kv_scatter_slots(p, p, p, p, p, 4, 8, 4, 3, 5, 15, 15, _lib.F16, None)
    assert rc == _lib.EINVAL and "16 bytes" in lib.minikv_last_error().decode()
    rc = lib.minikv_kv_write_range(p, p, p, 2, 30, p, p, 4, 8, 16, 2, 64, 128, 128, _lib.F16, None)
    assert rc == _lib.EINVAL and "exceeds block table" in lib.minikv_last_error().decode()
    # empty writes are no-ops that touch nothing
    assert lib.minikv_kv_scatter_slots(None, None, None, None, None, 0, 8, 4, 2, 16, 32, 32, _lib.F16, None) == 0


def test_product_package_never_imports_the_oracle():
    root = Path(__file__).resolve().parents[1] / "myvllm_mini_engine_b200"
    for path in root.rglob("*.py"):
        text = path.read_text()
        assert not re.search(r"^\s*(from|import)\s+oracle\b", text, flags=re.M), path
        assert "tests.golden" not in text, path


def test_missing_library_fails_loudly(monkeypatch, tmp_path):
    monkeypatch.setattr(_lib, "_LIB", None)
    monkeypatch.setenv("MINIKV_LIBRARY", str(tmp_path / "absent.so"))
    with pytest.raises(RuntimeError, match="no CPU fallback"):
        _lib.load()


def test_library_built_from_other_sources_is_refused(monkeypatch):
    from myvllm_mini_engine_b200 import build

    assert build.built_hash() == build.source_hash() == _lib.load().minikv_source_hash().decode()
    monkeypatch.setattr(_lib, "_LIB", None)
    monkeypatch.setattr(build, "source_hash", lambda: "0" * 64)
    with pytest.raises(RuntimeError, match="built from other sources"):
        _lib.load()
    monkeypatch.undo()
    assert _lib.load() is not None


def test_argmax_argument_errors():
    lib = _lib.load()
    assert lib.minikv_argmax_workspace_bytes(0, 10) < 0
    assert lib.minikv_argmax_workspace_bytes(4, 151936) > 0
    null = ctypes.c_void_p(16)
    rc = lib.minikv_argmax_rows(null, 0, 10, 10, _lib.BF16, null, 1 << 20, null, None)
    assert rc == _lib.EINVAL and "rows" in lib.minikv_last_error().decode()
    rc = lib.minikv_argmax_rows(null, 4, 10, 8, _lib.BF16, null, 1 << 20, null, None)
    assert rc == _lib.EINVAL and "row stride" in lib.minikv_last_error().decode()
    rc = lib.minikv_argmax_rows(null, 4, 151936, 151936, _lib.BF16, null, 16, null, None)
    assert rc == _lib.EINVAL and "workspace" in lib.minikv_last_error().decode()

"""The C-ABI library loads on CPU and exports every symbol include/muk.h declares.

No compute call is made (no GPU here); the GPU tests call through the same
library."""

import ctypes
import re
from pathlib import Path

import pytest

ROOT = Path(__file__).resolve().parents[1]
HEADER = ROOT / "include" / "muk.h"


def _declared():
    text = HEADER.read_text()
    return sorted(set(re.findall(r"^\s*(?:int|int64_t|size_t|const char\*)\s+(muk_\w+)\s*\(", text, re.M)))


def test_header_declares_entry_points():
    names = _declared()
    assert len(names) >= 18
    for must in ("muk_paged_decode_attn", "muk_paged_prefill_attn", "muk_gemm_bf16",
                 "muk_rope_kv_append", "muk_sample", "muk_grouped_gemm_bf16"):
        assert must in names


def test_library_exports_every_declared_symbol():
    from mu_b200 import _lib

    if not _lib.LIB_PATH.exists():
        pytest.skip("libmuk.so not built (run complexity-inference_b200/build.py)")
    lib = ctypes.CDLL(str(_lib.LIB_PATH))
    for name in _declared():
        assert hasattr(lib, name), name
    # the Python binding covers exactly the declared entry points
    assert sorted(_lib.SIGNATURES) == _declared()
    assert _lib.load().muk_version() >= 1


def test_binding_fails_loudly_without_library(tmp_path, monkeypatch):
    from mu_b200 import _lib

    monkeypatch.setattr(_lib, "_lib", None)
    monkeypatch.setattr(_lib, "LIB_PATH", tmp_path / "missing.so")
    with pytest.raises(_lib.MukError):
        _lib.load()

"""The C-ABI library loads without a GPU and exports exactly what include/mossgpu.h declares."""
from __future__ import annotations

import ctypes as C
import re
from pathlib import Path

import pytest

ROOT = Path(__file__).resolve().parents[1]


def declared_symbols() -> list[str]:
    text = (ROOT / "include" / "mossgpu.h").read_text()
    text = re.sub(r"/\*.*?\*/", "", text, flags=re.S)
    return sorted(set(re.findall(r"\b(mossgpu_[a-z0-9_]+)\s*\(", text)))


@pytest.fixture(scope="module")
def built_lib():
    import moss_b200
    moss_b200.build()
    return moss_b200


def test_header_and_python_binding_agree(built_lib):
    assert declared_symbols() == sorted(built_lib.EXPORTS)


def test_library_exports_every_declared_symbol(built_lib):
    lib = C.CDLL(str(built_lib.LIB_PATH))
    missing = [s for s in declared_symbols() if not hasattr(lib, s)]
    assert not missing, missing


def test_version_and_null_handles(built_lib):
    L = built_lib.lib()
    assert L.mossgpu_version().startswith(b"moss-b200")
    # every int entry point rejects a NULL engine with a non-zero status, no crash
    assert L.mossgpu_stream_close(None, 0) != 0
    assert L.mossgpu_last_error(None) == b"null engine"
    assert L.mossgpu_last_launch_count(None) == -1


def test_create_reports_errors_without_throwing(built_lib, tmp_path):
    L = built_lib.lib()
    err = C.create_string_buffer(256)
    assert not L.mossgpu_create(str(tmp_path / "missing.moss").encode(), 0, 1, 64, 0, err, 256)
    assert err.value  # a message, whatever the failure (no file, or no device here)


def test_missing_library_fails_loudly(built_lib, monkeypatch, tmp_path):
    monkeypatch.setattr(built_lib, "LIB_PATH", tmp_path / "libmossgpu.so")
    monkeypatch.setattr(built_lib, "_LIB", None)
    with pytest.raises(built_lib.MossGpuError):
        built_lib.lib()

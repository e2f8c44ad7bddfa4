"""The C ABI on a CPU-only box: the library loads, exports every declared symbol, and rejects
bad arguments with the reference's status codes (src/libstems_v1.h:54-63) without a GPU."""
from __future__ import annotations

import ctypes as C
import os
import re

import pytest

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))


def declared_symbols():
    names = []
    for fn in sorted(os.listdir(os.path.join(ROOT, "include"))):
        if fn.endswith(".h"):
            text = open(os.path.join(ROOT, "include", fn)).read()
            names += re.findall(r"STG_API\s+[^;(]*?\b(stg_\w+)\s*\(", text)
    return names


def test_header_declares_entry_points():
    names = declared_symbols()
    assert len(names) >= 10
    assert "stg_separate" in names and "stg_separate_host" in names


def test_library_exports_every_declared_symbol(pkg):
    L = C.CDLL(pkg.library_path())
    missing = [n for n in declared_symbols() if not hasattr(L, n)]
    assert not missing, f"not exported: {missing}"


def test_signatures_cover_the_header(pkg):
    assert set(declared_symbols()) <= set(pkg._SIGNATURES)


def test_version_and_device_count(pkg):
    assert "stems_gpu abi 1" in pkg.version()
    assert pkg.device_count() >= 0 or pkg.device_count() == -1


def test_null_arguments_are_rejected(pkg):
    L = pkg.lib()
    out = C.c_void_p()
    assert L.stg_engine_create(0, None) == 1
    assert L.stg_plan_htdemucs(None, None, 100, C.byref(out)) == 1
    assert out.value is None
    assert L.stg_plan_roformer(None, None, 100, None) == 1
    assert L.stg_plan_tfc(None, None, 100, None) == 1
    assert L.stg_separate(None, None, None, None, None) == 1
    assert L.stg_separate_host(None, None, None, None, None) == 1
    assert L.stg_plan_get_info(None, None) == 1
    L.stg_plan_destroy(None)
    L.stg_engine_destroy(None)
    assert L.stg_engine_last_error(None) == b""


def test_engine_on_a_missing_device_fails_cleanly(pkg):
    import torch
    if torch.cuda.is_available():
        pytest.skip("a GPU is present")
    h = C.c_void_p()
    rc = pkg.lib().stg_engine_create(0, C.byref(h))
    assert rc in (1, 7) and not h.value


def test_missing_library_raises_instead_of_falling_back(pkg, monkeypatch, tmp_path):
    monkeypatch.setattr(pkg, "_lib", None)
    monkeypatch.setattr(pkg, "LIB_PATH", str(tmp_path / "absent.so"))
    with pytest.raises(pkg.StemsError):
        pkg.lib()


def test_resampled_length_without_a_gpu(pkg, oracle_mod):
    for n, src, dst in [(44100, 48000, 44100), (1, 48000, 44100), (123457, 22050, 44100), (99, 44100, 44100)]:
        assert pkg.resampled_length(n, src, dst) == oracle_mod.resampled_length(n, src, dst)
    assert pkg.lib().stg_resampled_length(10, 0, 44100) == -1


def test_conversion_entry_points_reject_a_null_engine(pkg):
    L = pkg.lib()
    assert L.stg_prepare_input(None, None, 1, 10, 2, 48000, 2, 44100, None, None) == 1
    assert L.stg_restore_output(None, None, 2, 10, 44100, 48000, 10, None, None) == 1


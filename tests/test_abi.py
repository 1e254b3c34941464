"""The C ABI library loads, exports every entry point include/sffft.h declares, and validates its
arguments without touching a GPU."""
import ctypes
import os
import re

import pytest

import sffft_b200 as sf

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))

REFERENCE_CANDIDATES = {   # (plan, W) rows of the reference's RUN catalog, src/sffft.cu:507-513
    128: ["16x16/w4", "16x16/w8"],
    256: ["32x16/w4", "16x32/w4", "32x16/w8"],
    512: ["32x32/w4", "32x32/w8", "64x16/w4", "16x64/w4"],
    1024: ["64x32/w4", "32x64/w4", "64x32/w8", "32x64/w8"],
    2048: ["16x16x16/w4", "16x16x16/w8", "64x64/w8", "64x64/w4"],
    4096: ["32x16x16/w4", "16x32x16/w4", "16x16x32/w4", "32x16x16/w8", "16x16x32/w8"],
    8192: ["32x32x16/w4", "16x32x32/w4", "64x16x16/w4", "32x32x16/w8", "16x32x32/w8", "16x16x64/w8"],
}


def declared_functions():
    txt = open(os.path.join(ROOT, "include", "sffft.h")).read()
    txt = re.sub(r"/\*.*?\*/", "", txt, flags=re.S)
    return sorted(set(re.findall(r"\b(sffft_[a-z0-9_]+)\s*\(", txt)))


def test_exports_every_declared_symbol():
    names = declared_functions()
    assert len(names) >= 15
    lib = ctypes.CDLL(sf.LIB_PATH)
    missing = [n for n in names if not hasattr(lib, n)]
    assert not missing, missing


def test_catalog_contains_reference_candidates():
    cat = sf.catalog()
    by_len = {}
    for L, name in cat:
        by_len.setdefault(L, []).append(name)
    for L, names in REFERENCE_CANDIDATES.items():
        assert sorted(by_len[L]) == sorted(names), L
    assert sum(len(v) for L, v in by_len.items() if L <= 8192) == 28
    assert "32x32x32/w4" in by_len[16384]
    for L in list(REFERENCE_CANDIDATES) + [16384]:
        assert sf.default_config(L) in by_len[L]


def test_status_strings_and_shards():
    assert sf.status_string(0) == "ok"
    assert "timed out" in sf.status_string(sf.ERR_TIMEOUT)
    assert sf.shard_range(768, 8, 0) == (0, 96)
    assert sf.shard_range(768, 8, 7) == (672, 768)
    assert sf.shard_range(10, 4, 0) == (0, 3) and sf.shard_range(10, 4, 3) == (8, 10)
    spans = [sf.shard_range(1000, 7, g) for g in range(7)]
    assert spans[0][0] == 0 and spans[-1][1] == 1000
    assert all(a[1] == b[0] for a, b in zip(spans, spans[1:]))
    with pytest.raises(sf.SffftError):
        sf.shard_range(10, 0, 0)
    with pytest.raises(sf.SffftError):
        sf.shard_range(10, 2, 2)


def test_plan_create_rejects_bad_arguments():
    lib = sf.lib()
    h = ctypes.c_void_p()
    assert lib.sffft_plan_create(ctypes.byref(h), 1024, 7, 0, None, 1, 0) == sf.ERR_INVALID_ARGUMENT
    assert lib.sffft_plan_create(ctypes.byref(h), 1024, 0, 3, None, 1, 0) == sf.ERR_INVALID_ARGUMENT
    assert lib.sffft_plan_create(ctypes.byref(h), 1000, 0, 0, None, 1, 0) == sf.ERR_UNSUPPORTED
    assert lib.sffft_plan_create(ctypes.byref(h), 1024, 0, 0, b"32x32/w4", 1, 0) == sf.ERR_UNSUPPORTED
    assert lib.sffft_plan_create(ctypes.byref(h), 1024, 0, 0, b"nonsense", 1, 0) == sf.ERR_UNSUPPORTED
    assert lib.sffft_plan_create(None, 1024, 0, 0, None, 1, 0) == sf.ERR_INVALID_ARGUMENT
    assert not h.value


def test_null_handles_are_rejected():
    lib = sf.lib()
    assert lib.sffft_conv(None, 16, 16, 16, 1, 1, None) == sf.ERR_INVALID_ARGUMENT
    assert lib.sffft_conv_ws(None, 16, 16, 16, 1, 1, 256, 1 << 20, None) == sf.ERR_INVALID_ARGUMENT
    assert lib.sffft_conv_workspace_bytes(None, 1, 1, ctypes.byref(ctypes.c_size_t())) == sf.ERR_INVALID_ARGUMENT
    assert lib.sffft_plan_set_workspace(None, None, 0) == sf.ERR_INVALID_ARGUMENT
    assert lib.sffft_filter_spectrum(None, 16, 0, 1, 16, None) == sf.ERR_INVALID_ARGUMENT
    assert lib.sffft_filter_spectrum_ex(None, 16, 0, 1, 1, 16, None) == sf.ERR_INVALID_ARGUMENT
    assert lib.sffft_rfft(None, 16, 0, 1, 16, 16, None) == sf.ERR_INVALID_ARGUMENT
    assert lib.sffft_irfft(None, 16, 1, 16, 16, None) == sf.ERR_INVALID_ARGUMENT
    assert lib.sffft_plan_destroy(None) == sf.ERR_INVALID_ARGUMENT
    assert lib.sffft_plan_check(None) == sf.ERR_INVALID_ARGUMENT
    assert lib.sffft_baseline_destroy(None) == sf.ERR_INVALID_ARGUMENT
    assert lib.sffft_pipe_create(None, None, 1, 1, 0) == sf.ERR_INVALID_ARGUMENT
    assert lib.sffft_conv_host(None, 16, 16, 16, None) == sf.ERR_INVALID_ARGUMENT
    assert lib.sffft_pipe_destroy(None) == sf.ERR_INVALID_ARGUMENT

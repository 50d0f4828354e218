"""The C-ABI library loads without a GPU and exports every declared symbol."""
import ctypes
import os

import pytest

from mi_b200 import capi


@pytest.fixture(scope="module")
def built_lib():
    from importlib import util
    here = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
    spec = util.spec_from_file_location(
        "mi_build", os.path.join(here, "minimal-inference_b200", "csrc", "build.py"))
    mod = util.module_from_spec(spec)
    spec.loader.exec_module(mod)
    mod.build()
    return capi.lib()


def test_header_declares_the_hot_path():
    syms = capi.header_symbols()
    for name in ("mi_append_paged_kv_cache", "mi_paged_decode", "mi_paged_prefill",
                 "mi_page_pool_init", "mi_page_alloc", "mi_page_release", "mi_slot_alloc",
                 "mi_slot_release", "mi_step_prepare", "mi_last_error", "mi_version",
                 "mi_paged_decode_workspace_size", "mi_paged_prefill_workspace_size"):
        assert name in syms


def test_library_exports_every_header_symbol(built_lib):
    for name in capi.header_symbols():
        assert hasattr(built_lib, name), name
        assert name in capi._SIGS, f"{name} has no ctypes signature"


def test_version_and_host_errors_without_gpu(built_lib):
    assert built_lib.mi_version() >= 100
    # argument validation happens on the host and needs no device
    rc = built_lib.mi_page_pool_init(None, None, 0, None)
    assert rc == 1  # MI_ERR_INVALID
    assert b"pool_init" in built_lib.mi_last_error()
    rc = built_lib.mi_paged_decode(None, 0, 0, None, 0, 0, 0, 0, 0, None, None, None,
                                   1, 8, 0.1, None, None, None, 0, None, None)
    assert rc == 1
    assert b"decode" in built_lib.mi_last_error()


def test_workspace_sizes(built_lib):
    n = built_lib.mi_paged_decode_workspace_size(32, 32, 8, 128)
    assert n > 32 * 8 * 4
    assert built_lib.mi_paged_decode_workspace_size(0, 32, 8, 128) == 0


def test_missing_library_fails_loudly(monkeypatch, tmp_path):
    monkeypatch.setattr(capi, "LIB_PATH", str(tmp_path / "absent.so"))
    monkeypatch.setattr(capi, "_lib", None)
    with pytest.raises(capi.MiError):
        capi.lib()


def test_status_names():
    assert capi.status_names(1 | 64) == ["OUT_OF_PAGES", "TIMEOUT"]


def _header_params() -> dict:
    """Parameter count of every function declared in include/mi_paged.h."""
    import re
    with open(capi.HEADER_PATH) as f:
        text = re.sub(r"/\*.*?\*/", "", f.read(), flags=re.S)
    out = {}
    for m in re.finditer(r"\b(mi_[a-z0-9_]+)\s*\(([^;{]*?)\)\s*;", text, flags=re.S):
        params = m.group(2).strip()
        out[m.group(1)] = 0 if params in ("", "void") else params.count(",") + 1
    return out


def test_ctypes_signatures_match_the_header():
    """Every ctypes signature takes as many arguments as the header declares:
    a call with a shifted argument list would hand a kernel wrong pointers."""
    declared = _header_params()
    assert declared, "no declarations parsed"
    for name, n in declared.items():
        assert name in capi._SIGS, f"{name} has no ctypes signature"
        assert len(capi._SIGS[name][0]) == n, (
            f"{name}: header declares {n} parameters, ctypes {len(capi._SIGS[name][0])}")


def test_ctypes_argument_types_match_the_header():
    """Parameter by parameter: pointers bind as c_void_p, int32_t / int64_t /
    size_t / float as their ctypes types (a swapped pair would pass a count
    check)."""
    import re
    with open(capi.HEADER_PATH) as f:
        text = re.sub(r"/\*.*?\*/", "", f.read(), flags=re.S)
    scalar = {"int32_t": ctypes.c_int32, "int64_t": ctypes.c_int64, "size_t": ctypes.c_size_t,
              "float": ctypes.c_float, "mi_stream_t": ctypes.c_void_p}
    checked = 0
    for m in re.finditer(r"\b(mi_[a-z0-9_]+)\s*\(([^;{]*?)\)\s*;", text, flags=re.S):
        name, params = m.group(1), m.group(2).strip()
        if params in ("", "void"):
            continue
        for i, p in enumerate(x.strip() for x in params.split(",")):
            t = re.sub(r"\b[A-Za-z_][A-Za-z0-9_]*$", "", p).strip()
            want = ctypes.c_void_p if "*" in t else scalar[t]
            got = capi._SIGS[name][0][i]
            assert got is want, f"{name} parameter {i} ({p}): ctypes {got.__name__}"
            checked += 1
    assert checked > 100

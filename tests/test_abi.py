"""The C ABI library loads without a GPU and exports every function that
include/dsb/dsb.h declares (no compute calls are made here)."""

import ctypes

import deepseek_cpp_infer_b200 as dsb


def test_library_exports_every_header_function():
    names = dsb.header_functions()
    assert "dsb_mla_decode" in names and "dsb_ctx_create" in names
    l = ctypes.CDLL(dsb.LIB_PATH)
    missing = [n for n in names if not hasattr(l, n)]
    assert not missing, missing


def test_bindings_cover_header():
    declared = set(dsb.header_functions())
    bound = {name for name, _, _ in dsb._PROTOS}
    assert declared == bound, declared ^ bound


def test_version_and_null_context_errors():
    l = dsb.lib()
    assert l.dsb_version() >= 100
    assert l.dsb_ctx_destroy(None) == dsb.DSB_OK
    assert l.dsb_sync(None) == dsb.DSB_EINVAL
    assert l.dsb_last_error(None) == b"null context"

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


def test_header_is_plain_c_and_links(tmp_path):
    """include/dsb/dsb.h compiles as C99 and C++17 with warnings as errors; a C
    program links against libdsb.so and runs its host-only entry points
    without a GPU (version, checkpoint and tokenizer errors)."""
    import os
    import subprocess

    inc = os.path.join(os.path.dirname(os.path.dirname(os.path.abspath(__file__))), "include")
    libdir = os.path.dirname(dsb.LIB_PATH)
    src = tmp_path / "use_dsb.c"
    src.write_text(r'''
#include <stdio.h>
#include <string.h>
#include "dsb/dsb.h"
int main(void) {
  dsb_checkpoint* ck = NULL;
  dsb_tokenizer* tk = NULL;
  int rc1 = dsb_checkpoint_open("/nonexistent-model-dir", &ck);
  int rc2 = dsb_tokenizer_load("/nonexistent-tokenizer.json", &tk);
  printf("%d %d %d %d %d\n", dsb_version() >= 100, rc1 == DSB_EINVAL, ck == NULL, rc2 == DSB_EINVAL,
         strstr(dsb_checkpoint_error(), "config.json") != NULL);
  return 0;
}
''')
    exe = tmp_path / "use_dsb"
    subprocess.run(["gcc", "-std=c99", "-Wall", "-Wextra", "-Werror", "-pedantic", f"-I{inc}", str(src), "-o",
                    str(exe), f"-L{libdir}", "-ldsb", f"-Wl,-rpath,{libdir}"], check=True)
    out = subprocess.run([str(exe)], check=True, capture_output=True, text=True).stdout.split()
    assert out == ["1"] * 5, out
    cxx = tmp_path / "use_dsb.cpp"
    cxx.write_text('#include "dsb/dsb.h"\nint main() { return dsb_version() > 0 ? 0 : 1; }\n')
    subprocess.run(["g++", "-std=c++17", "-Wall", "-Wextra", "-Werror", "-pedantic", f"-I{inc}", "-fsyntax-only",
                    str(cxx)], check=True)

"""The C ABI library loads on a machine without a GPU and exports every symbol the public header
declares (no compute calls are made here)."""

import re
from pathlib import Path

import pytest

from ripvec_b200 import _lib
from ripvec_b200.build import LIB, build

HEADER = Path(__file__).resolve().parents[1] / "include" / "ripvec_b200.h"


def declared_symbols():
    text = HEADER.read_text()
    text = re.sub(r"/\*.*?\*/", "", text, flags=re.S)
    return sorted(set(re.findall(r"\b(rv_[a-z0-9_]+)\s*\(", text)))


@pytest.fixture(scope="module")
def lib():
    build()  # no-op when up to date; nvcc cross-compiles for sm_100a without a GPU
    assert LIB.exists()
    return _lib.lib()


def test_library_exports_every_declared_symbol(lib):
    syms = declared_symbols()
    assert len(syms) >= 20
    missing = [s for s in syms if not hasattr(lib, s)]
    assert not missing, missing


def test_binding_table_covers_the_header():
    assert sorted(_lib.SIGNATURES) == declared_symbols()


def test_null_arguments_are_rejected_without_a_device(lib):
    import ctypes as C

    assert lib.rv_create(None, 0, None) == _lib.RV_E_INVALID
    assert lib.rv_index_create(0, None, 0, 63, _lib.RV_DTYPE_F32, 0, C.byref(C.c_void_p())) == _lib.RV_E_INVALID
    d = _lib.ModelDesc()
    d.arch = 99
    assert lib.rv_create(C.byref(d), 0, C.byref(C.c_void_p())) == _lib.RV_E_INVALID
    assert lib.rv_last_error(None) == b"null context"


def test_search_entry_points_reject_a_null_index_without_a_device(lib):
    """Every PolarQuant, cascade and duplicate-pair entry point checks its handle before touching
    a device."""
    import ctypes as C

    inv = _lib.RV_E_INVALID
    assert lib.rv_index_build_polar(None, None, 4) == inv
    assert lib.rv_index_has_polar(None) == 0
    assert lib.rv_index_polar_export(None, None, None) == inv
    assert lib.rv_index_polar_scores(None, None, 1, None) == inv
    assert lib.rv_index_rank_turboquant(None, None, 1, 10, 0.0, None, None, None, None) == inv
    assert lib.rv_index_rank_turboquant_device(None, None, 1, 10, 0.0, None, None, None, None) == inv
    assert lib.rv_index_build_cascade(None, 64) == inv
    assert lib.rv_index_cascade_dim(None) == 0
    assert lib.rv_index_cascade_rows(None, None) == inv
    assert lib.rv_index_rank_cascade(None, None, 1, 10, 0.0, None, None, None, None) == inv
    cnt = C.c_int64(-1)
    assert lib.rv_index_find_duplicates(None, 0.85, 20, None, None, None, None, C.byref(cnt)) == inv
    assert lib.rv_index_rank(None, None, 0.0, 0, None, None, None, C.byref(cnt)) == inv
    assert lib.rv_index_topk_noalloc(None, None, 1, 10, 0.0, None, None, None, None) == inv
    assert lib.rv_index_topk_noalloc(None, None, 0, 10, 0.0, None, None, None, None) == inv
    assert lib.rv_index_last_error(None) == b"null index"
    # the exponential test hook checks its arguments before it touches a device
    assert lib.rv_debug_exp2_poly(None, None, 0, None) == _lib.RV_OK
    assert lib.rv_debug_exp2_poly(None, None, 4, None) == inv
    assert lib.rv_debug_exp2_poly(None, None, -1, None) == inv


def test_noalloc_argument_checks_without_a_device(lib):
    """rv_index_topk_noalloc checks its limits before it touches a device: an empty (n = 0)
    index needs no device copy, so it is created here on a machine without a GPU only if the
    runtime allows it; the limit checks are then exercised, and nq = 0 returns RV_OK."""
    import ctypes as C

    h = C.c_void_p()
    rc = lib.rv_index_create(0, None, 0, 64, _lib.RV_DTYPE_F32, 0, C.byref(h))
    if rc != _lib.RV_OK:
        pytest.skip("no CUDA runtime device for an index handle")
    try:
        assert lib.rv_index_topk_noalloc(h, None, 0, 10, 0.0, None, None, None, None) == _lib.RV_OK
        assert lib.rv_index_topk_noalloc(h, None, 17, 10, 0.0, None, None, None, None) == _lib.RV_E_INVALID
        assert b"at most 16 queries" in lib.rv_index_last_error(h)
        assert lib.rv_index_topk_noalloc(h, None, 1, 65, 0.0, None, None, None, None) == _lib.RV_E_INVALID
        assert lib.rv_index_topk_noalloc(h, None, 1, 10, 0.0, None, None, None, None) == _lib.RV_E_INVALID
    finally:
        lib.rv_index_destroy(h)


def test_model_desc_layout_matches_header(tmp_path):
    """The ctypes mirror of rv_model_desc has the size and field offsets a C compiler gives."""
    import ctypes as C
    import shutil
    import subprocess

    cc = shutil.which("gcc") or shutil.which("cc")
    if cc is None:
        pytest.skip("no C compiler")
    src = tmp_path / "layout.c"
    src.write_text('#include <stddef.h>\n#include <stdio.h>\n#include "ripvec_b200.h"\n'
                   'int main(void){printf("%zu %zu %zu", sizeof(rv_model_desc),'
                   ' offsetof(rv_model_desc, norm_eps), offsetof(rv_model_desc, max_batch_tokens));return 0;}\n')
    exe = tmp_path / "layout"
    subprocess.run([cc, f"-I{HEADER.parent}", str(src), "-o", str(exe)], check=True)
    size, eps_off, mbt_off = map(int, subprocess.run([str(exe)], capture_output=True, text=True).stdout.split())
    assert C.sizeof(_lib.ModelDesc) == size
    assert _lib.ModelDesc.norm_eps.offset == eps_off
    assert _lib.ModelDesc.max_batch_tokens.offset == mbt_off

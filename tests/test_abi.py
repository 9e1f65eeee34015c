"""The C ABI: the library builds, loads and exports every entry point include/fanar_b200.h declares; argument checks
return FVS_EINVAL / FVS_ERANGE before any device work (so these run without a GPU)."""
import ctypes as C
import os
import re

import pytest

from conftest import REPO, pkg


@pytest.fixture(scope="module")
def lib():
    pkg("build").build()
    return pkg("_lib").lib()


def declared():
    src = open(os.path.join(REPO, "include", "fanar_b200.h")).read()
    return sorted(set(re.findall(r"^\s*(?:int|uint32_t|const char\*)\s+(fvs_\w+)\s*\(", src, re.M)))


def test_every_declared_symbol_is_exported(lib):
    names = declared()
    assert len(names) >= 10
    for n in names:
        assert hasattr(lib, n), n
    assert set(names) == set(pkg("_lib").SIGNATURES), "ctypes signatures and header disagree"


def test_identity(lib):
    assert lib.fvs_arch() == b"sm_100a"
    assert lib.fvs_version() >= 100
    assert lib.fvs_i8_tile_rows() % 32 == 0


def test_argument_errors(lib):
    n = None
    # bad mode / R / nulls
    assert lib.fvs_i8_scan(n, 2, n, n, 1, 256, n, n, n, n, n, n, 1, n, 1, n, n, n, n, n, n, 1, n, 1) == -1
    assert lib.fvs_i8_scan(n, 0, n, n, 1, 128, n, n, n, n, n, n, 1, n, 1, n, n, n, n, n, n, 1, n, 1) == -1
    assert lib.fvs_threshold(n, n, 4, n, n, 8, 2, n, 1, 1, n) == -1
    dummy = C.c_void_p(16)
    assert lib.fvs_select_topk(n, dummy, dummy, dummy, 1, 10, 5000, dummy, dummy, dummy, n, 0.0, 0) == -2
    assert lib.fvs_refine(n, dummy, 1536, dummy, dummy, dummy, dummy, 1, 10, 1.0, 10, dummy, 1536, dummy, dummy,
                          dummy, n) == -1  # K must exceed k
    assert lib.fvs_merge_topk(n, dummy, dummy, 8, 1, 1024, 10, dummy, n) == -2
    odd = C.c_void_p(20)                                   # not 16-byte aligned: the row loads would fault
    assert lib.fvs_exact_scores(n, odd, 1536, dummy, 1, 10, dummy, 1536, dummy) == -1
    assert lib.fvs_exact_scores(n, dummy, 1536, dummy, 1, 10, odd, 1536, dummy) == -1
    T = (C.c_int32 * 9)(*range(9))
    assert lib.fvs_lut_build(n, dummy, 1, 64, 64, 1, dummy, 9, T, T, dummy, dummy) == -2  # more than 8 tiers


def test_zero_batch_is_a_no_op(lib):
    dummy = C.c_void_p(16)
    assert lib.fvs_select_topk(None, dummy, dummy, dummy, 0, 10, 20, dummy, dummy, dummy, None, 0.0, 0) == 0

"""ctypes binding of libfanar_b200.so (the C ABI declared in include/fanar_b200.h).

The library is loaded from this package directory.  There is no fallback: if the shared object is missing or does not
export a declared symbol, loading raises, and every search entry point fails loudly.
"""
from __future__ import annotations

import ctypes as C
import os

HERE = os.path.dirname(os.path.abspath(__file__))
LIB_PATH = os.path.join(HERE, "libfanar_b200.so")

P = C.c_void_p
I32 = C.c_int
I64 = C.c_int64
F32 = C.c_float

# name -> (restype, argtypes); mirrors include/fanar_b200.h
SIGNATURES = {
    "fvs_version": (I32, []),
    "fvs_arch": (C.c_char_p, []),
    "fvs_i8_tile_rows": (I32, []),
    "fvs_set_wait_limit": (C.c_uint32, [C.c_uint32]),
    "fvs_quantize": (I32, [P, P, I32, I32, I32, P, P]),
    "fvs_query_prep": (I32, [P, P, I32, I32, I32, P, P, P]),
    "fvs_route_topk": (I32, [P, P, I32, I32, I32, P]),
    "fvs_pairs": (I32, [P, P, I32, I32, I32, I32, P, P, P, P, P, P, P, P]),
    "fvs_pairs_split": (I32, [P, P, I32, I32, I32, I32, P, P, P, P, P, P, P, P, P]),
    "fvs_pairs_noalloc": (I32, [P, P, I32, I32, I32, I32, P, P, P, P, P, P, P]),
    "fvs_i8_scan": (I32, [P, I32, P, P, I32, I32, P, P, P, P, P, P, I32, P, I32, P, P, P, P, P, P, I32, P, I32]),
    "fvs_i8_scan_tc": (I32, [P, I32, P, P, I32, I32, P, P, P, P, P, P, I32, P, I32, P, I64, P, P, P, P, P, I32, P,
                              I32, P]),
    "fvs_i8_scan_cells": (I32, [P, I32, P, P, I32, I32, P, P, P, P, P, P, I32, P, I32, P, I64, P, P, P, P, P, I32, P,
                                 I32, P, P]),
    "fvs_route_pairs": (I32, [P, P, I32, I32, I32, I32, P, P, I32, P, P, P, P, P, P, P, P, P, P, P, I32, P]),
    "fvs_route_pairs_scaled": (I32, [P, P, I32, I32, I32, I32, P, P, P, I32, P, P, P, P, P, P, P, P, P, P, P, I32,
                                      P]),
    "fvs_cell_part_tiles": (I32, []),
    "fvs_cell_lists": (I32, [P, P, I32, P, P, P, P, P, P, I32]),
    "fvs_threshold": (I32, [P, P, I32, P, P, I32, I32, P, I32, I32, P]),
    "fvs_select_topk": (I32, [P, P, P, P, I32, I32, I32, P, P, P, P, F32, I32]),
    "fvs_lut_build": (I32, [P, P, I32, I32, I32, I32, P, I32, P, P, P, P]),
    "fvs_lut_score": (I32, [P, P, I32, I32, P, P, I32, I32, I32, P, P, P, P, P, P, P, I64, P, P, P, P, P]),
    "fvs_lut_score_zq": (I32, [P, P, I32, I32, P, P, I32, I32, I32, I32, I32, P, P, P, P, P, P, P, I64, P, P, P]),
    "fvs_refine": (I32, [P, P, I32, P, P, P, P, I32, I32, F32, I32, P, I32, P, P, P, P]),
    "fvs_i8_scan_small": (I32, [P, I32, P, P, I32, I32, P, I32, I32, P, I32, P, P, P, P, P, P, P, P, I32, P, I32]),
    "fvs_project_quantize": (I32, [P, P, I32, I32, I32, P, P, I32, P, P, P, I32, P]),
    "fvs_trellis_tile_rows": (I32, []),
    "fvs_trellis_scan": (I32, [P, I32, P, I32, I32, P, P, P, P, P, P, I32, P, I32, P, I32, P, I32, P, P, P, P, P,
                                I32, P, I32]),
    "fvs_trellis_scan_cells": (I32, [P, I32, P, I32, I32, P, P, P, P, P, P, I32, P, I32, P, I32, P, I32, P, P, P, P,
                                      P, I32, P, I32, P, P]),
    "fvs_trellis_scan_small": (I32, [P, I32, P, I32, I32, P, I32, I32, P, I32, P, P, I32, P, I32, P, P, P, P, P, I32, P,
                                      I32, I32]),
    "fvs_tiered_score": (I32, [P, P, I32, I32, P, P, I32, I32, I32, P, P, P, P, P, P, P, I64, P, P]),
    "fvs_route_topk_scaled": (I32, [P, P, I32, I32, I32, P, P]),
    "fvs_viterbi_encode": (I32, [P, P, I32, I32, P, I32, P]),
    "fvs_dense_scan_tc": (I32, [P, I32, P, P, I32, I32, P, P, I64, P, P, P, P, I32, P, I64, P]),
    "fvs_rth_largest": (I32, [P, P, I32, I32, I64, I32, P]),
    "fvs_lut_score_rec": (I32, [P, P, I32, I32, P, P, I32, I32, I32, I32, I32, P, P, P, P, P, I32, I32, I64, P, P,
                                 P]),
    "fvs_tiered_score_rec": (I32, [P, P, I32, I32, P, P, I32, I32, I32, P, P, P, P, P, I32, I32, I64, P, P]),
    "fvs_flagged_gather": (I32, [P, P, I32, I32, P, P, I32, P, P, P]),
    "fvs_rows_scatter": (I32, [P, P, I32, I32, P, I32, P, P, P]),
    "fvs_exact_scores": (I32, [P, P, I32, P, I32, I32, P, I32, P]),
    "fvs_merge_topk": (I32, [P, P, P, I32, I32, I32, I32, P, P]),
}

ERRORS = {-1: "FVS_EINVAL (bad argument)", -2: "FVS_ERANGE (size above the kernel's limit)"}


class FvsError(RuntimeError):
    pass


_lib = None


def lib():
    """The loaded library (loaded on first use)."""
    global _lib
    if _lib is None:
        if not os.path.exists(LIB_PATH):
            raise FvsError(f"{LIB_PATH} is missing: build it with `python fanarvse-paper_b200/build.py` "
                           "(the CUDA library is required; there is no CPU path)")
        L = C.CDLL(LIB_PATH)
        for name, (res, args) in SIGNATURES.items():
            fn = getattr(L, name)  # AttributeError if the library lacks a declared entry point
            fn.restype = res
            fn.argtypes = args
        _lib = L
    return _lib


def check(rc: int, what: str):
    if rc != 0:
        msg = ERRORS.get(rc, f"CUDA error {rc}")
        raise FvsError(f"{what} failed: {msg}")


def ptr(t):
    """device (or host) address of a tensor, or None."""
    return None if t is None else C.c_void_p(t.data_ptr())


def stream_handle(torch_stream=None):
    import torch
    s = torch_stream if torch_stream is not None else torch.cuda.current_stream()
    return C.c_void_p(s.cuda_stream)


def i32_array(vals):
    return (C.c_int32 * len(vals))(*[int(v) for v in vals])


def f32_array(vals):
    return (C.c_float * len(vals))(*[float(v) for v in vals])


def ptr_array(tensors):
    return (C.c_void_p * len(tensors))(*[t.data_ptr() for t in tensors])

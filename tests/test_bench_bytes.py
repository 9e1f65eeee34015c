"""The algorithmic byte counts behind bench.py's roofline lines, on a toy index with hand-counted answers."""
import importlib.util
import os
import types

import numpy as np
import torch

HERE = os.path.dirname(os.path.abspath(__file__))


def _bench():
    spec = importlib.util.spec_from_file_location("bench_mod", os.path.join(os.path.dirname(HERE), "bench.py"))
    m = importlib.util.module_from_spec(spec)
    spec.loader.exec_module(m)
    return m


def _engine(last, off, TS=((0, 32, 4), (32, 64, 2)), rec=True):
    T = len(TS)
    ix = types.SimpleNamespace(off_np=np.asarray(off, np.int64), TS=list(TS), T=T, D=TS[-1][1],
                               rec=torch.zeros(1) if rec else None, RB=32)
    return types.SimpleNamespace(ix=ix, _last=last)


# cells of 40, 0, 70 and 16 rows: global 32-row blocks per cell 2, 0, 3 (rows 40..109 touch blocks 1, 2, 3) and 1
OFF = [0, 40, 40, 110, 126]


def test_first_pass_bytes_from_cell_counts():
    b = _bench()
    ccnt1 = torch.tensor([3, 0, 1, 0], dtype=torch.int32)       # pairs of the first pass by cell
    E = _engine(dict(ccnt1=ccnt1), OFF)
    B, R = 5, 256
    rows = 40 + 70                                               # cells probed by the first pass
    blocks = 3 * 2 + 1 * 3                                       # one block maximum per (pair, block of its cell)
    assert b.first_bytes(E, B, R) == rows * (R + 4) + 4 * 8 + B * (R + 12) + blocks * 4


def test_first_pass_bytes_streaming_scan():
    b = _bench()
    probe = torch.tensor([[2, 0, 3], [2, 3, 0]])                 # first n1 = 2 columns: cells {2, 0} and {2, 3}
    E = _engine(dict(probe=probe, n1=2), OFF)
    rows = 40 + 70 + 16
    blocks = 2 + 3 * 2 + 1
    assert b.first_bytes(E, 2, 256) == rows * 260 + 4 * 8 + 2 * 268 + blocks * 4


def test_emit_bytes_counts_probed_cells_once_and_clamps_to_the_buffer():
    b = _bench()
    ccnt = torch.tensor([2, 0, 5, 1], dtype=torch.int32)
    cnt = torch.tensor([10, 9000, 0], dtype=torch.int32)        # the second query overflowed an 8192-entry buffer
    E = _engine(dict(ccnt=ccnt, cnt=cnt, M=8192, npairs=8), OFF)
    assert b.emit_bytes(E, 3, 256) == (40 + 70 + 16) * 260 + 8 * 8 + 3 * 268 + (10 + 8192) * 8


def test_lut_bytes_per_live_candidate():
    b = _bench()
    ncnt = torch.tensor([7, 0, 100], dtype=torch.int32)
    E = _engine(dict(ncnt=ncnt), OFF)
    assert b.lut_bytes(E, 3) == 107 * (32 + 16) + 3 * (64 * 4 + 4)
    E = _engine(dict(ncnt=None, est=torch.zeros(3, 4)), OFF, rec=False)
    per = (32 * 4 + 32 * 2) // 8 + 4 * 2                          # plane bytes + (scale, sigma) per tier
    assert b.lut_bytes(E, 3) == 12 * (per + 16) + 3 * (64 * 4 + 4)

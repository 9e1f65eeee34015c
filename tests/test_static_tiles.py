"""Host-side work list of the int8 scan: tiles cover every row of every cell exactly once, start on global 32-row
boundaries, and MB matches the reference's `_static_make` (`src/s1cell.py:161-168`)."""
import numpy as np
import pytest

from conftest import pkg
from oracle import fvs_oracle as O


@pytest.mark.parametrize("seed", [0, 1, 2])
@pytest.mark.parametrize("tile_rows", [128, 256])
def test_tiles_cover_cells(seed, tile_rows):
    rng = np.random.default_rng(seed)
    sizes = rng.integers(0, 400, 64)
    sizes[:5] = [0, 1, 31, 32, 33]
    off = np.concatenate([[0], np.cumsum(sizes)])
    cell, row0, MB = pkg("engine").static_tiles(off, tile_rows)
    assert MB == O.static_blocks(off)[4]
    assert (row0 % 32 == 0).all()
    for c in range(len(sizes)):
        t = row0[cell == c]
        cover = np.zeros(off[-1] + tile_rows + 64, int)
        for r in t:
            cover[r:r + tile_rows] += 1
        assert (cover[off[c]:off[c + 1]] == 1).all()
        if sizes[c]:
            assert t.min() == (off[c] // 32) * 32 and t.max() < off[c + 1]
        else:
            assert len(t) == 0


@pytest.mark.parametrize("seed", [0, 1])
@pytest.mark.parametrize("part_tiles", [1, 3, 8])
def test_cell_parts_cover_cells(seed, part_tiles):
    """The cell-major scans' work-list order (`cell | part << 16`): decoded as the scans' producers decode an entry --
    first row (cs & ~31) + part * part_tiles * 128, at most part_tiles tiles of 128 rows up to the cell's end -- the
    parts of every listed cell cover its rows exactly once, in the listed cell order, one empty part for an empty
    cell."""
    rng = np.random.default_rng(seed)
    sizes = rng.integers(0, 4000, 48)
    sizes[:6] = [0, 1, 127, 128, 129, 3 * 128 * part_tiles + 5]
    off = np.concatenate([[0], np.cumsum(sizes)])
    order = np.argsort(-sizes, kind="stable")
    e = pkg("engine").cell_part_order(off, order, part_tiles)
    assert e.dtype == np.int32
    cells, parts = e & 0xffff, e >> 16
    # cells appear in the given order, each as a run of parts 0, 1, ...
    runs = [c for i, c in enumerate(cells) if i == 0 or c != cells[i - 1]]
    assert runs == list(order)
    cover = np.zeros(off[-1] + 1024, int)
    for c, p in zip(cells, parts):
        cs, ce = off[c], off[c + 1]
        first = (cs & ~31) + p * part_tiles * 128
        if ce <= cs:
            assert p == 0
            continue
        assert first < ce
        ntiles = min(part_tiles, (ce - first + 127) // 128)
        lo, hi = max(first, cs), min(first + ntiles * 128, ce)
        cover[lo:hi] += 1
    assert (cover[:off[-1]] == 1).all() and not cover[off[-1]:].any()

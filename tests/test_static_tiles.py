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

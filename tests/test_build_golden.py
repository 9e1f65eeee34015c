"""The repository's index build reproduces the reference's build byte for byte on identical inputs.

`tests/golden/build_reference.npz` holds the outputs of the reference's own `build_codes`, `tiered.allocate`,
`tiered.DIST`, `uniform_cb`, `encode_uniform` and `tiered.build` (run by `tests/golden/make_golden_build.py` on CPU
tensors, with the 1-D codebooks that faiss would fit supplied as the Lloyd-Max levels).  Every array the query kernels
read -- int8 codes and scales, the projection, the tier table, uniform steps, bit planes, rotations, fp16 scales and
sigmas -- is compared exactly."""
import os

import numpy as np
import pytest
import torch

from conftest import GOLDEN, pkg


@pytest.fixture(scope="module")
def gb():
    return dict(np.load(os.path.join(GOLDEN, "build_reference.npz")))


@pytest.fixture(scope="module")
def ib():
    return pkg("index_build")


def _inputs(f):
    X16 = torch.from_numpy(f["X16"])
    order = torch.from_numpy(f["order"]).long()
    off_t = torch.from_numpy(f["off"])
    return X16, order, off_t


def test_int8_codes_match_reference(gb, ib):
    f = gb
    X16, order, off_t = _inputs(f)
    Z, zs, Vr = ib.build_i8_codes(X16, order, off_t, torch.from_numpy(f["means16"]), torch.from_numpy(f["Vp"]), 256)
    np.testing.assert_array_equal(Z.numpy(), f["Z"])
    np.testing.assert_array_equal(zs.numpy(), f["zs"])
    np.testing.assert_array_equal(Vr.numpy(), f["Vr"])


def test_mse_table_and_tiers_match_reference(gb, ib):
    f = gb
    np.testing.assert_array_equal(np.array([ib.dist(b) for b in range(9)]), f["DIST"])
    TS = ib.allocate(torch.from_numpy(f["lam"]), int(f["bits"]))
    np.testing.assert_array_equal(np.array(TS, np.int64), f["TS"])
    # the same water-filling given an explicit table
    TS2 = ib.allocate(torch.from_numpy(f["lam"]), int(f["bits"]), dist_table={b: float(f["DIST"][b]) for b in range(9)})
    assert TS2 == TS


def test_uniform_steps_match_reference(gb, ib):
    """`uniform_cb`'s step, restated, on the same device and sample count as the golden run"""
    f = gb
    got = [ib.uniform_delta_sampled(int(b), "cpu", n=20000) for b in f["uniform_widths"]]
    np.testing.assert_array_equal(np.array(got), f["uniform_delta"])


def _cb_uniform(deltas):
    CB = {}
    for b, dl in deltas.items():
        lv = (torch.arange(2 ** b).float() - (2 ** b - 1) / 2) * dl
        CB[b] = (lv, (lv[1:] + lv[:-1]) / 2)
    return CB


def test_tiered_uniform_code_matches_reference(gb, ib):
    f = gb
    X16, order, _ = _inputs(f)
    TS = [tuple(int(v) for v in r) for r in f["TS"]]
    deltas = {int(b): float(d) for b, d in zip(f["uniform_widths"], f["uniform_delta"])}
    cu = ib.tiered_build(X16, order, torch.from_numpy(f["c"]), torch.from_numpy(f["V"]), TS, _cb_uniform(deltas),
                         seed=int(f["seed"]))
    for t in range(len(TS)):
        np.testing.assert_array_equal(cu["rots"][t].numpy(), f[f"rot{t}"])
        np.testing.assert_array_equal(cu["planes"][t].numpy(), f[f"u_planes{t}"])
    np.testing.assert_array_equal(cu["scale"].numpy(), f["u_scale"])
    np.testing.assert_array_equal(cu["sig"].numpy(), f["u_sig"])


def test_tiered_lloyd_code_matches_reference(gb, ib):
    f = gb
    X16, order, _ = _inputs(f)
    TS = [tuple(int(v) for v in r) for r in f["TS"]]
    CB = {}
    for b in sorted({bb for _, _, bb in TS}):
        lv = ib.lloyd_levels_f32(b)
        CB[b] = (torch.from_numpy(lv), torch.from_numpy((lv[1:] + lv[:-1]) / 2))
    cl = ib.tiered_build(X16, order, torch.from_numpy(f["c"]), torch.from_numpy(f["V"]), TS, CB, seed=int(f["seed"]))
    for t in range(len(TS)):
        np.testing.assert_array_equal(cl["planes"][t].numpy(), f[f"l_planes{t}"])
    np.testing.assert_array_equal(cl["scale"].numpy(), f["l_scale"])
    np.testing.assert_array_equal(cl["sig"].numpy(), f["l_sig"])


def test_build_index_uses_the_reference_steps(ib):
    """a host build takes the exact-density step; it sits on the reference's grid next to the sampled one"""
    grid = np.linspace(0.02, 2.5, 600)
    for b in (1, 2, 3):
        a = ib.uniform_delta(b)
        s = ib.uniform_delta_sampled(b, "cpu", n=20000)
        assert a in grid and s in grid
        assert abs(np.searchsorted(grid, a) - np.searchsorted(grid, s)) <= 30

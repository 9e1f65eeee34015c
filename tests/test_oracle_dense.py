"""Pin the oracle's routing-free int8 scan (`throughput/brute.py` `Brute`) to the reference's own outputs: codes,
query codes, sample scores, thresholds, emit counts and sets, stage-1 top-K and flags, bit for bit."""
import os

import numpy as np
import pytest
import torch

from conftest import GOLDEN
from oracle import fvs_oracle as O


@pytest.fixture(scope="module")
def gd():
    return dict(np.load(os.path.join(GOLDEN, "dense_reference.npz")))


@pytest.mark.parametrize("tag", ["a_", "b_"])
def test_dense_codes_and_scan_match_reference(gd, tag):
    f = gd
    R, K, M = (int(v) for v in f[tag + "params"])
    # the projections themselves are fp32 GEMMs whose summation order belongs to the BLAS (it changes with the CPU's
    # vector width and thread count): on the machine that made the fixture the quantisation of torch's product was
    # bit-exact; elsewhere a last-bit difference in a product can move a code by one step or a row scale by one fp16
    # step, so those are allowed on a handful of entries.  Everything below starts from the reference's own codes.
    V = torch.from_numpy(f["V"])[:, :R]
    mu = torch.from_numpy(f["mu"])
    zx = ((torch.from_numpy(f["X16"]).float() - mu) @ V).numpy()
    Z, a = O._i8code(zx)
    dz = np.abs(Z.astype(np.int32) - f[tag + "Z"].astype(np.int32))
    assert dz.max() <= 1 and (dz != 0).mean() < 1e-3
    a16, g16 = a.astype(np.float16), f[tag + "zs"]
    ulp = np.abs(a16.view(np.int16).astype(np.int32) - g16.view(np.int16).astype(np.int32))
    assert ulp.max() <= 1 and (ulp != 0).mean() < 2e-3
    Zn, zsn = O.dense_codes(f["X16"], f["mu"], f["V"], R)
    assert (Zn != f[tag + "Z"]).mean() < 1e-3
    np.testing.assert_allclose(zsn.astype(np.float32), f[tag + "zs"].astype(np.float32), rtol=1e-3)
    zq = ((torch.from_numpy(f["Q"]) - mu) @ V).numpy()
    q8, qs = O._i8code(zq)
    dq = np.abs(q8.astype(np.int32) - f[tag + "q8"].astype(np.int32))
    assert dq.max() <= 1 and (dq != 0).mean() < 1e-3
    np.testing.assert_allclose(qs, f[tag + "qs"], rtol=2e-6)
    Z, zs, q8, qs = f[tag + "Z"], f[tag + "zs"], f[tag + "q8"], f[tag + "qs"]
    out = O.dense_search(q8, qs, Z, zs, K, over=float(f[tag + "over"]), M=M)
    np.testing.assert_array_equal(out["sample"], f[tag + "sample_scores"])
    np.testing.assert_array_equal(out["t0"], f[tag + "t0"])
    np.testing.assert_array_equal(out["cnt"], f[tag + "cnt"])
    np.testing.assert_array_equal(out["ok"], f[tag + "ok"])
    eq, ev, ep = f[tag + "emit_q"], f[tag + "emit_val"], f[tag + "emit_pos"]
    for q in range(len(out["cnt"])):
        sel = eq == q
        o = np.argsort(ep[sel])
        if out["cnt"][q] <= M:                   # the reference's buffer holds every emitted row
            np.testing.assert_array_equal(ep[sel][o], out["pos_l"][q])
            np.testing.assert_array_equal(ev[sel][o], out["est_l"][q])
        else:                                    # overflow: the reference kept M of them (which ones is racy)
            assert sel.sum() == M and np.isin(ep[sel], out["pos_l"][q]).all()
    for q in np.nonzero(out["ok"])[0]:
        np.testing.assert_array_equal(np.sort(out["pos"][q]), np.sort(f[tag + "pos"][q]))
        np.testing.assert_array_equal(np.sort(out["est"][q]), np.sort(f[tag + "est"][q]))

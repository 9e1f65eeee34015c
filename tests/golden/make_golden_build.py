"""Golden vectors of the reference's index build (run in the build container, not on the GPU box).

Runs, on CPU tensors, the reference's own build functions for the arrays the query path consumes:
  * `enginei8.build_codes` (`throughput/enginei8.py:19-27`): int8 stage-1 codes Z, scales zs, projection Vr;
  * `tiered.allocate` (`src/tiered.py:19-27`): the water-filling tier table TS, and `tiered.DIST`;
  * `s2lut.uniform_cb` (`throughput/s2lut.py:9-16`): the uniform step per bit width;
  * `s2lut.encode_uniform` -> `tiered.build` (`throughput/s2lut.py:18-29`, `src/tiered.py:29-44`): uniform-codebook
    planes, scales and sigmas, and the Haar rotations;
  * `tiered.build` with the module's own (Lloyd-Max) codebooks: planes, scales and sigmas.

Stand-ins, each for something this container lacks:
  * `faiss` (imported by `tiered` for its 1-D codebooks, `src/tiered.py:3-10`): a `Kmeans` whose `train` yields the
    Lloyd-Max levels of N(0,1) (`index_build.lloyd_levels_f32`).  faiss is unpinned in the reference's requirements;
    everything the module derives from the levels (DIST, thresholds, CB) is computed by the reference's own code.
  * the modules' device constant: `tiered` runs its codebook set-up at import with `dev = "cuda"`, so its source is
    executed with that one assignment set to "cpu"; `s2lut` / `enginei8` read `dev` at call time and are set after
    import (as `make_golden.py` does).
  * `uniform_cb`'s sample count inside `encode_uniform` is lowered from 2,000,000 to N_UNIFORM so that the CPU run takes
    seconds; the count is an argument of the reference function, and the fixture records the steps it gave.
  * `engine_cell`, `engine3`, `civf8`: the stand-ins of `make_golden.py` (only so that `enginei8` imports).

Inputs (X16, the cell assignment, the PCA bases) come from this repository's build of a small synthetic set; the
fixture stores them, so the test feeds identical inputs to `index_build` and compares every output byte for byte.

Usage:  python tests/golden/make_golden_build.py --ref <checkout of the reference repository> [--out tests/golden]
"""
from __future__ import annotations

import argparse
import importlib
import os
import sys
import types

os.environ["TRITON_INTERPRET"] = "1"

import numpy as np
import torch

HERE = os.path.dirname(os.path.abspath(__file__))
REPO = os.path.dirname(os.path.dirname(HERE))
sys.path.insert(0, REPO)
sys.path.insert(0, HERE)
synth = importlib.import_module("fanarvse-paper_b200.synth")
ib = importlib.import_module("fanarvse-paper_b200.index_build")

N_UNIFORM = 20000


def load_reference(ref):
    import make_golden as mg
    faiss = types.ModuleType("faiss")

    class Kmeans:
        def __init__(self, d, k, niter=None, seed=None):
            self.k = k

        def train(self, x):
            self.centroids = ib.lloyd_levels_f32(int(np.log2(self.k)))[:, None].copy()

    faiss.Kmeans = Kmeans
    sys.modules["faiss"] = faiss
    sys.path[:0] = [f"{ref}/throughput", f"{ref}/src"]
    src = open(f"{ref}/src/tiered.py").read()
    assert src.count('dev = "cuda"') == 1
    tiered = types.ModuleType("tiered")
    tiered.__file__ = f"{ref}/src/tiered.py"
    exec(compile(src.replace('dev = "cuda"', 'dev = "cpu"'), tiered.__file__, "exec"), tiered.__dict__)
    sys.modules["tiered"] = tiered
    mods = mg.load_reference(ref)            # stubs engine_cell / engine3 / civf8 (and an empty tiered) ...
    sys.modules["tiered"] = tiered           # ... so put the real one back for s2lut
    s2lut = importlib.reload(mods["s2lut"])
    s2lut.dev = "cpu"
    mods["s2lut"], mods["tiered"] = s2lut, tiered
    mods["enginei8"].dev = "cpu"
    return mods


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--ref", required=True)
    ap.add_argument("--out", default=HERE)
    a = ap.parse_args()
    mods = load_reference(a.ref)
    tiered, s2lut, ei = mods["tiered"], mods["s2lut"], mods["enginei8"]

    n, d, nlist, seed = 1500, 256, 12, 5
    ds = synth.make_dataset(synth.MixtureSpec(n=n, d=d, comps=6, nq=4, seed=seed), "cpu", gt_k=10)
    X16 = ds["base16"]
    with torch.no_grad():
        c = X16[:50000].float().mean(0)
        cen = ib.spherical_kmeans(X16, nlist, seed, n, 15)
        order, off_t = ib.assign_cells(X16, cen)
        means16 = ib.cell_means(X16, order, off_t).half()
        mu = X16.float().mean(0)
        _, Vp = ib.pca_eigh(X16[::2].float() - mu)                      # int8 code basis
        S = X16.float() - c
        S = S / S.norm(dim=1, keepdim=True)
        lam, V = ib.pca_eigh(S)                                         # refinement basis
        lam = lam.clamp(min=1e-12)
    bits = int(2.5 * d)
    out = dict(X16=X16.numpy(), order=order.to(torch.int32).numpy(), off=off_t.numpy(), means16=means16.numpy(),
               c=c.numpy(), Vp=Vp.numpy(), V=V.numpy(), lam=lam.numpy(), bits=np.int64(bits), seed=np.int64(seed))

    # int8 stage-1 codes
    s1 = dict(order=order.to(torch.int32), off_t=off_t, means16=means16)
    Z, zs, Vr = ei.build_codes(s1, X16, Vp, R=256)
    out.update(Z=Z.numpy(), zs=zs.numpy(), Vr=Vr.numpy())

    # tier table and the module's MSE table
    TS = tiered.allocate(lam, bits)
    out["TS"] = np.array(TS, np.int64)
    out["DIST"] = np.array([tiered.DIST[b] for b in range(9)], np.float64)

    # uniform steps at the lowered sample count, and the uniform-codebook build through encode_uniform
    widths = sorted({bb for _, _, bb in TS})
    orig = s2lut.uniform_cb
    out["uniform_widths"] = np.array(widths, np.int64)
    out["uniform_delta"] = np.array([orig(b, n=N_UNIFORM)[1] for b in widths], np.float64)
    s2lut.uniform_cb = lambda b: orig(b, n=N_UNIFORM)
    cu = s2lut.encode_uniform(dict(TS=TS, V=V), X16, order, c, seed=seed)
    s2lut.uniform_cb = orig
    assert [cu["deltas"][b] for b in widths] == out["uniform_delta"].tolist()
    for t in range(len(TS)):
        out[f"u_planes{t}"] = cu["planes"][t].numpy()
        out[f"rot{t}"] = cu["rots"][t].numpy()
    out["u_scale"], out["u_sig"] = cu["scale"].numpy(), cu["sig"].numpy()

    # Lloyd-Max build (the module's own CB)
    cl = tiered.build(X16, order, c, V, TS, seed=seed)
    for t in range(len(TS)):
        out[f"l_planes{t}"] = cl["planes"][t].numpy()
    out["l_scale"], out["l_sig"] = cl["scale"].numpy(), cl["sig"].numpy()

    path = os.path.join(a.out, "build_reference.npz")
    np.savez_compressed(path, **out)
    print("wrote", path, {k: v.shape for k, v in out.items() if hasattr(v, "shape")})


if __name__ == "__main__":
    main()

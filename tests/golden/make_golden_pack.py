"""Golden packed refinement records from the reference's own `tiered_fused.pack` (`src/tiered_fused.py:112-125`),
applied to the tiered codes stored in the throughput-mode and default-engine golden files.

Usage:  python tests/golden/make_golden_pack.py --ref <checkout of the reference repository> [--out tests/golden]
"""
from __future__ import annotations

import argparse
import importlib
import os
import sys
import types

import numpy as np
import torch

HERE = os.path.dirname(os.path.abspath(__file__))


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--ref", required=True, help="checkout of the reference repository (read only)")
    ap.add_argument("--out", default=HERE)
    args = ap.parse_args()
    sys.path[:0] = [f"{args.ref}/src"]
    sys.modules.setdefault("tiered", types.ModuleType("tiered"))     # only `pack` is used (no codebooks needed)
    tf = importlib.import_module("tiered_fused")
    out = {}
    for tag, name in (("i8_", "i8_reference.npz"), ("tr_", "trellis_reference.npz")):
        f = np.load(os.path.join(HERE, name))
        TS = [tuple(int(v) for v in r) for r in f["TS"]]
        code = dict(TS=TS, planes=[torch.from_numpy(f[f"planes{t}"]) for t in range(len(TS))],
                    scale=torch.from_numpy(f["scale"]), sig=torch.from_numpy(f["sig"]))
        pk = tf.pack(code, pin=False)
        out.update({tag + "rec": pk["rec"].numpy(), tag + "RB": np.asarray(pk["RB"]), tag + "soff": np.asarray(pk["soff"]),
                    tag + "toff": np.asarray(pk["toff"])})
        print(tag, "RB", pk["RB"], "soff", pk["soff"], "toff", pk["toff"])
    path = os.path.join(args.out, "pack_reference.npz")
    np.savez_compressed(path, **out)
    print("wrote", path, os.path.getsize(path), "bytes")


if __name__ == "__main__":
    main()

"""Golden vectors of the routing-free int8 scan (`throughput/brute.py`) from the reference itself.

Runs the reference's real `Brute` class (code build, `qcode`, `scores` on the sample, `search` with the fused
threshold-emit kernel `_scan` MODE=1) on CPU tensors under the Triton interpreter.  The reference's `_scan` needs R a
power of two (`tl.arange(0, R)`), so the goldens use R = 128 and R = 256; the B200 kernel's R = 1536 case is checked
against the oracle restatement pinned here.

Usage:  python tests/golden/make_golden_dense.py --ref <checkout of the reference repository> [--out tests/golden]
"""
from __future__ import annotations

import argparse
import importlib
import os
import sys

os.environ["TRITON_INTERPRET"] = "1"

import numpy as np
import torch

HERE = os.path.dirname(os.path.abspath(__file__))
REPO = os.path.dirname(os.path.dirname(HERE))
sys.path.insert(0, REPO)
sys.path.insert(0, HERE)
synth = importlib.import_module("fanarvse-paper_b200.synth")
from make_golden import Rec  # noqa: E402


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--ref", required=True, help="checkout of the reference repository (read only)")
    ap.add_argument("--out", default=HERE)
    args = ap.parse_args()
    sys.path[:0] = [f"{args.ref}/throughput"]
    brute = importlib.import_module("brute")
    brute.dev = "cpu"
    n, d, nq = 3000, 256, 36
    ds = synth.make_dataset(synth.MixtureSpec(n=n, d=d, comps=10, nq=nq, seed=5), "cpu", gt_k=10)
    X16 = ds["base16"]
    mu = X16[:200000].float().mean(0)
    S = X16[::10].float() - mu
    _, V = torch.linalg.eigh(torch.cov(S.T))
    V = V.flip(1).contiguous()
    f = dict(X16=X16.numpy(), Q=ds["queries"].numpy(), mu=mu.numpy(), V=V.numpy())
    rec = Rec(brute._scan)
    brute._scan = rec
    for tag, R, K, over, M in (("a_", 128, 40, 2.0, None), ("b_", 256, 60, 3.0, 160)):
        b = brute.Brute(X16, mu, V, R=R)
        Qb = ds["queries"]
        q, qs = b.qcode(Qb)
        n0 = len(rec.calls)
        with torch.no_grad():
            pos, est, ok, cnt = b.search(Qb, K, over=over, M=M)
        sample_call, emit_call = rec.calls[n0], rec.calls[n0 + 1]
        sc = sample_call[0][8]                     # dense sample scores [B, n_sample]
        a = emit_call[0]                           # (q, qs, Z, zs, t0, cnt, bval, bpos, out, B, N, CAP)
        Mb = int(a[11])
        cntv = a[5].numpy()
        used = np.minimum(cntv, Mb)
        bval, bpos = a[6].numpy(), a[7].numpy()
        f.update({tag + "params": np.asarray([R, K, Mb], np.int64), tag + "over": np.asarray(over),
                  tag + "Z": b.Z.numpy(), tag + "zs": b.zs.numpy(), tag + "q8": q.numpy(), tag + "qs": qs.numpy(),
                  tag + "sidx": b.sidx.numpy(), tag + "sample_scores": sc.numpy(), tag + "t0": a[4].numpy(),
                  tag + "cnt": cntv, tag + "pos": pos.numpy(), tag + "est": est.numpy(), tag + "ok": ok.numpy(),
                  tag + "emit_q": np.repeat(np.arange(len(cntv)), used).astype(np.int32),
                  tag + "emit_val": np.concatenate([bval[i, :used[i]] for i in range(len(cntv))]).astype(np.float32),
                  tag + "emit_pos": np.concatenate([bpos[i, :used[i]] for i in range(len(cntv))]).astype(np.int32)})
        print(tag, "R", R, "K", K, "M", Mb, "ok", int(ok.sum()), "/", len(ok), "cnt range", int(cntv.min()), int(cntv.max()))
    path = os.path.join(args.out, "dense_reference.npz")
    np.savez_compressed(path, **f)
    print("wrote", path, os.path.getsize(path), "bytes")


if __name__ == "__main__":
    main()

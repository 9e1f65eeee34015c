"""Golden vectors of the default engine's query path (trellis stage 1 + tiered stage 2) from the reference itself.

Runs the reference's real `engine_cell.EngineS._gpu` (batch > 32: `s1cell.search_static` with `_first_compact_s` /
`_emit_loop_s` and the `decode2._decode_tile2` decoder, then `tiered_fused.score`, classification, stage 3; batch <= 8:
`s1small_cell.search_small`; 8 < batch <= 32: `s1small_cell.search_mask`) on CPU tensors under the Triton
interpreter.  Stand-ins: `engine3` (base class Engine8 with the reference's `_score` and a
stage-3 hook calling `stage3_zc._stage3`; `rf.L = 10`), `tiered` (only its codebook table `CB`, filled with this
repository's Lloyd-Max levels since faiss is absent), `civf8`; `tiered_fused._HP` (a host-pointer wrapper for
zero-copy reads of pinned memory) becomes the identity.  The trellis code itself is produced with the
reference's own encoder functions (`trellis.make_table`, `trellis.viterbi`, `trellis_scan.viterbi_paths`,
`trellis_scan.paths_to_words`) following `src/rev_fanardb.py:36-58` and `src/engine_cell.py:8-24`.

Usage:  python tests/golden/make_golden_trellis.py --ref <checkout of the reference repository> [--out tests/golden]
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
from make_golden import Rec  # noqa: E402


def load_reference(ref, CB):
    sys.path[:0] = [f"{ref}/throughput", f"{ref}/src"]
    tiered = types.ModuleType("tiered")
    tiered.CB = CB
    sys.modules["tiered"] = tiered
    sys.modules["civf8"] = types.ModuleType("civf8")
    e3 = types.ModuleType("engine3")
    rf = types.SimpleNamespace(L=10)
    mods = {}

    class Engine8:
        H = None
        H16 = None

        def __init__(self, s1, code):
            self.s1, self.code, self.graphs = s1, code, {}

        def _score(self, Qb, QC, pos):
            return mods["tiered_fused"].score(self.code, Qb, QC, pos)

        def _s3(self, Qb, ids, est, sure, amb):
            score = torch.where(sure, est + 10, torch.full_like(est, -1e9))
            B, KC = ids.shape
            mods["s3"][(KC, B)](Engine8.H16, ids.contiguous(), amb.to(torch.int8).contiguous(),
                                Qb.float().contiguous(), score, KC, D=Qb.shape[1], BD=512)
            return score

    class Engine4:
        pass

    e3.Engine8, e3.Engine4, e3.rf = Engine8, Engine4, rf
    sys.modules["engine3"] = e3
    for m in ("trellis", "trellis_scan", "decode2", "s1cell", "s1small_cell", "tiered_fused", "stage3_zc",
              "engine_cell"):
        mods[m] = importlib.import_module(m)
    for m in ("trellis", "trellis_scan", "s1cell", "s1small_cell", "tiered_fused", "engine_cell"):
        mods[m].dev = "cpu"
    # `tiered_fused` wraps non-CUDA planes in a host-pointer shim for zero-copy reads; on the interpreter the CPU
    # tensor itself is what the kernel must get
    mods["tiered_fused"]._HP = lambda x: x
    mods["s3"] = Rec(mods["stage3_zc"]._stage3)
    mods["Engine8"] = Engine8
    return mods


def trellis_code(mods, X16, s1, W1, L=10, seed=0):
    """stage-1 trellis code of the cell residuals with the reference's encoder (`src/engine_cell.py:8-24`)."""
    tr, ts = mods["trellis"], mods["trellis_scan"]
    R = W1.shape[1]
    Tt = tr.make_table(L)
    g = torch.Generator().manual_seed(seed)
    G = torch.randn(64, R, generator=g)
    best = None
    for a in np.linspace(0.6, 1.3, 15):
        m = float(((G - tr.viterbi(G, Tt, L, 1, float(a))) ** 2).mean())
        if best is None or m < best[0]:
            best = (m, float(a))
    alpha = best[1]
    tab = (alpha * Tt).contiguous()
    off = torch.as_tensor(s1["off"])
    N = len(s1["order"])
    cell = torch.searchsorted(off, torch.arange(N), right=True) - 1
    Rr = X16[s1["order"].long()].float() - s1["means16"].float()[cell]
    Z = Rr @ W1
    nz = Z.norm(dim=1).clamp(min=1e-6)
    Zs = Z / nz[:, None] * R ** 0.5
    path = torch.cat([ts.viterbi_paths(Zs[i:i + 256], Tt, L, alpha) for i in range(0, N, 256)])
    words = ts.paths_to_words(path, L).to(torch.int32)
    Y = tab[path]
    yn = Y.norm(dim=1)
    fip = (Zs * Y).sum(1) / (yn * R ** 0.5)
    scale1 = (nz / (fip * yn)).half()
    return dict(W1=W1, tab=tab, alpha=alpha, words=words, scale1=scale1)


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--ref", required=True, help="checkout of the reference repository (read only)")
    ap.add_argument("--out", default=HERE)
    args = ap.parse_args()
    n, d, nq, nlist, bits = 1536, 256, 40, 32, 640
    ds = synth.make_dataset(synth.MixtureSpec(n=n, d=d, comps=12, nq=nq, seed=1), "cpu", gt_k=10)
    X16 = ds["base16"]
    s1, i8, codes = ib.build_index(X16, nlist, R=256, refine_bits=bits, seed=1, kmeans_sample=n, uniform=False,
                                   lloyd=True)
    code = codes["lloyd"]
    CB = {}
    for b in sorted({bb for _, _, bb in code["TS"]}):
        lv = torch.as_tensor(ib.lloyd_table(b)[0])
        CB[b] = (lv, (lv[1:] + lv[:-1]) / 2)
    mods = load_reference(args.ref, CB)
    # stage-1 rotation W1 = V[:, :R] @ Haar(R) over the first rows' covariance (`src/rev_fanardb.py:37-38`)
    torch.manual_seed(1)
    S = X16[:50000].float()
    c = S.mean(0)
    ev, V = torch.linalg.eigh(torch.cov((S - c).T))
    V = V.flip(1)
    W1 = (V[:, :256] @ torch.linalg.qr(torch.randn(256, 256))[0]).contiguous()
    tc = trellis_code(mods, X16, s1, W1)
    s1t = dict(s1)
    s1t.update(tc)
    s1t["c"] = s1["c"]
    s1t["off_t"] = torch.as_tensor(s1["off"])
    code_ref = {kk: v for kk, v in code.items() if kk not in ("VP", "cbf")}
    recs = {"first": Rec(mods["s1cell"]._first_compact_s), "emit": Rec(mods["s1cell"]._emit_loop_s),
            "score": Rec(mods["tiered_fused"]._tiered_score)}
    mods["s1cell"]._first_compact_s, mods["s1cell"]._emit_loop_s = recs["first"], recs["emit"]
    mods["tiered_fused"]._tiered_score = recs["score"]
    mods["Engine8"].H16 = X16
    E = mods["engine_cell"].EngineS(s1t, code_ref)
    K, z, nprobe, k = 24, 2.0, 12, 10
    Q = ds["queries"]
    with torch.no_grad():
        ok, I, nr, ids = E._gpu(Q, K, z, nprobe, k)
    t = lambda x: x.detach().cpu().numpy() if torch.is_tensor(x) else np.asarray(x)
    f = dict(Q=t(Q), c=t(s1["c"]), off=np.asarray(s1["off"], np.int64), order=t(s1["order"]), means16=t(s1["means16"]),
             inv_mnorm=t(s1["inv_mnorm"]), W1=t(W1), tab=t(tc["tab"]), words=t(tc["words"]), scale1=t(tc["scale1"]),
             H16=t(X16), TS=np.asarray(code["TS"], np.int64), scale=t(code["scale"]), sig=t(code["sig"]),
             params=np.asarray([K, nprobe, k], np.int64), z=np.asarray(z), out_ok=t(ok), out_I=t(I), out_reads=t(nr),
             out_ids=t(ids), QM=t(Q.half() @ s1["means16"].T))
    for ti in range(len(code["TS"])):
        f[f"planes{ti}"] = t(code["planes"][ti])
        f[f"cbf{ti}"] = t(CB[code["TS"][ti][2]][0])
    f["VP"] = t(code_ref["VP"])
    a = recs["first"].calls[0][0]   # (Qh, qid, coff, ccnt, pcell, pblk, ps, pe, words, tab, scale, qcp, bmc, MB)
    f.update(k_Qh=t(a[0]), k_qid1=t(a[1]), k_coff1=t(a[2]), k_ccnt1=t(a[3]), k_qcp1=t(a[11]), k_bmc=t(a[12]),
             k_MB=np.asarray(a[13]))
    a = recs["emit"].calls[0][0]    # (..., qcp, t0, cnt, bval, bpos, CAP)
    cnt, bval, bpos, M = t(a[13]), t(a[14]), t(a[15]), int(a[16])
    used = np.minimum(cnt, M)
    f.update(k_qid=t(a[1]), k_coff=t(a[2]), k_ccnt=t(a[3]), k_qcp=t(a[11]), k_t0=t(a[12]), k_cnt=cnt,
             k_M=np.asarray(M), k_emit_q=np.repeat(np.arange(len(cnt)), used).astype(np.int32),
             k_emit_val=np.concatenate([bval[q, :used[q]] for q in range(len(cnt))]).astype(np.float32),
             k_emit_pos=np.concatenate([bpos[q, :used[q]] for q in range(len(cnt))]).astype(np.int32))
    a = recs["score"].calls[0][0]   # (pos, qc, est, sd, scale, sig, qn2, B, M, N, q0, p0, c0, ...)
    f.update(k_pos=t(a[0]), k_QC=t(a[1]), k_est=t(a[2]), k_sd=t(a[3]), k_qn2=t(a[6]))
    a = mods["s3"].calls[0][0]      # (H, ids, amb, Q, score, KC)
    f.update(k_ids=t(a[1]), k_amb=t(a[2]), k_score=t(a[4]))
    # small batches (`EngineC._gpu`, `src/engine_cell.py:49-60`): B <= 8 takes `search_small` (fp32 dot), 8 < B <= 32
    # `search_mask` (fp16 tensor-core dot), both with an 8192-entry buffer and (beta, rho) = (1.1, 0.75)
    sm = mods["s1small_cell"]
    for tag, rows, kern in (("s6_", slice(0, 6), "_small_scan"), ("m20_", slice(6, 26), "_mask_scan")):
        rec = Rec(getattr(sm, kern))
        setattr(sm, kern, rec)
        mods["s3"].calls.clear()
        Qs = Q[rows].contiguous()
        with torch.no_grad():
            ok, I, nr, ids = E._gpu(Qs, K, z, nprobe, k)
        setattr(sm, kern, rec.kern)
        a0, a1 = rec.calls[0][0], rec.calls[1][0]
        if kern == "_small_scan":   # (q, probe, off, words, tab, scale, qc, t0, cnt, bval, bpos, bm, NPR, NP_USE, CAP, NB)
            bm, t0, cnt, bval, bpos, CAP = a0[11], a1[7], a1[8], a1[9], a1[10], int(a1[14])
            f[tag + "probe"] = t(a1[1])
        else:                       # (q, pm, off, words, tab, scale, qc, t0, cnt, bval, bpos, bm, B, NC, CAP, NB, LEVEL)
            bm, t0, cnt, bval, bpos, CAP = a0[11], a1[7], a1[8], a1[9], a1[10], int(a1[14])
            f[tag + "pm"] = t(a1[1])
        cntv = t(cnt)
        used = np.minimum(cntv, CAP)
        f.update({tag + "Q": t(Qs), tag + "bm": t(bm), tag + "t0": t(t0), tag + "cnt": cntv, tag + "CAP": np.asarray(CAP),
                  tag + "emit_q": np.repeat(np.arange(len(cntv)), used).astype(np.int32),
                  tag + "emit_val": np.concatenate([t(bval)[i, :used[i]] for i in range(len(cntv))]).astype(np.float32),
                  tag + "emit_pos": np.concatenate([t(bpos)[i, :used[i]] for i in range(len(cntv))]).astype(np.int32),
                  tag + "out_ok": t(ok), tag + "out_I": t(I), tag + "out_reads": t(nr), tag + "out_ids": t(ids),
                  tag + "ids": t(mods["s3"].calls[0][0][1]), tag + "score": t(mods["s3"].calls[0][0][4])})
        print(tag, "ok", int(t(ok).sum()), "/", len(Qs), "cnt", cntv.min(), cntv.max())
    path = os.path.join(args.out, "trellis_reference.npz")
    np.savez_compressed(path, **f)
    print("wrote", path, os.path.getsize(path), "bytes; ok", int(t(ok).sum()), "/", len(Q))


if __name__ == "__main__":
    main()

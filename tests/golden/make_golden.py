"""Generate golden vectors from the reference implementation itself (run in the build container, not on the GPU box).

The reference (MohammedMohsen0404/FanarVSE-paper) is Python + Triton.  Its kernels run on CPU tensors under the Triton
interpreter (TRITON_INTERPRET=1), and its throughput-mode orchestration (`throughput/enginei8.py` EngineI8.stage1_i8,
_gpu, _finish, _fallback) runs unchanged once the modules that need faiss, CUDA or the paper's data files are replaced
by stand-ins:
  * `engine_cell`, `engine3`: only the base classes / constants EngineI8 derives from (EngineS, EngineC.SMALL, Engine8)
    and a stage-3 hook that calls the reference's `stage3_zc._stage3` kernel on a CPU tensor;
  * `tiered`: imported by s2lut but only used by `encode_uniform` (index build);
  * `civf8`: CuPy kernels, not used when EngineI8.CUDA is False.
Every kernel launch (`_first8c`, `_emit8c`, `_lut_kernel`, `_score_lut`, `_stage3`) is wrapped to record its arguments
after the launch, so the fixture holds the reference's own intermediate values (pairs, bmc, t0, cnt/bval/bpos, LUT,
est/sd, scores) next to the final (ok, I, reads, ids).

Usage:  python tests/golden/make_golden.py --ref <checkout of the reference repository> [--out tests/golden]
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
synth = importlib.import_module("fanarvse-paper_b200.synth")
ib = importlib.import_module("fanarvse-paper_b200.index_build")


class Rec:
    """Wraps a Triton kernel; records (args, constexprs) after each launch (clones, so outputs are captured)."""

    def __init__(self, kern):
        self.kern, self.calls = kern, []

    def __getitem__(self, grid):
        def launch(*args, **kw):
            self.kern[grid](*args, **kw)
            self.calls.append(([a.clone() if torch.is_tensor(a) else a for a in args], dict(kw), grid))
        return launch


def load_reference(ref):
    sys.path[:0] = [f"{ref}/throughput", f"{ref}/src"]
    ec = types.ModuleType("engine_cell")
    e3 = types.ModuleType("engine3")

    class EngineS:
        def __init__(self, s1, code):
            self.s1, self.code, self.graphs = s1, code, {}

    class EngineC:
        SMALL, TINY = 32, 8

    class Engine8:
        H = None

    class Engine4:
        pass

    ec.EngineS, ec.EngineC, ec.route = EngineS, EngineC, None
    e3.Engine8, e3.Engine4, e3.rf = Engine8, Engine4, None
    sys.modules["engine_cell"] = ec
    sys.modules["engine3"] = e3
    sys.modules["tiered"] = types.ModuleType("tiered")
    sys.modules["civf8"] = types.ModuleType("civf8")
    mods = {m: importlib.import_module(m) for m in ("ivf8c_kern", "s1cell", "s2lut", "stage3_zc", "enginei8")}
    for m in ("s1cell", "s2lut", "enginei8"):
        mods[m].dev = "cpu"
    return mods


def make_index(n, d, comps, nq, nlist, bits, seed=0):
    spec = synth.MixtureSpec(n=n, d=d, comps=comps, nq=nq, seed=seed)
    ds = synth.make_dataset(spec, "cpu", gt_k=10)
    s1, i8, codes = ib.build_index(ds["base16"], nlist, R=256, refine_bits=bits, seed=seed, kmeans_sample=n)
    return ds, s1, i8, codes["uniform"]


def ragged_off(N, NC, seed):
    """cell boundaries with empty cells, 1-row cells, cells straddling and filling 32-row blocks."""
    rng = np.random.default_rng(seed)
    fixed = np.array([0, 1, 31, 33, 64, 0, 97, 2], np.int64)
    w = rng.random(NC - len(fixed)) + 0.05
    rest = np.floor(w / w.sum() * (N - fixed.sum())).astype(np.int64)
    rest[-1] += N - fixed.sum() - rest.sum()
    sizes = np.concatenate([fixed, rest])
    return np.concatenate([[0], np.cumsum(sizes)]).astype(np.int64)


def run_engine(mods, s1, code, i8, H16, Q, K, z, nprobe, k, MSZ, fb_rows=None):
    ei = mods["enginei8"]
    s3k = Rec(mods["stage3_zc"]._stage3)

    def _s3(self, Qb, ids, est, sure, amb):
        score = torch.where(sure, est + 10, torch.full_like(est, -1e9))
        B, KC = ids.shape
        s3k[(KC, B)](H16, ids.contiguous(), amb.to(torch.int8).contiguous(), Qb.float().contiguous(), score, KC,
                     D=Qb.shape[1], BD=512)
        return score

    recs = {"first": Rec(mods["ivf8c_kern"]._first8c), "emit": Rec(mods["ivf8c_kern"]._emit8c),
            "lut": Rec(mods["s2lut"]._lut_kernel), "score": Rec(mods["s2lut"]._score_lut), "s3": s3k}
    ei._first8c, ei._emit8c = recs["first"], recs["emit"]
    mods["s2lut"]._lut_kernel, mods["s2lut"]._score_lut = recs["lut"], recs["score"]
    E = ei.EngineI8(s1, code, i8["Z"], i8["zs"], i8["Vr"])
    type(E)._s3 = _s3
    E.FASTPAIRS = True
    E.ROUTE16 = True
    E.LUTF, E.K2, E.PROJ = True, None, False
    E.RHO, E.MSZ, E.BQ, E.NW, E.NROUTE = 0.6, MSZ, 16, 2, True
    E.DELTA, E.LUTH = 0.07, True
    with torch.no_grad():
        ok, I, nr, ids = E._gpu(Q, K, z, nprobe, k)
        out = dict(ok=ok, I=I, reads=nr, ids=ids, est1=E._est1)
        nmain = {kk: len(r.calls) for kk, r in recs.items()}
        if fb_rows is not None and len(fb_rows):
            fI, fr, fids = E._fallback(Q[fb_rows], K, z, nprobe, k)
            out.update(fb_rows=torch.as_tensor(fb_rows), fb_I=fI, fb_reads=fr, fb_ids=fids)
    return out, recs, nmain, E


def pack_case(prefix, ds_Q, s1, i8, code, H16, out, recs, nmain, E, K, z, nprobe, k, MSZ):
    f = {}
    t = lambda x: x.detach().cpu().numpy() if torch.is_tensor(x) else np.asarray(x)
    f["nq"] = np.asarray(len(ds_Q))
    for key in ("means16", "inv_mnorm"):
        f["s1_" + key] = t(s1[key])
    f["s1_off"] = np.asarray(s1["off"], np.int64)
    f["params"] = np.asarray([K, nprobe, k, MSZ], np.int64)
    f["z"] = np.asarray(z, np.float64)
    f["QM"] = t(ds_Q.half() @ E.meansN.T)
    for key, v in out.items():
        f["out_" + key] = t(v)
    # first-pass launch: (q8, qs, qid, coff, ccnt, pcell, pblk, ps, pe, Z, zs, qcp, bmc, MB)
    a, kw, grid = recs["first"].calls[0]
    for i, name in enumerate(["q8", "qs", "qid1", "coff1", "ccnt1", "pcell", "pblk", "ps", "pe"]):
        f["k_" + name] = t(a[i])
    f["k_qcp1"], f["k_bmc"], f["k_MB"] = t(a[11]), t(a[12]), np.asarray(a[13])
    # emit launch: (..., qcp, t0, cnt, bval, bpos, CAP)
    a, kw, grid = recs["emit"].calls[0]
    f["k_qid"], f["k_coff"], f["k_ccnt"], f["k_qcp"] = t(a[2]), t(a[3]), t(a[4]), t(a[11])
    f["k_t0"], f["k_cnt"], f["k_M"] = t(a[12]), t(a[13]), np.asarray(a[16])
    cnt, bval, bpos = t(a[13]), t(a[14]), t(a[15])
    used = np.minimum(cnt, int(a[16]))
    f["k_emit_q"] = np.repeat(np.arange(len(cnt)), used).astype(np.int32)
    f["k_emit_val"] = np.concatenate([bval[q, :used[q]] for q in range(len(cnt))]).astype(np.float32)
    f["k_emit_pos"] = np.concatenate([bpos[q, :used[q]] for q in range(len(cnt))]).astype(np.int32)
    # LUT build: (Zq, L, D, NNIB)
    a, kw, grid = recs["lut"].calls[0]
    f["k_Zq"], f["k_L"] = t(a[0]), t(a[1])
    # score_lut: (pos, qc, est, sd, L, LW, scale, sig, qsum, qn2, B, M, N, ncnt, ...)
    a, kw, grid = recs["score"].calls[0]
    f["k_pos"], f["k_QC"], f["k_est"], f["k_sd"] = t(a[0]), t(a[1]), t(a[2]), t(a[3])
    f["k_qsum"], f["k_qn2"], f["k_ncnt"] = t(a[8]), t(a[9]), t(a[13])
    # stage 3: (H, ids, amb, Q, score, KC)
    a, kw, grid = recs["s3"].calls[0]
    f["k_ids"], f["k_amb"], f["k_score"] = t(a[1]), t(a[2]), t(a[4])
    return {prefix + kk: v for kk, v in f.items()}


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--ref", required=True, help="checkout of the reference repository (read only)")
    ap.add_argument("--out", default=HERE)
    args = ap.parse_args()
    mods = load_reference(args.ref)
    torch.manual_seed(0)
    fx = {}
    # case A: k-means cells, most queries exact, a few overflow the small emit buffer
    ds, s1, i8, code = make_index(n=1536, d=256, comps=12, nq=48, nlist=32, bits=640, seed=0)
    code = {kk: v for kk, v in code.items() if kk not in ("VP",)}
    H16 = ds["base16"]
    K, z, nprobe, k, MSZ = 16, 1.25, 12, 10, 160
    out, recs, nmain, E = run_engine(mods, s1, code, i8, H16, ds["queries"], K, z, nprobe, k, MSZ, fb_rows=[0, 5, 7])
    fx.update(pack_case("A_", ds["queries"], s1, i8, code, H16, out, recs, nmain, E, K, z, nprobe, k, MSZ))
    t = lambda x: x.detach().cpu().numpy()
    fx.update(Q=t(ds["queries"]), c=t(s1["c"]), order=t(s1["order"]), Z=t(i8["Z"]), zs=t(i8["zs"]), Vr=t(i8["Vr"]),
              H16=t(H16), TS=np.asarray(code["TS"], np.int64), scale=t(code["scale"]), sig=t(code["sig"]),
              VP16=t(code["VP16"]), deltas=np.asarray([code["deltas"][bb] for _, _, bb in code["TS"]], np.float64))
    for ti in range(len(code["TS"])):
        fx[f"planes{ti}"] = t(code["planes"][ti])
    # case B: ragged cells (empty, 1-row, 31/33/64-row cells), same codes, random cell means
    NC = 40
    off = ragged_off(1536, NC, 1)
    g = torch.Generator().manual_seed(5)
    m = torch.nn.functional.normalize(torch.randn(NC, 256, generator=g), dim=1) * 0.3
    s1b = dict(s1)
    s1b.update(off=off, off_t=torch.as_tensor(off), means16=m.half(), inv_mnorm=1.0 / m.half().float().norm(dim=1))
    s1b["cen"] = s1b["inv_mnorm"]
    code_b = {kk: v for kk, v in code.items() if kk not in ("VP", "VP16", "cbf", "NIB")}
    K, nprobe, MSZ = 12, 14, 4096
    out, recs, nmain, E = run_engine(mods, s1b, code_b, i8, H16, ds["queries"][:40], K, 2.0, nprobe, k, MSZ)
    fx.update(pack_case("B_", ds["queries"][:40], s1b, i8, code_b, H16, out, recs, nmain, E, K, 2.0, nprobe, k, MSZ))
    os.makedirs(args.out, exist_ok=True)
    path = os.path.join(args.out, "i8_reference.npz")
    np.savez_compressed(path, **fx)
    print("wrote", path, os.path.getsize(path), "bytes")


if __name__ == "__main__":
    main()

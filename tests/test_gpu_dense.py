"""GPU parity of the routing-free int8 scan (tcgen05 dense contraction, `fvs_dense_scan_tc`) against the reference's
golden vectors (`Brute` under the Triton interpreter, R = 128 and 256) and the oracle (R = 1536, several query blocks,
ragged B and N).  Integer products are exact and the score is two rounded multiplies, so sample scores, thresholds,
counts, emitted sets and stage-1 top-K are compared bit for bit."""
import os

import numpy as np
import pytest
import torch

from conftest import GOLDEN, assert_end_to_end, pkg
from oracle import fvs_oracle as O

pytestmark = pytest.mark.gpu
DEV = "cuda"


def c(x):
    return x.detach().cpu().numpy()


@pytest.fixture(scope="module")
def gd():
    return dict(np.load(os.path.join(GOLDEN, "dense_reference.npz")))


@pytest.fixture(scope="module")
def dm():
    pkg("build").build()
    return pkg("dense")


def _check_emit(cnt, bval, bpos, M, pos_l, est_l):
    for q in range(len(cnt)):
        n = min(int(cnt[q]), M)
        o = np.argsort(bpos[q, :n])
        if cnt[q] <= M:
            np.testing.assert_array_equal(bpos[q, :n][o], pos_l[q])
            np.testing.assert_array_equal(bval[q, :n][o], est_l[q])
        else:
            assert np.isin(bpos[q, :n], pos_l[q]).all()
            assert len(np.unique(bpos[q, :n])) == n


@pytest.mark.parametrize("tag", ["a_", "b_"])
def test_dense_scan_matches_reference_golden(gd, dm, tag):
    f = gd
    R, K, M = (int(v) for v in f[tag + "params"])
    t = lambda a, dt: torch.from_numpy(np.ascontiguousarray(a)).to(DEV, dt)
    D = dm.DenseB200.from_codes(t(f[tag + "Z"], torch.int8), t(f[tag + "zs"], torch.float16), t(f["mu"], torch.float32),
                                t(f["V"], torch.float32))
    q8qs = (t(f[tag + "q8"], torch.int8), t(f[tag + "qs"], torch.float32))
    pos, est, ok, cnt = D.search(None, K, over=float(f[tag + "over"]), M=M, q8qs=q8qs)
    torch.cuda.synchronize()
    D.check_status()
    last = D._last
    np.testing.assert_array_equal(c(last["sample"]), f[tag + "sample_scores"])
    np.testing.assert_array_equal(c(last["t0"]), f[tag + "t0"])
    np.testing.assert_array_equal(c(cnt), f[tag + "cnt"])
    np.testing.assert_array_equal(c(ok), f[tag + "ok"])
    # emitted sets (positions and estimates) of every query whose buffer did not overflow
    eq, ev, ep = f[tag + "emit_q"], f[tag + "emit_val"], f[tag + "emit_pos"]
    bval, bpos = c(last["bval"]), c(last["bpos"])
    for q in range(len(f[tag + "cnt"])):
        n = min(int(f[tag + "cnt"][q]), M)
        sel = eq == q
        if f[tag + "cnt"][q] <= M:
            o1, o2 = np.argsort(ep[sel]), np.argsort(bpos[q, :n])
            np.testing.assert_array_equal(bpos[q, :n][o2], ep[sel][o1])
            np.testing.assert_array_equal(bval[q, :n][o2], ev[sel][o1])
    for q in np.nonzero(f[tag + "ok"])[0]:
        np.testing.assert_array_equal(np.sort(c(pos[q])), np.sort(f[tag + "pos"][q]))
        np.testing.assert_array_equal(np.sort(c(est[q])), np.sort(f[tag + "est"][q]))


def test_dense_qcode_matches_reference(gd, dm):
    f = gd
    t = lambda a, dt: torch.from_numpy(np.ascontiguousarray(a)).to(DEV, dt)
    D = dm.DenseB200.from_codes(t(f["a_Z"], torch.int8), t(f["a_zs"], torch.float16), t(f["mu"], torch.float32),
                                t(f["V"], torch.float32))
    q8, qs = D.qcode(t(f["Q"], torch.float32))
    # the projection is a cuBLAS fp32 GEMM (another summation order than the reference's CPU product): the scale
    # agrees within a few ulp and codes differ at most by one step where a value sits on a rounding boundary
    np.testing.assert_allclose(c(qs), f["a_qs"], rtol=1e-5)
    d = np.abs(c(q8).astype(np.int32) - f["a_q8"].astype(np.int32))
    assert d.max() <= 1 and (d > 0).mean() < 1e-3


@pytest.mark.parametrize("B,N,R", [(300, 20000, 1536), (37, 4999, 1536), (260, 3001, 384)])
def test_dense_scan_matches_oracle(dm, B, N, R):
    g = torch.Generator().manual_seed(B + N + R)
    Z = torch.randint(-127, 128, (N, R), generator=g, dtype=torch.int8)
    zs = (torch.rand(N, generator=g) * 0.01 + 0.001).half()
    q8 = torch.randint(-127, 128, (B, R), generator=g, dtype=torch.int8)
    qs = torch.rand(B, generator=g) * 0.01 + 0.001
    K, over, M = 50, 2.0, 600
    D = dm.DenseB200.from_codes(Z.to(DEV), zs.to(DEV), torch.zeros(R, device=DEV), torch.eye(R, device=DEV))
    pos, est, ok, cnt = D.search(None, K, over=over, M=M, q8qs=(q8.to(DEV), qs.to(DEV)))
    torch.cuda.synchronize()
    D.check_status()
    ref = O.dense_search(q8.numpy(), qs.numpy(), Z.numpy(), zs.numpy(), K, over=over, M=M)
    last = D._last
    np.testing.assert_array_equal(c(last["sample"]), ref["sample"])
    np.testing.assert_array_equal(c(last["t0"]), ref["t0"])
    np.testing.assert_array_equal(c(cnt), ref["cnt"])
    np.testing.assert_array_equal(c(ok), ref["ok"])
    _check_emit(ref["cnt"], c(last["bval"]), c(last["bpos"]), M, ref["pos_l"], ref["est_l"])
    for q in np.nonzero(ref["ok"])[0]:
        np.testing.assert_array_equal(c(pos[q]), ref["pos"][q])       # ties by position: fully ordered
        np.testing.assert_array_equal(c(est[q]), ref["est"][q])


def test_dense_engine_end_to_end(dm):
    synth, ib, eng = pkg("synth"), pkg("index_build"), pkg("engine")
    ds = synth.make_dataset(synth.MixtureSpec(n=40000, d=512, comps=32, nq=200, seed=9), DEV, gt_k=10)
    X16 = ds["base16"]
    s1, i8, codes = ib.build_index(X16, 64, R=256, refine_bits=1280, seed=9, kmeans_sample=40000)
    ix = eng.IndexI8(s1, i8, codes["uniform"], X16, DEV)
    mu = X16.float().mean(0)
    _, V = ib.pca_eigh(X16[::10].float() - mu)
    D = dm.DenseB200(X16[s1["order"].long()].contiguous(), mu, V, R=512)
    E = dm.EngineB200Dense(ix, D)
    E.MSZ = 4096
    Q = ds["queries"]
    K, z, k = 100, 2.0, 10
    I, reads, ids = E.search(Q, K, z, 0, k)
    r = synth.recall(I.long().cpu(), ds["gt"].cpu(), 10)
    assert r >= 0.95, r
    D.check_status()
    # against the oracle on the same inputs: stage 1 (`Brute`) from the product's query codes, then the LUT stage 2,
    # classification, exact re-rank and final top-k of the throughput engine
    e = E.search_eager(Q, K, z, 0, k)
    last = D._last
    q8, qs = c(last["q8"]), c(last["qs"])
    ref = O.dense_search(q8, qs, c(D.Z), c(D.zs), K, over=E.OVER, M=E.MSZ)
    np.testing.assert_array_equal(c(last["t0"]), ref["t0"])
    np.testing.assert_array_equal(c(last["cnt"]), ref["cnt"])
    ok = ref["ok"]
    np.testing.assert_array_equal(c(e["ok"]).astype(bool), ok)
    import __graft_entry__ as ge
    oi = ge.oracle_index(s1, i8, codes["uniform"], X16)
    code = oi["code"]
    TS = code["TS"]
    Zq = c(e["Zq"]).astype(np.float32)         # the fp16 product, taken as its .float()
    QC = c((Q @ ix.c).contiguous())
    Lt = O.lut_build(Zq, half=E.LUTH)
    qsum, qn2 = O.tier_sums(Zq, TS)
    est, sd = O.lut_score(ref["pos"], QC, Lt, TS, code["planes"], code["deltas"], code["scale"], code["sig"], qsum, qn2)
    sure, amb = O.classify(est, sd, z, k)
    oids = np.asarray(oi["order"])[ref["pos"]]
    oI = O.final_topk(oids, O.stage3(oi["H16"], oids, amb, c(Q), est, sure), k)
    np.testing.assert_array_equal(c(e["ids"])[ok], oids[ok])
    np.testing.assert_allclose(c(e["est"])[ok], est[ok], rtol=1e-5, atol=1e-5)
    g = {key: c(e[key]) for key in ("ok", "ids", "reads", "I", "est", "sd")}
    assert_end_to_end(g, dict(ok=ok, ids=oids, reads=amb.sum(1), I=oI, est=est, sd=sd), z, k)


@pytest.mark.parametrize("r", [1, 7, 16, 17, 32, 33, 200])
def test_rth_largest_matches_sort(dm, r):
    lib = pkg("_lib")
    g = torch.Generator().manual_seed(r)
    B, n, ld = 37, 5003, 5010
    v = torch.randn(B, ld, generator=g)
    v[:, ::7] = v[:, 3:4]                       # ties
    v[0, :] = 0.5                               # a row of equal values
    vd = v.to(DEV)
    out = torch.empty(B, device=DEV)
    lib.check(lib.lib().fvs_rth_largest(lib.stream_handle(), lib.ptr(vd), B, n, ld, r, lib.ptr(out)), "rth")
    want = -np.sort(-v[:, :n].numpy(), 1)[:, r - 1]
    np.testing.assert_array_equal(c(out), want)

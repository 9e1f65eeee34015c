"""GPU parity of the throughput-mode path (C ABI kernels) against the reference's golden vectors and the CPU oracle.

Bar: integer / set / index results bit-exact (pairs, block maxima, thresholds, emit counts and sets, stage-1 top-K,
delta counts, LUT entries, candidate ids, final ids on exact queries); fp32 sums whose order differs (tier sums,
LUT-scored estimates, exact dot products) within 1e-5 relative -- tighter than the 1e-3 the task sets for refined
distances."""
import numpy as np
import pytest
import torch

from conftest import assert_end_to_end, golden_index, pkg
from oracle import fvs_oracle as O

pytestmark = pytest.mark.gpu
DEV = "cuda"


def c(x):
    return x.detach().cpu().numpy()


@pytest.fixture(scope="module")
def eng():
    pkg("build").build()
    return pkg("engine")


def _set_scan(E, scan):
    """"cells": the cell-major tcgen05 scan at every batch size (the product path); "tc": the tile-major tcgen05 scan;
    "small": the streaming scan at every batch size; "mma": the mma.sync baseline."""
    E.SCAN = scan if scan in ("mma", "tc", "cells") else "cells"
    E.SMALL = 10 ** 9 if scan == "small" else 0


def _golden_engine(eng, f, case):
    idx = golden_index(f, case)
    code = idx["code"]
    s1 = dict(off=idx["off"], order=idx["order"], c=idx["c"], means16=idx["means16"], inv_mnorm=idx["inv_mnorm"])
    i8 = dict(Z=idx["Z"], zs=idx["zs"], Vr=idx["Vr"])
    ix = eng.IndexI8(s1, i8, dict(code, VP16=f["VP16"]), idx["H16"], DEV)
    E = eng.EngineB200I8(ix)
    K, nprobe, k, M = (int(v) for v in f[case + "params"])
    E.MSZ = M
    return E, ix, idx, K, nprobe, k, M


@pytest.mark.parametrize("scan", ["cells", "tc", "mma"])
@pytest.mark.parametrize("case", ["A_", "B_"])
def test_stage1_matches_reference_golden(golden_i8, eng, case, scan):
    f = golden_i8
    E, ix, idx, K, nprobe, k, M = _golden_engine(eng, f, case)
    E.SCAN = scan
    B = int(f[case + "nq"])
    Q = torch.from_numpy(f["Q"][:B]).to(DEV)
    QMc = torch.from_numpy(f[case + "QM"])
    probe = QMc.topk(nprobe, 1).indices.to(DEV)          # the reference's routing (CPU topk) as input
    q8qs = (torch.from_numpy(f[case + "k_q8"]).to(DEV), torch.from_numpy(f[case + "k_qs"]).to(DEV))
    pos, ok, est1, ncnt = E.stage1_i8(Q, QMc.to(DEV), probe, K, q8qs=q8qs)
    last = E._last
    # block maxima of every (query, first-pass cell) pair at every block of the cell; the product addresses pairs
    # through its slot list, the reference through its stable-sort order
    n1, MB = last["n1"], int(f[case + "k_MB"])
    _, _, _, _, o = O.pairs(c(probe)[:, :n1], len(idx["off"]) - 1, f[case + "QM"])
    ginv = O.pair_slots(o, B, n1)
    gb = f[case + "k_bmc"].reshape(-1, MB)[ginv]
    pb = c(last["bmc"]).reshape(-1, MB)[c(last["slot"])]
    valid = gb > -1e29
    np.testing.assert_array_equal(pb[valid], gb[valid])
    np.testing.assert_array_equal(c(last["t0"]), f[case + "k_t0"])
    cnt = c(last["cnt"])
    np.testing.assert_array_equal(cnt, f[case + "k_cnt"])
    np.testing.assert_array_equal(c(ok), f[case + "out_ok"])
    good = cnt <= M
    np.testing.assert_array_equal(c(est1)[good], f[case + "out_est1"][good])
    np.testing.assert_array_equal(c(pos)[good], f[case + "k_pos"][good])
    np.testing.assert_array_equal(c(ncnt), f[case + "k_ncnt"])
    assert int(E.status) == 0


@pytest.mark.parametrize("case", ["A_", "B_"])
def test_stage2_stage3_match_reference_golden(golden_i8, eng, case):
    f = golden_i8
    E, ix, idx, K, nprobe, k, M = _golden_engine(eng, f, case)
    B = int(f[case + "nq"])
    Q = torch.from_numpy(f["Q"][:B]).to(DEV)
    Zq = torch.from_numpy(f[case + "k_Zq"]).to(DEV)
    Lt, qsum, qn2, _ = E.luts(Q, True, Zq=Zq)
    np.testing.assert_array_equal(c(Lt), f[case + "k_L"])
    np.testing.assert_allclose(c(qsum), f[case + "k_qsum"], rtol=1e-5, atol=1e-6)
    np.testing.assert_allclose(c(qn2), f[case + "k_qn2"], rtol=1e-5, atol=1e-7)
    pos = torch.from_numpy(f[case + "k_pos"]).to(DEV)
    QC = torch.from_numpy(f[case + "k_QC"]).to(DEV)
    ncnt = torch.from_numpy(f[case + "k_ncnt"]).to(DEV)
    gq = (torch.from_numpy(f[case + "k_L"]).to(DEV), torch.from_numpy(f[case + "k_qsum"]).to(DEV),
          torch.from_numpy(f[case + "k_qn2"]).to(DEV))
    est, sd = E.score_lut(QC, pos, gq, ncnt, True)
    np.testing.assert_allclose(c(est), f[case + "k_est"], rtol=1e-5, atol=1e-5)
    np.testing.assert_allclose(c(sd), f[case + "k_sd"], rtol=1e-5, atol=1e-7)
    # the fused path (table built in shared memory from Zq) gives the same estimates
    est2, sd2 = E.score_lut_zq(QC, pos, Zq, ncnt, True)
    np.testing.assert_allclose(c(est2), f[case + "k_est"], rtol=1e-5, atol=1e-5)
    np.testing.assert_allclose(c(sd2), f[case + "k_sd"], rtol=1e-5, atol=1e-7)
    ge, gs = torch.from_numpy(f[case + "k_est"]).to(DEV), torch.from_numpy(f[case + "k_sd"]).to(DEV)
    I, reads, ids, score_k = E.refine(Q, pos, ge, gs, float(f[case + "z"]), k)
    np.testing.assert_array_equal(c(ids), f[case + "k_ids"])
    np.testing.assert_array_equal(c(reads), f[case + "out_reads"])
    np.testing.assert_array_equal(c(I), f[case + "out_I"])
    gsc = f[case + "k_score"]
    want = np.take_along_axis(gsc, np.argsort(-gsc, 1, kind="stable")[:, :k], 1)
    np.testing.assert_allclose(c(score_k), want, rtol=1e-5, atol=1e-5)


def _random_index(eng, n, d, nlist, nq, seed, comps=32):
    synth, ib = pkg("synth"), pkg("index_build")
    ds = synth.make_dataset(synth.MixtureSpec(n=n, d=d, comps=comps, nq=nq, seed=seed), DEV, gt_k=10)
    s1, i8, codes = ib.build_index(ds["base16"], nlist, R=256, seed=seed, kmeans_sample=min(n, 200000))
    ix = eng.IndexI8(s1, i8, codes["uniform"], ds["base16"], DEV)
    import __graft_entry__ as ge
    return ds, ix, ge.oracle_index(s1, i8, codes["uniform"], ds["base16"])


@pytest.mark.parametrize("n,d,nlist,nq,K,nprobe,k,M", [
    (40000, 768, 128, 64, 100, 24, 10, 3072),
    (30000, 1536, 96, 48, 60, 16, 10, 1024),
    (20000, 256, 64, 33, 40, 64, 10, 4096),       # every cell probed
    (20000, 256, 64, 1, 40, 12, 10, 4096),        # batch 1
    (12000, 256, 16, 450, 40, 12, 10, 4096),      # up to 450 queries per cell: cells scanned in several query groups
    (24000, 256, 8, 200, 40, 4, 10, 8192),        # cells of ~3000 rows: the cell-major scan takes each as 3 parts
])
@pytest.mark.parametrize("scan", ["cells", "tc", "small", "mma"])
def test_search_matches_oracle(eng, n, d, nlist, nq, K, nprobe, k, M, scan):
    ds, ix, oi = _random_index(eng, n, d, nlist, nq, seed=7)
    E = eng.EngineB200I8(ix)
    E.MSZ = M
    E.FB_INGRAPH = 0           # the main pass alone (its recompute is checked in test_in_graph_recompute)
    _set_scan(E, scan)
    Q = ds["queries"]
    r = E.search_eager(Q, K, 1.25, nprobe, k)
    QM, probe = E.route(Q, nprobe)

    class Knobs(O.I8Knobs):
        MSZ = M

    o = O.search_i8(oi, c(Q), K, 1.25, nprobe, k, Knobs, QM=c(QM), probe=c(probe), q8qs=(c(r["q8"]), c(r["qs"])),
                    Zq=c(r["Zq"]), fallback=False)
    ok = c(r["ok"])
    np.testing.assert_array_equal(ok, o["ok"])
    np.testing.assert_array_equal(c(r["t0"]), o["t0"])
    np.testing.assert_array_equal(c(r["cnt"]), o["cnt"])
    np.testing.assert_array_equal(c(r["ids"])[ok], o["ids"][ok])
    np.testing.assert_allclose(c(r["est"])[ok], o["est"][ok], rtol=1e-5, atol=1e-5)
    np.testing.assert_allclose(c(r["sd"])[ok], o["sd"][ok], rtol=1e-4, atol=1e-6)
    # classification, exact re-rank and final top-k on the product's own stage-2 output (the fp32 sums above may
    # differ in the last bits, which can move a candidate across the ambiguity boundary)
    sure, amb = O.classify(c(r["est"]), c(r["sd"]), 1.25, k)
    np.testing.assert_array_equal(c(r["reads"])[ok], amb.sum(1)[ok])
    score = O.stage3(oi["H16"], c(r["ids"]), amb, c(Q), c(r["est"]), sure)
    np.testing.assert_array_equal(c(r["I"])[ok], O.final_topk(c(r["ids"]), score, k)[ok])
    # end to end against the oracle's own stage 2: identical final ids wherever the ambiguous sets agree; every other
    # row differs only by candidates within 1e-5 of a classification boundary
    g = {key: c(r[key]) for key in ("ok", "t0", "cnt", "ids", "reads", "I", "est", "sd")}
    assert_end_to_end(g, o, 1.25, k)
    # emitted sets (positions, estimates) equal the oracle's for every query that fit the buffer
    mnorm = (np.float32(1) / oi["inv_mnorm"].astype(np.float32)).astype(np.float32)
    qid, coff, ccnt, qcp, _ = O.pairs(c(probe), len(oi["off"]) - 1, c(QM), mnorm)
    cnt, pos_l, est_l = O.emit(c(r["q8"]), c(r["qs"]), qid, coff, ccnt, oi["off"], oi["Z"], oi["zs"], qcp,
                               c(r["t0"]), len(Q))
    bval, bpos = c(r["bval"]), c(r["bpos"])
    for q in range(len(Q)):
        if cnt[q] <= M:
            o2 = np.argsort(bpos[q, :cnt[q]], kind="stable")
            np.testing.assert_array_equal(bpos[q, :cnt[q]][o2], pos_l[q])
            np.testing.assert_array_equal(bval[q, :cnt[q]][o2], est_l[q])
    assert int(E.status) == 0


def test_search_async_matches_search(eng):
    """search_async: two searches in flight on the two alternating graphs, a third on the first graph again, each
    result equal to search() on the same batch (flagged rows recomputed from the host included); an empty batch"""
    ds, ix, oi = _random_index(eng, 30000, 512, 96, 64, seed=11)
    E = eng.EngineB200I8(ix)
    E.MSZ = 160                      # small emit buffer: flagged rows beyond the graph's capacity, recomputed
    K, z, nprobe, k = 30, 1.5, 20, 10
    Q = ds["queries"]
    Qa, Qb = Q[:40].contiguous(), Q[20:60].contiguous()
    want = [E.search(x, K, z, nprobe, k) for x in (Qa, Qb)]
    h1 = E.search_async(Qa, K, z, nprobe, k)
    h2 = E.search_async(Qb, K, z, nprobe, k)
    r1 = h1.result()
    h3 = E.search_async(Qa, K, z, nprobe, k)
    r2, r3 = h2.result(), h3.result()
    assert h1.result() is r1
    for got, w in ((r1, want[0]), (r2, want[1]), (r3, want[0])):
        for a, b in zip(got, w):
            np.testing.assert_array_equal(c(a), c(b))
    assert E.nbad > 0
    I0, nr0, ids0 = E.search_async(Q[:0], K, z, nprobe, k).result()
    assert I0.shape == (0, k) and nr0.shape == (0,) and ids0.shape == (0, K)


def test_graph_search_and_fallback(eng):
    """search() (CUDA graph + recompute of flagged queries) equals the oracle's EngineI8 search: the main pass on the
    exact queries, `_fallback` (rho 1, M 65536, fp32 LUT, no delta rule) on the flagged ones."""
    ds, ix, oi = _random_index(eng, 30000, 512, 96, 64, seed=11)
    E = eng.EngineB200I8(ix)
    E.MSZ = 160                      # small emit buffer: many queries overflow and are recomputed
    K, z, nprobe, k = 30, 1.5, 20, 10
    Q = ds["queries"]
    I, nr, ids = E.search(Q, K, z, nprobe, k)
    assert E.nbad > 0
    r = E.search_eager(Q, K, z, nprobe, k)
    QM, probe = E.route(Q, nprobe)

    class Knobs(O.I8Knobs):
        MSZ = 160

    o = O.search_i8(oi, c(Q), K, z, nprobe, k, Knobs, QM=c(QM), probe=c(probe), q8qs=(c(r["q8"]), c(r["qs"])),
                    Zq=c(r["Zq"]), fallback=False)
    ok = o["ok"]
    np.testing.assert_array_equal(c(r["ok"]), ok)
    # the graph's rows (the main pass on the exact queries) against the oracle: identical final ids wherever the
    # ambiguous sets agree, other rows only by candidates within 1e-5 of a classification boundary
    g = dict(ok=c(r["ok"]), t0=c(r["t0"]), cnt=c(r["cnt"]), ids=c(ids), reads=c(nr), I=c(I), est=c(r["est"]),
             sd=c(r["sd"]))
    assert_end_to_end(g, o, z, k)
    bad = np.nonzero(~ok)[0]
    Qb = Q[torch.from_numpy(bad).to(DEV)]
    QMb, probeb = E.route(Qb, nprobe)
    q8b, qsb = E.quantize(Qb)
    Zqb = (Qb.half() @ ix.VP16).float()
    fb = O._search_i8_core(oi, c(Qb), K, z, nprobe, k, Knobs, c(QMb), c(probeb), (c(q8b), c(qsb)), c(Zqb),
                           rho_override=1.0)
    np.testing.assert_array_equal(c(ids)[bad], fb["ids"])          # stage-1 candidates of the recompute: exact
    # the recompute's stage 2 on the GPU (same calls as `_fallback`) for the boundary check of its rows
    QCb = (Qb @ ix.c).contiguous()
    posb, okb, _, _ = E.stage1_i8(Qb, QMb, probeb, K, rho_override=1.0, M_override=65536, q8qs=(q8b, qsb))
    estb, sdb = E.score_lut_zq(QCb, posb, Zqb.contiguous(), None, False)
    gb = dict(ok=c(okb), ids=c(ids)[bad], reads=c(nr)[bad], I=c(I)[bad], est=c(estb), sd=c(sdb))
    assert_end_to_end(gb, dict(fb, ok=np.ones(len(bad), bool)), z, k)
    # replay with the same inputs is deterministic
    I2, nr2, ids2 = E.search(Q, K, z, nprobe, k)
    np.testing.assert_array_equal(c(I2), c(I))


@pytest.mark.parametrize("M,K,kind,B", [(700, 50, "ties", 7), (701, 50, "ties", 7), (4000, 100, "ties", 7),
                                         (4000, 100, "cont", 7), (8192, 100, "cont", 7), (8192, 100, "ties", 7),
                                         (8196, 100, "cont", 7), (16384, 100, "cont", 7), (16384, 250, "ties", 7),
                                         (4000, 400, "ties", 7), (16384, 500, "cont", 7), (1400, 600, "ties", 7),
                                         (4000, 100, "flat", 7), (700, 50, "cont", 300), (4000, 100, "ties", 300),
                                         (8192, 100, "cont", 300), (8192, 100, "ties", 300), (8192, 128, "cont", 300),
                                         (4000, 100, "flat", 300), (8192, 100, "flat", 300), (2048, 129, "ties", 300)])
def test_select_topk_ties(eng, M, K, kind, B):
    """stage-1 top-K orders by (estimate desc, position asc), also through ties and cnt < K, cnt > M; register-resident
    kernel (M a multiple of 4, K <= 512; more than 8192 candidates by its global-memory branch; K <= 128 by the
    bound-and-rank selection, which falls back to histogram passes when more than 1024 candidates reach its bound, as
    with equal scores) at 1024 threads per query (B below the SM count) and 256 (B = 300), and shared-memory kernel
    (the other shapes)."""
    L = pkg("_lib")
    lib = L.lib()
    rng = np.random.default_rng(0)
    if kind == "ties":
        vals = rng.integers(-20, 20, (B, M)).astype(np.float32) / 4  # many ties
    elif kind == "flat":
        vals = np.full((B, M), 1.5, np.float32)                     # every score equal
    else:
        vals = (rng.standard_normal((B, M)) * 3).astype(np.float32)
    posv = np.stack([rng.permutation(100000)[:M] for _ in range(B)]).astype(np.int32)
    cnt = np.resize(np.array([0, 10, K - 1, K, K + 1, M, M + 200, M // 2, M // 3 + 1, 3 * K], np.int32), B)
    tv, tp, tc = (torch.from_numpy(x).to(DEV) for x in (vals, posv, cnt))
    pos = torch.empty(B, K, dtype=torch.int64, device=DEV)
    est = torch.empty(B, K, device=DEV)
    ok = torch.empty(B, dtype=torch.uint8, device=DEV)
    nc = torch.empty(B, dtype=torch.int32, device=DEV)
    L.check(lib.fvs_select_topk(L.stream_handle(), L.ptr(tv), L.ptr(tp), L.ptr(tc), B, M, K, L.ptr(pos), L.ptr(est),
                                L.ptr(ok), L.ptr(nc), 0.3, 9), "select")
    n = np.minimum(cnt, M)
    pl = [posv[q, :n[q]].astype(np.int64) for q in range(B)]
    el = [vals[q, :n[q]] for q in range(B)]
    op, oe, ook = O.select_topk(pl, el, cnt, K, M)
    np.testing.assert_array_equal(c(pos), op)
    np.testing.assert_array_equal(c(est), oe)
    np.testing.assert_array_equal(c(ok).astype(bool), ook)
    np.testing.assert_array_equal(c(nc), O.delta_count(oe, 0.3))


def test_merge_topk(eng):
    L = pkg("_lib")
    lib = L.lib()
    rng = np.random.default_rng(1)
    G, B, kin, k = 4, 9, 10, 10
    ids = rng.permutation(10 ** 6)[:G * B * kin].reshape(G, B, kin).astype(np.int64)
    sc = (rng.integers(0, 30, (G, B, kin)) / 8).astype(np.float32)
    ti, ts = torch.from_numpy(ids).to(DEV), torch.from_numpy(sc).to(DEV)
    I = torch.empty(B, k, dtype=torch.int64, device=DEV)
    S = torch.empty(B, k, device=DEV)
    L.check(lib.fvs_merge_topk(L.stream_handle(), L.ptr(ti), L.ptr(ts), G, B, kin, k, L.ptr(I), L.ptr(S)), "merge")
    oi, os_ = O.merge_topk(ids, sc, k)
    np.testing.assert_array_equal(c(I), oi)
    np.testing.assert_array_equal(c(S), os_)


@pytest.mark.parametrize("G,kin,k", [(4, 10, 10), (8, 100, 100), (16, 100, 10)])
def test_merge_topk_wide_ids(eng, G, kin, k):
    """global ids at and above 2^32 and -1 ("no result") entries come back unchanged, in (score desc, id asc) order,
    also through equal scores whose ids differ only above bit 31; rank-placement (G*kin <= 1024) and sorting-network
    (larger) kernels"""
    L = pkg("_lib")
    lib = L.lib()
    rng = np.random.default_rng(G * kin)
    B = 5
    ids = (rng.permutation(10 ** 6)[:G * B * kin].astype(np.int64) + (rng.integers(0, 4, G * B * kin) << 32))
    ids = ids.reshape(G, B, kin)
    ids[0, 1, :] = ids[0, 1, 0] % (1 << 32) + (np.arange(kin, dtype=np.int64) << 32)   # equal low words
    sc = (rng.integers(0, 6, (G, B, kin)) / 4).astype(np.float32)                      # many ties
    ids[:, 2, kin // 2:] = -1
    sc[:, 2, kin // 2:] = -1e30
    ids[:, 3, :] = -1
    sc[:, 3, :] = -1e30
    ti, ts = torch.from_numpy(ids).to(DEV), torch.from_numpy(sc).to(DEV)
    I = torch.empty(B, k, dtype=torch.int64, device=DEV)
    S = torch.empty(B, k, device=DEV)
    L.check(lib.fvs_merge_topk(L.stream_handle(), L.ptr(ti), L.ptr(ts), G, B, kin, k, L.ptr(I), L.ptr(S)), "merge")
    oi, os_ = O.merge_topk(ids, sc, k)
    np.testing.assert_array_equal(c(I), oi)
    np.testing.assert_array_equal(c(S), os_)
    assert (c(I)[3] == -1).all()


@pytest.mark.parametrize("NC,npr", [(4096, 352), (4093, 352), (4096, 600), (16384, 96), (8, 3), (2000, 1)])
def test_route_topk_ties(eng, NC, npr):
    """top-n_p cells by (fp16 score desc, cell asc), also through many equal scores; register-resident kernel
    (NC a multiple of 8 up to 16384, n_p <= 512) and shared-memory kernel (the other shapes)."""
    L = pkg("_lib")
    lib = L.lib()
    rng = np.random.default_rng(3)
    B = 37
    QM = (rng.integers(-200, 200, (B, NC)) / 256).astype(np.float16)     # heavy ties
    tq = torch.from_numpy(QM).to(DEV)
    probe = torch.empty(B, npr, dtype=torch.int64, device=DEV)
    L.check(lib.fvs_route_topk(L.stream_handle(), L.ptr(tq), B, NC, npr, L.ptr(probe)), "route")
    want = np.stack([O.topk_desc(QM[q].astype(np.float32), npr) for q in range(B)])
    np.testing.assert_array_equal(c(probe), want)


@pytest.mark.parametrize("ncols", [1, 23, 352])
def test_pairs_csr(eng, ncols):
    """pair lists: per-cell query sets, pair constants and slots agree with the stable-sort restatement."""
    L = pkg("_lib")
    lib = L.lib()
    rng = np.random.default_rng(4)
    B, NC, npr = 300, 4096, 352
    probe = np.stack([rng.permutation(NC)[:npr] for _ in range(B)]).astype(np.int64)
    QM = (rng.standard_normal((B, NC)) * 0.3).astype(np.float16)
    mnorm = (rng.random(NC) + 0.5).astype(np.float32)
    tp, tq, tm = (torch.from_numpy(x).to(DEV) for x in (probe, QM, mnorm))
    n = B * ncols
    qid = torch.empty(n, dtype=torch.int32, device=DEV)
    qcp = torch.empty(n, device=DEV)
    coff = torch.empty(NC, dtype=torch.int32, device=DEV)
    ccnt = torch.empty(NC, dtype=torch.int32, device=DEV)
    slot = torch.empty(n, dtype=torch.int32, device=DEV)
    work = torch.empty(NC, dtype=torch.int32, device=DEV)
    L.check(lib.fvs_pairs(L.stream_handle(), L.ptr(tp), B, npr, ncols, NC, L.ptr(tq), L.ptr(tm), L.ptr(qid),
                          L.ptr(coff), L.ptr(ccnt), L.ptr(qcp), L.ptr(slot), L.ptr(work)), "pairs")
    oq, oc, on, oqc, o = O.pairs(probe[:, :ncols], NC, QM, mnorm)
    np.testing.assert_array_equal(c(coff), oc)
    np.testing.assert_array_equal(c(ccnt), on)
    gq, gqc, gs = c(qid), c(qcp), c(slot)
    for cc in range(NC):
        a, b = oc[cc], oc[cc] + on[cc]
        np.testing.assert_array_equal(np.sort(gq[a:b]), np.sort(oq[a:b]))
    # slot[q*ncols + j] is where pair (q, j) landed: its query and constant are the pair's
    qq = np.repeat(np.arange(B), ncols)
    jj = np.tile(np.arange(ncols), B)
    np.testing.assert_array_equal(gq[gs], qq)
    want = (QM[qq, probe[qq, jj]].astype(np.float32) * mnorm[probe[qq, jj]]).astype(np.float32)
    np.testing.assert_array_equal(gqc[gs], want)


@pytest.mark.parametrize("n1", [1, 23, 352])
def test_pairs_split(eng, n1):
    """one pair list for both passes: in every cell the pairs from the first n1 columns come first and form the first
    pass's list (coff, ccnt1), the whole range the emit pass's list (coff, ccnt); slots point at the first-pass pairs."""
    L = pkg("_lib")
    lib = L.lib()
    rng = np.random.default_rng(6)
    B, NC, npr = 300, 4096, 352
    probe = np.stack([rng.permutation(NC)[:npr] for _ in range(B)]).astype(np.int64)
    QM = (rng.standard_normal((B, NC)) * 0.3).astype(np.float16)
    mnorm = (rng.random(NC) + 0.5).astype(np.float32)
    tp, tq, tm = (torch.from_numpy(x).to(DEV) for x in (probe, QM, mnorm))
    n = B * npr
    qid = torch.empty(n, dtype=torch.int32, device=DEV)
    qcp = torch.empty(n, device=DEV)
    coff, ccnt, ccnt1 = (torch.empty(NC, dtype=torch.int32, device=DEV) for _ in range(3))
    slot = torch.empty(B * n1, dtype=torch.int32, device=DEV)
    work = torch.empty(2 * NC, dtype=torch.int32, device=DEV)
    L.check(lib.fvs_pairs_split(L.stream_handle(), L.ptr(tp), B, npr, n1, NC, L.ptr(tq), L.ptr(tm), L.ptr(qid),
                                L.ptr(coff), L.ptr(ccnt), L.ptr(ccnt1), L.ptr(qcp), L.ptr(slot), L.ptr(work)),
            "pairs_split")
    oq, oc, on, oqc, o = O.pairs(probe, NC, QM, mnorm)
    oq1, oc1, on1, _, _ = O.pairs(probe[:, :n1], NC, QM, mnorm)
    np.testing.assert_array_equal(c(coff), oc)
    np.testing.assert_array_equal(c(ccnt), on)
    np.testing.assert_array_equal(c(ccnt1), on1)
    gq, gqc, gs = c(qid), c(qcp), c(slot)
    for cc in range(0, NC, 7):
        a, m, b = oc[cc], oc[cc] + on1[cc], oc[cc] + on[cc]
        np.testing.assert_array_equal(np.sort(gq[a:m]), np.sort(oq1[oc1[cc]:oc1[cc] + on1[cc]]))
        np.testing.assert_array_equal(np.sort(gq[a:b]), np.sort(oq[a:b]))
    qq = np.repeat(np.arange(B), n1)
    jj = np.tile(np.arange(n1), B)
    np.testing.assert_array_equal(gq[gs], qq)
    cells = probe[qq, jj]
    assert ((gs >= oc[cells]) & (gs < oc[cells] + on1[cells])).all()
    want = (QM[qq, cells].astype(np.float32) * mnorm[cells]).astype(np.float32)
    np.testing.assert_array_equal(gqc[gs], want)


@pytest.mark.parametrize("B,NC,npr,n1,scaled", [(300, 4096, 72, 13, 0), (37, 8192, 256, 30, 0),
                                                 (1000, 16384, 512, 1, 0), (64, 8, 8, 8, 0), (513, 4096, 352, 23, 0),
                                                 (200, 2048, 128, 64, 0), (300, 8192, 256, 40, 1),
                                                 (300, 8192, 256, 40, 2), (37, 4096, 72, 13, 1),
                                                 (1000, 16384, 512, 1, 2), (64, 8, 8, 8, 1), (200, 2048, 400, 64, 2)])
def test_route_pairs_matches_separate_kernels(eng, B, NC, npr, n1, scaled):
    """fvs_route_pairs (routing selection + both pair lists + cell lists in two launches) gives the probe list of
    fvs_route_topk, the pair layout of fvs_pairs_split and the lists of fvs_cell_lists, also through tied scores; its
    cursors are left zero, so a second call on the same work buffer gives the same result.  fvs_route_pairs_scaled
    (scaled = 1: pair constants with the norm factor, 2: without, as the default engine) gives the probe list of
    fvs_route_topk_scaled, also through scores tied after the scaling.  The order is given as cell-part entries
    (cell | part << 16, some cells in two or three parts): the lists hold the entries whose cells have pairs."""
    L = pkg("_lib")
    lib = L.lib()
    rng = np.random.default_rng(B + NC)
    QM = (rng.integers(-300, 300, (B, NC)) / 512).astype(np.float16)        # many ties
    mnorm = (rng.random(NC) + 0.5).astype(np.float32)
    if scaled == 2:
        mnorm = np.ones(NC, np.float32)           # no norm factor: the kernel's constant float(QM) equals QM * 1
    sc = np.where(rng.random(NC) < 0.5, 1.0, rng.random(NC) + 0.5).astype(np.float32)   # many equal scales
    order = np.argsort(-rng.integers(0, 50, NC), kind="stable").astype(np.int32)
    nparts = np.where(rng.random(NC) < 0.2, rng.integers(2, 4, NC), 1)
    within = np.arange(int(nparts.sum())) - np.repeat(np.cumsum(nparts) - nparts, nparts)
    oe = (np.repeat(order, nparts) | (within << 16)).astype(np.int32)   # cell-part entries
    NP = len(oe)
    tq, tm, to, tsc = (torch.from_numpy(x).to(DEV) for x in (QM, mnorm, oe, sc))
    mptr = None if scaled == 2 else L.ptr(tm)
    work = torch.zeros(2 * NC + 1, dtype=torch.int32, device=DEV)
    outs = []
    for _ in range(2):
        probe = torch.empty(B, npr, dtype=torch.int64, device=DEV)
        qid = torch.empty(B * npr, dtype=torch.int32, device=DEV)
        qcp = torch.empty(B * npr, device=DEV)
        coff, ccnt, ccnt1 = (torch.empty(NC, dtype=torch.int32, device=DEV) for _ in range(3))
        l1, l2 = (torch.empty(NP, dtype=torch.int32, device=DEV) for _ in range(2))
        slot = torch.empty(B * n1, dtype=torch.int32, device=DEV)
        nl = torch.empty(2, dtype=torch.int32, device=DEV)
        zero = torch.ones(B, dtype=torch.int32, device=DEV)
        tail = (L.ptr(to), NP, L.ptr(probe), L.ptr(qid), L.ptr(qcp), L.ptr(coff), L.ptr(ccnt), L.ptr(ccnt1), L.ptr(slot),
                L.ptr(l1), L.ptr(l2), L.ptr(nl), L.ptr(zero), B, L.ptr(work))
        if scaled:
            L.check(lib.fvs_route_pairs_scaled(L.stream_handle(), L.ptr(tq), B, NC, npr, n1, L.ptr(tsc), mptr, *tail),
                    "route_pairs_scaled")
        else:
            L.check(lib.fvs_route_pairs(L.stream_handle(), L.ptr(tq), B, NC, npr, n1, L.ptr(tm), *tail), "route_pairs")
        torch.cuda.synchronize()
        assert int(work.abs().sum()) == 0 and int(zero.abs().sum()) == 0
        outs.append([c(x) for x in (probe, qid, qcp, coff, ccnt, ccnt1, slot, l1, l2, nl)])
    for i in (0, 3, 4, 5, 9):                            # everything but the within-cell order of the pairs
        np.testing.assert_array_equal(outs[0][i], outs[1][i])
    for i, j in ((7, 0), (8, 1)):                        # the lists up to their lengths
        np.testing.assert_array_equal(outs[0][i][:outs[0][9][j]], outs[1][i][:outs[1][9][j]])
    probe, qid, qcp, coff, ccnt, ccnt1, slot, l1, l2, nl = outs[0]
    # routing: the separate kernel's probe list
    p2 = torch.empty(B, npr, dtype=torch.int64, device=DEV)
    if scaled:
        L.check(lib.fvs_route_topk_scaled(L.stream_handle(), L.ptr(tq), B, NC, npr, L.ptr(tsc), L.ptr(p2)), "route")
    else:
        L.check(lib.fvs_route_topk(L.stream_handle(), L.ptr(tq), B, NC, npr, L.ptr(p2)), "route")
    np.testing.assert_array_equal(probe, c(p2))
    # pairs: counts and offsets exact, each cell's first-pass and other segments equal as sets, slots and constants
    oq, oc, on, _, _ = O.pairs(probe, NC, QM, mnorm)
    oq1, oc1, on1, _, _ = O.pairs(probe[:, :n1], NC, QM, mnorm)
    np.testing.assert_array_equal(coff, oc)
    np.testing.assert_array_equal(ccnt, on)
    np.testing.assert_array_equal(ccnt1, on1)
    for cc in range(0, NC, max(1, NC // 500)):
        a, m, e = oc[cc], oc[cc] + on1[cc], oc[cc] + on[cc]
        np.testing.assert_array_equal(np.sort(qid[a:m]), np.sort(oq1[oc1[cc]:oc1[cc] + on1[cc]]))
        np.testing.assert_array_equal(np.sort(qid[a:e]), np.sort(oq[a:e]))
    qq = np.repeat(np.arange(B), n1)
    jj = np.tile(np.arange(n1), B)
    np.testing.assert_array_equal(qid[slot], qq)
    cells = probe[qq, jj]
    assert ((slot >= oc[cells]) & (slot < oc[cells] + on1[cells])).all()
    qa = np.repeat(np.arange(B), npr)
    pc = probe.ravel()
    want = (QM[qa, pc].astype(np.float32) * mnorm[pc]).astype(np.float32)
    got = np.zeros(B * npr, np.float32)
    # the constant of every pair sits at the pair's position: match by (query, cell) through the slots' layout
    pos_of = {}
    for cc in range(NC):
        for pos in range(oc[cc], oc[cc] + on[cc]):
            pos_of[(int(qid[pos]), cc)] = pos
    got = np.array([qcp[pos_of[(int(q), int(cc))]] for q, cc in zip(qa, pc)], np.float32)
    np.testing.assert_array_equal(got, want)
    # cell lists: the cells of `order` with pairs
    cells = oe & 0xffff
    np.testing.assert_array_equal(nl, [int((on1[cells] > 0).sum()), int((on[cells] > 0).sum())])
    np.testing.assert_array_equal(l1[:nl[0]], oe[on1[cells] > 0])
    np.testing.assert_array_equal(l2[:nl[1]], oe[on[cells] > 0])


def test_quantize_matches_reference_formula(eng):
    """the quantisation kernel equals the reference's torch expression on the same projected queries."""
    L = pkg("_lib")
    lib = L.lib()
    g = torch.Generator(device=DEV).manual_seed(5)
    z = torch.randn(257, 256, device=DEV, generator=g) * 0.05
    z[3] = 0
    z[7, 5] = 3.0
    qs_ref = z.abs().amax(1).clamp(min=1e-12) / 127
    q8_ref = torch.round(z / qs_ref[:, None]).clamp(-127, 127).to(torch.int8)
    q8 = torch.empty_like(q8_ref)
    qs = torch.empty_like(qs_ref)
    L.check(lib.fvs_quantize(L.stream_handle(), L.ptr(z), 257, 256, 256, L.ptr(q8), L.ptr(qs)), "quantize")
    np.testing.assert_array_equal(c(qs), c(qs_ref))
    np.testing.assert_array_equal(c(q8), c(q8_ref))


@pytest.mark.parametrize("B,d,ldq", [(2000, 1536, 1536), (1, 1536, 1536), (257, 768, 768), (33, 1000, 1004),
                                    (130, 256, 256)])
def test_project_quantize_fp32_accuracy(eng, B, d, ldq):
    """fvs_project_quantize (3xTF32 products on the tensor cores, split over K): z within a few 1e-6 relative of the
    float64 product (the tensor cores' fp32 accumulation over up to ~200 K-steps per split is the larger term; a SIMT
    fp32 GEMM is near 1e-7), so qs agrees to 5e-6 relative and q8 equals the reference's quantisation of the exact z
    except where z / qs lies within 1e-3 of a rounding boundary (well under 0.1 % of the codes)."""
    L = pkg("_lib")
    lib = L.lib()
    g = torch.Generator(device=DEV).manual_seed(B + d)
    Qfull = torch.randn(B, ldq, device=DEV, generator=g)
    Q = Qfull[:, :d]
    Vr = torch.randn(d, 256, device=DEV, generator=g) / d ** 0.5
    Vr[:, 7] *= 1e-3                                          # a column of small values
    VrT = Vr.t().contiguous()
    big = ((VrT.view(torch.int32) + 0x1000) & ~0x1FFF).view(torch.float32).contiguous()
    small = (VrT - big).contiguous()
    q8 = torch.empty(B, 256, dtype=torch.int8, device=DEV)
    qs = torch.empty(B, device=DEV)
    part = torch.empty(16 * B * 256, device=DEV)
    status = torch.zeros(1, dtype=torch.int32, device=DEV)
    L.check(lib.fvs_project_quantize(L.stream_handle(), L.ptr(Qfull), B, d, ldq, L.ptr(big), L.ptr(small), 256,
                                     L.ptr(q8), L.ptr(qs), L.ptr(part), 16, L.ptr(status)), "project_quantize")
    torch.cuda.synchronize()
    assert int(status) == 0
    z64 = Q.double() @ Vr.double()
    qs64 = z64.abs().amax(1).clamp(min=1e-12) / 127
    np.testing.assert_allclose(c(qs).astype(np.float64), c(qs64), rtol=5e-6)
    x = c(z64 / qs64[:, None])
    want = np.clip(np.round(x), -127, 127)
    near_tie = np.abs(np.abs(x - np.floor(x)) - 0.5) < 1e-3
    got = c(q8).astype(np.float64)
    assert np.all((got == want) | near_tie)
    assert near_tie.mean() < 5e-3


@pytest.mark.parametrize("B,d,ldq", [(1, 1536, 1536), (257, 768, 768), (33, 1536, 1600)])
def test_query_prep_matches_torch(eng, B, d, ldq):
    """fvs_query_prep: the fp16 copy equals `Qb.half()` bit for bit; the centre product equals `Qb @ c` within fp32
    summation-order rounding."""
    L = pkg("_lib")
    lib = L.lib()
    g = torch.Generator(device=DEV).manual_seed(B)
    Qfull = torch.randn(B, ldq, device=DEV, generator=g)
    Qfull[0, :8] = torch.tensor([1e-8, -1e-8, 65504.0, 70000.0, -3.5, 0.0, -0.0, 2.0 ** -24], device=DEV)
    Q = Qfull[:, :d]
    cvec = torch.randn(d, device=DEV, generator=g)
    Qh = torch.empty(B, d, dtype=torch.float16, device=DEV)
    qc = torch.empty(B, device=DEV)
    L.check(lib.fvs_query_prep(L.stream_handle(), L.ptr(Qfull), B, d, ldq, L.ptr(cvec), L.ptr(Qh), L.ptr(qc)),
            "query_prep")
    np.testing.assert_array_equal(c(Qh.view(torch.int16)), c(Q.half().view(torch.int16)))
    ref = (Q.double() @ cvec.double()).float()
    scale = (Q.abs().double() @ cvec.abs().double()).float()
    assert ((qc - ref).abs() <= 1e-5 * scale + 1e-30).all()
    assert lib.fvs_query_prep(L.stream_handle(), L.ptr(Qfull), B, d + 2, ldq, L.ptr(cvec), L.ptr(Qh),
                              L.ptr(qc)) == -1                     # d not a multiple of 4


def test_search_host_matches_search(eng):
    """latency mode (ids copied to pinned host memory inside the graph) returns the device search's ids"""
    synth, ib = pkg("synth"), pkg("index_build")
    ds = synth.make_dataset(synth.MixtureSpec(n=20000, d=256, comps=16, nq=40, seed=3), DEV, gt_k=10)
    s1, i8, codes = ib.build_index(ds["base16"], 48, R=256, refine_bits=640, seed=3, kmeans_sample=20000)
    ix = eng.IndexI8(s1, i8, codes["uniform"], ds["base16"], DEV)
    E = eng.EngineB200I8(ix)
    E.MSZ = 600                                          # small buffer: some rows take the recompute path
    Q = ds["queries"]
    for B in (1, 5, 40):
        I, _, _ = E.search(Q[:B].contiguous(), 40, 1.5, 12, 10)
        h = E.search_host(Q[:B].contiguous(), 40, 1.5, 12, 10)
        np.testing.assert_array_equal(h, c(I))


@pytest.mark.parametrize("msz", [600, 160])
def test_in_graph_recompute(eng, msz):
    """batches of FB_MIN_BATCH rows or more recompute up to FB_INGRAPH flagged rows inside their own graph (from the
    main pass's routing and query codes), the rest on the host: the flagged rows equal the oracle's `_fallback` on the
    same inputs, the other rows the main pass; the ids of the recompute are exact."""
    ds, ix, oi = _random_index(eng, 30000, 512, 96, 320, seed=13)
    E = eng.EngineB200I8(ix)
    E.MSZ = msz                      # 600: a few flagged rows (all in the graph); 160: more than FB_INGRAPH
    K, z, nprobe, k = 30, 1.5, 20, 10
    Q = ds["queries"]
    assert len(Q) >= E.FB_MIN_BATCH
    I, nr, ids = E.search(Q, K, z, nprobe, k)
    r = E.search_eager(Q, K, z, nprobe, k)
    QM, probe = E.route(Q, nprobe)
    q8, qs = E.quantize(Q)

    class Knobs(O.I8Knobs):
        MSZ = msz

    o = O.search_i8(oi, c(Q), K, z, nprobe, k, Knobs, QM=c(QM), probe=c(probe), q8qs=(c(q8), c(qs)),
                    Zq=c(E.rotated_query(Q)), fallback=False)
    ok = o["ok"]
    nbad = int((~ok).sum())
    assert nbad > 0 and E.nbad >= nbad
    if msz == 160:
        assert nbad > E.FB_INGRAPH               # some rows take the host path
    g = dict(ok=c(r["ok"]), t0=c(r["t0"]), cnt=c(r["cnt"]), ids=c(ids), reads=c(nr), I=c(I), est=c(r["est"]),
             sd=c(r["sd"]))
    assert_end_to_end(g, o, z, k)
    bad = np.nonzero(~ok)[0]
    Zq = E.rotated_query(Q)
    fb = O._search_i8_core(oi, c(Q)[bad], K, z, nprobe, k, Knobs, c(QM)[bad], c(probe)[bad], (c(q8)[bad], c(qs)[bad]),
                           c(Zq)[bad], rho_override=1.0)
    in_graph = bad[:E.FB_INGRAPH]
    n = len(in_graph)
    np.testing.assert_array_equal(c(ids)[in_graph], fb["ids"][:n])
    # the recompute's stage 2 on the GPU (the calls of the in-graph recompute) for the boundary check of its rows
    bi = torch.from_numpy(in_graph).to(DEV)
    posb, okb, _, _ = E.stage1_i8(Q[bi], QM[bi], probe[bi].contiguous(), K, rho_override=1.0, M_override=65536,
                                  q8qs=(q8[bi], qs[bi]), small=True)
    QC = E.query_prep(Q)[0]                       # the centre products the in-graph recompute gathers
    estb, sdb = E.score_lut_zq(QC[bi].contiguous(), posb, Zq[bi].contiguous(), None, False)
    gb = dict(ok=c(okb), ids=c(ids)[in_graph], reads=c(nr)[in_graph], I=c(I)[in_graph], est=c(estb), sd=c(sdb))
    ob = {key: fb[key][:n] for key in ("ids", "reads", "I", "est", "sd")}
    assert_end_to_end(gb, dict(ob, ok=np.ones(n, bool)), z, k)
    I2, _, _ = E.search(Q, K, z, nprobe, k)
    np.testing.assert_array_equal(c(I2), c(I))


def test_packed_records_match_planes(golden_i8, eng):
    """stage 2 from packed records (one row per candidate) equals stage 2 from the separate planes, bit for bit"""
    f = golden_i8
    E, ix, idx, K, nprobe, k, M = _golden_engine(eng, f, "A_")
    assert ix.rec is not None
    B = int(f["A_nq"])
    Q = torch.from_numpy(f["Q"][:B]).to(DEV)
    QC = (Q @ ix.c).contiguous()
    g = torch.Generator().manual_seed(5)
    pos = torch.randint(0, ix.N, (B, K), generator=g).to(DEV)
    Zq = E.rotated_query(Q)
    ncnt = torch.randint(1, K + 1, (B,), generator=g, dtype=torch.int32).to(DEV)
    for half in (True, False):
        for nc in (None, ncnt):
            a = E.score_lut_zq(QC, pos, Zq, nc, half)
            rec, ix.rec = ix.rec, None
            b = E.score_lut_zq(QC, pos, Zq, nc, half)
            ix.rec = rec
            np.testing.assert_array_equal(c(a[0]), c(b[0]))
            np.testing.assert_array_equal(c(a[1]), c(b[1]))


@pytest.mark.parametrize("K", [100, 128, 40, 200])
def test_packed_records_large_batch_match_planes(golden_i8, eng, K):
    """the large-batch record kernel (one candidate per thread, one CTA per query and slice of 128 candidates: one
    partly filled slice at K = 100 and 40, a full one at 128, two at 200) equals stage 2 from the separate planes (one
    warp per candidate, the same products summed in another order) within fp32 rounding, on a batch above the SM
    count; rows past ncnt read as no candidate in both"""
    f = golden_i8
    E, ix, idx, _, nprobe, k, M = _golden_engine(eng, f, "A_")
    B = 301
    Q0 = torch.from_numpy(f["Q"]).to(DEV)
    g = torch.Generator().manual_seed(11)
    Q = (Q0[torch.randint(0, Q0.shape[0], (B,), generator=g).to(DEV)]
         + 0.05 * torch.randn(B, Q0.shape[1], generator=g).to(DEV)).contiguous()
    QC = (Q @ ix.c).contiguous()
    pos = torch.randint(0, ix.N, (B, K), generator=g).to(DEV)
    Zq = E.rotated_query(Q)
    ncnt = torch.randint(1, K + 1, (B,), generator=g, dtype=torch.int32).to(DEV)
    for half in (True, False):
        for nc in (None, ncnt):
            a = E.score_lut_zq(QC, pos, Zq, nc, half)
            rec, ix.rec = ix.rec, None
            b = E.score_lut_zq(QC, pos, Zq, nc, half)
            ix.rec = rec
            np.testing.assert_allclose(c(a[0]), c(b[0]), rtol=1e-5, atol=1e-5)
            np.testing.assert_allclose(c(a[1]), c(b[1]), rtol=1e-5, atol=1e-6)


def test_empty_batch_and_argument_errors(eng):
    """a batch of zero queries returns empty results; bad arguments raise before any device work"""
    ds, ix, oi = _random_index(eng, 20000, 256, 64, 8, seed=17)
    E = eng.EngineB200I8(ix)
    Q = ds["queries"]
    I, nr, ids = E.search(Q[:0], 40, 1.5, 12, 10)
    assert I.shape == (0, 10) and nr.shape == (0,) and ids.shape == (0, 40)
    with pytest.raises(ValueError):
        E.search(Q, 10, 1.5, 12, 10)                      # K must exceed k
    L = pkg("_lib")
    with pytest.raises(L.FvsError):
        E.route(Q, ix.NC + 1)                             # more probes than cells

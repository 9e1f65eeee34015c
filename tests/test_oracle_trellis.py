"""Pin the oracle's default-engine path (trellis stage 1, tiered gather stage 2) to the reference's own outputs.

Stage-1 scores of this path are fp16 dot products accumulated in fp32 (`tl.dot` in the reference), so they are
compared within fp32 rounding; thresholds, emitted sets and candidates are compared exactly where no estimate lies
within that rounding of the decision boundary."""
import os

import numpy as np
import pytest
import torch

from conftest import GOLDEN
from oracle import fvs_oracle as O

TOL = 2e-6


@pytest.fixture(scope="module")
def gt():
    return dict(np.load(os.path.join(GOLDEN, "trellis_reference.npz")))


def tindex(f):
    TS = [tuple(int(v) for v in r) for r in f["TS"]]
    code = dict(TS=TS, planes=[f[f"planes{t}"] for t in range(len(TS))], cbf=[f[f"cbf{t}"] for t in range(len(TS))],
                scale=f["scale"], sig=f["sig"], VP=f["VP"])
    return dict(off=f["off"], order=f["order"], means16=f["means16"], inv_mnorm=f["inv_mnorm"], c=f["c"], W1=f["W1"],
                tab=f["tab"], words=f["words"], scale1=f["scale1"], H16=f["H16"], code=code)


def test_decode_and_first_pass(gt):
    f = gt
    idx = tindex(f)
    K, nprobe, k = (int(v) for v in f["params"])
    QM = f["QM"]
    probe = torch.from_numpy(QM.astype(np.float32) * f["inv_mnorm"]).topk(nprobe, 1).indices.numpy()
    off = f["off"]
    NC, N = len(off) - 1, int(off[-1])
    n1 = min(max(int(np.ceil(1.1 * K / (N / NC / 32 + 1))), 1), nprobe)
    qid, coff, ccnt, qcp, o = O.pairs(probe[:, :n1], NC, QM)
    np.testing.assert_array_equal(qid, f["k_qid1"])
    np.testing.assert_array_equal(qcp, f["k_qcp1"])
    score = lambda qr, rw, qc: O.trellis_scores(f["k_Qh"], f["words"], f["tab"], f["scale1"], qr, rw, qc)
    bmc = O.first_pass(None, None, qid, coff, ccnt, off, None, None, qcp, int(f["k_MB"]), score=score)
    g = f["k_bmc"].reshape(-1)
    valid = g > -1e29
    np.testing.assert_array_equal(bmc > -1e29, valid)
    np.testing.assert_allclose(bmc[valid], g[valid], rtol=TOL, atol=TOL)
    t0 = O.threshold(bmc, O.pair_slots(o, len(QM), n1), len(QM), n1, int(f["k_MB"]), int(np.ceil(0.75 * K)))
    np.testing.assert_allclose(t0, f["k_t0"], rtol=TOL, atol=TOL)


def test_emit_and_select(gt):
    f = gt
    off = f["off"]
    NC = len(off) - 1
    K = int(f["params"][0])
    score = lambda qr, rw, qc: O.trellis_scores(f["k_Qh"], f["words"], f["tab"], f["scale1"], qr, rw, qc)
    # the reference's own threshold as input
    cnt, pos_l, est_l = O.emit(None, None, f["k_qid"], f["k_coff"], f["k_ccnt"], off, None, None, f["k_qcp"],
                               f["k_t0"], len(f["k_t0"]), score=score)
    eq, ev, ep = f["k_emit_q"], f["k_emit_val"], f["k_emit_pos"]
    for q in range(len(cnt)):
        sel = eq == q
        gp, gv = ep[sel], ev[sel]
        o2 = np.argsort(gp, kind="stable")
        gp, gv = gp[o2], gv[o2]
        # entries far from the threshold agree exactly as sets; estimates agree within fp32 rounding
        far_g = np.abs(gv - f["k_t0"][q]) > TOL * (1 + abs(f["k_t0"][q]))
        far_o = np.abs(est_l[q] - f["k_t0"][q]) > TOL * (1 + abs(f["k_t0"][q]))
        np.testing.assert_array_equal(np.sort(gp[far_g]), np.sort(pos_l[q][far_o]))
        common, ia, ib_ = np.intersect1d(gp, pos_l[q], return_indices=True)
        np.testing.assert_allclose(gv[ia], est_l[q][ib_], rtol=TOL, atol=TOL)
    pos, est1, ok = O.select_topk(pos_l, est_l, cnt, K, int(f["k_M"]))
    np.testing.assert_array_equal(ok, f["out_ok"])
    np.testing.assert_array_equal(np.sort(pos, 1), np.sort(f["k_pos"], 1))


def test_tiered_gather_stage2_and_final(gt):
    f = gt
    idx = tindex(f)
    code = idx["code"]
    Q = f["Q"]
    Zq = Q.astype(np.float64) @ f["VP"].astype(np.float64)
    est, sd = O.tiered_score(f["k_pos"], f["k_QC"], Zq, code["TS"], code["planes"], code["cbf"], code["scale"],
                             code["sig"])
    np.testing.assert_allclose(est, f["k_est"], rtol=1e-5, atol=1e-5)
    np.testing.assert_allclose(sd, f["k_sd"], rtol=1e-5, atol=1e-6)
    k = int(f["params"][2])
    sure, amb = O.classify(f["k_est"], f["k_sd"], float(f["z"]), k)
    np.testing.assert_array_equal(amb, f["k_amb"].astype(bool))
    ids = f["order"][f["k_pos"]]
    np.testing.assert_array_equal(ids, f["k_ids"])
    np.testing.assert_array_equal(O.final_topk(ids, f["k_score"], k), f["out_I"])


def test_search_trellis_end_to_end(gt):
    f = gt
    idx = tindex(f)
    K, nprobe, k = (int(v) for v in f["params"])
    probe = torch.from_numpy(f["QM"].astype(np.float32) * f["inv_mnorm"]).topk(nprobe, 1).indices.numpy()
    out = O.search_trellis(idx, f["Q"], K, float(f["z"]), nprobe, k, QM=f["QM"], probe=probe, Qh=f["k_Qh"])
    np.testing.assert_array_equal(out["ok"], f["out_ok"])
    same = out["reads"] == f["out_reads"]
    assert same.mean() >= 0.9
    np.testing.assert_array_equal(out["I"][same], f["out_I"][same])


def test_trellis_encoder_matches_reference_words(gt):
    """The oracle's table, Viterbi and bit packing re-encode the golden cell residuals to the reference's own words."""
    f = gt
    tab = f["tab"]
    T = O.trellis_table(10)
    alpha = float(tab[np.argmax(np.abs(T))] / T[np.argmax(np.abs(T))])
    np.testing.assert_allclose(tab, (np.float32(alpha) * T).astype(np.float32), rtol=1e-6)
    off = torch.as_tensor(f["off"])
    N = len(f["order"])
    cell = torch.searchsorted(off, torch.arange(N), right=True) - 1
    X16 = torch.from_numpy(f["H16"])
    rows = torch.arange(0, N, 7)[:160]                   # a spread sample of rows (the encoder is O(R 2^L) per row)
    Rr = X16[torch.from_numpy(f["order"]).long()[rows]].float() - torch.from_numpy(f["means16"]).float()[cell[rows]]
    Z = Rr @ torch.from_numpy(f["W1"])
    nz = Z.norm(dim=1).clamp(min=1e-6)
    Zs = (Z / nz[:, None] * 256 ** 0.5).numpy()
    path = O.viterbi_paths(Zs, (np.float32(alpha) * T).astype(np.float32), 10)
    words = O.paths_to_words(path, 10)
    same = (words == f["words"][rows.numpy()]).all(1)
    assert same.all(), same.mean()


@pytest.mark.parametrize("tag", ["s6_", "m20_"])
def test_small_batch_paths_match_reference(gt, tag):
    """B <= 8 (`search_small`, fp32 estimate) and 8 < B <= 32 (`search_mask`, fp16 tensor-core estimate): threshold,
    emitted sets, exactness flags and final ids as the reference's `EngineC._gpu`."""
    f = gt
    idx = tindex(f)
    K, nprobe, k = (int(v) for v in f["params"])
    Q = f[tag + "Q"]
    QM = (Q.astype(np.float16).astype(np.float32) @ f["means16"].astype(np.float32).T).astype(np.float16)
    probe = torch.from_numpy(QM.astype(np.float32) * f["inv_mnorm"]).topk(nprobe, 1).indices.numpy()
    out = O.search_trellis(idx, Q, K, float(f["z"]), nprobe, k, QM=QM, probe=probe)
    np.testing.assert_allclose(out["t0"], f[tag + "t0"], rtol=TOL, atol=TOL)
    np.testing.assert_array_equal(out["ok"], f[tag + "out_ok"])
    eq, ev, ep = f[tag + "emit_q"], f[tag + "emit_val"], f[tag + "emit_pos"]
    for q in range(len(Q)):
        sel = eq == q
        tq = f[tag + "t0"][q]
        far = lambda v: np.abs(v - tq) > TOL * (1 + abs(tq))
        np.testing.assert_array_equal(np.sort(ep[sel][far(ev[sel])]), np.sort(out["pos_l"][q][far(out["est_l"][q])]))
    same = out["reads"] == f[tag + "out_reads"]
    assert same.mean() >= 0.8
    np.testing.assert_array_equal(out["I"][same], f[tag + "out_I"][same])

"""Pin the CPU oracle to the reference's own outputs (golden vectors from tests/golden/make_golden.py).

Integer work (pairs, block maxima, thresholds, emitted sets, counts, LUT entries) must match bit for bit; floating
sums whose order the reference leaves to Triton (tier sums, LUT-scored estimates, exact dot products) within 1e-5
relative."""
import numpy as np
import pytest
import torch

from conftest import golden_index
from oracle import fvs_oracle as O

CASES = ["A_", "B_"]


def _probe(f, case, nprobe):
    """routing as the reference does it on the CPU (torch topk over the fp16 product QM)."""
    return torch.from_numpy(f[case + "QM"]).topk(nprobe, 1).indices.numpy()


def _setup(f, case):
    K, nprobe, k, M = (int(v) for v in f[case + "params"])
    idx = golden_index(f, case)
    off = idx["off"]
    NC = len(off) - 1
    N = int(off[-1])
    B = int(f[case + "nq"])
    mnorm = (np.float32(1.0) / idx["inv_mnorm"].astype(np.float32)).astype(np.float32)
    return K, nprobe, k, M, idx, off, NC, N, B, mnorm


@pytest.mark.parametrize("case", CASES)
def test_static_blocks(golden_i8, case):
    f = golden_i8
    pcell, pblk, ps, pe, MB = O.static_blocks(f[case + "s1_off"])
    for name, v in zip(["pcell", "pblk", "ps", "pe"], [pcell, pblk, ps, pe]):
        np.testing.assert_array_equal(v, f[case + "k_" + name])
    assert MB == int(f[case + "k_MB"])


@pytest.mark.parametrize("case", CASES)
def test_pairs_first_pass_threshold_emit(golden_i8, case):
    f = golden_i8
    K, nprobe, k, M, idx, off, NC, N, B, mnorm = _setup(f, case)
    probe = _probe(f, case, nprobe)
    n1 = O.first_pass_cells(K, N, NC, nprobe)
    QM = f[case + "QM"]
    qid, coff, ccnt, qcp, o = O.pairs(probe[:, :n1], NC, QM, mnorm)
    np.testing.assert_array_equal(qid, f[case + "k_qid1"])
    np.testing.assert_array_equal(coff, f[case + "k_coff1"])
    np.testing.assert_array_equal(ccnt, f[case + "k_ccnt1"])
    np.testing.assert_array_equal(qcp, f[case + "k_qcp1"])
    q8, qs = f[case + "k_q8"], f[case + "k_qs"]
    MB = int(f[case + "k_MB"])
    bmc = O.first_pass(q8, qs, qid, coff, ccnt, off, idx["Z"], idx["zs"], qcp, MB)
    np.testing.assert_array_equal(bmc, f[case + "k_bmc"].reshape(-1))
    inv = O.pair_slots(o, B, n1)
    t0 = O.threshold(bmc, inv, B, n1, MB, int(np.ceil(0.6 * K)))
    np.testing.assert_array_equal(t0, f[case + "k_t0"])
    qid, coff, ccnt, qcp, _ = O.pairs(probe, NC, QM, mnorm)
    np.testing.assert_array_equal(qid, f[case + "k_qid"])
    np.testing.assert_array_equal(qcp, f[case + "k_qcp"])
    cnt, pos_l, est_l = O.emit(q8, qs, qid, coff, ccnt, off, idx["Z"], idx["zs"], qcp, t0, B)
    np.testing.assert_array_equal(cnt, f[case + "k_cnt"])
    eq, ev, ep = f[case + "k_emit_q"], f[case + "k_emit_val"], f[case + "k_emit_pos"]
    for q in range(B):
        if cnt[q] > M:
            continue
        sel = eq == q
        o2 = np.argsort(ep[sel], kind="stable")
        np.testing.assert_array_equal(pos_l[q], ep[sel][o2])
        np.testing.assert_array_equal(est_l[q], ev[sel][o2])
    pos, est1, ok = O.select_topk(pos_l, est_l, cnt, K, M)
    np.testing.assert_array_equal(ok, f[case + "out_ok"])
    good = cnt <= M
    np.testing.assert_array_equal(est1[good], f[case + "out_est1"][good])
    np.testing.assert_array_equal(pos[good], f[case + "k_pos"][good])
    np.testing.assert_array_equal(O.delta_count(f[case + "out_est1"], 0.07), f[case + "k_ncnt"])


@pytest.mark.parametrize("case", CASES)
def test_quantize_matches_reference(golden_i8, case):
    f = golden_i8
    q8, qs = O.quantize_queries(f["Q"][:int(f[case + "nq"])], f["Vr"])
    np.testing.assert_allclose(qs, f[case + "k_qs"], rtol=1e-6)
    diff = np.abs(q8.astype(int) - f[case + "k_q8"].astype(int))
    assert diff.max() <= 1 and (diff > 0).mean() < 1e-3


@pytest.mark.parametrize("case", CASES)
def test_lut_stage2(golden_i8, case):
    f = golden_i8
    idx = golden_index(f, case)
    code = idx["code"]
    L = O.lut_build(f[case + "k_Zq"], half=True)
    np.testing.assert_array_equal(L, f[case + "k_L"])
    qsum, qn2 = O.tier_sums(f[case + "k_Zq"], code["TS"])
    np.testing.assert_allclose(qsum, f[case + "k_qsum"], rtol=1e-5, atol=1e-6)
    np.testing.assert_allclose(qn2, f[case + "k_qn2"], rtol=1e-5, atol=1e-7)
    est, sd = O.lut_score(f[case + "k_pos"], f[case + "k_QC"], f[case + "k_L"], code["TS"], code["planes"],
                          code["deltas"], code["scale"], code["sig"], f[case + "k_qsum"], f[case + "k_qn2"],
                          f[case + "k_ncnt"])
    np.testing.assert_allclose(est, f[case + "k_est"], rtol=1e-5, atol=1e-5)
    np.testing.assert_allclose(sd, f[case + "k_sd"], rtol=1e-5, atol=1e-7)


@pytest.mark.parametrize("case", CASES)
def test_classify_stage3_final(golden_i8, case):
    f = golden_i8
    K, nprobe, k, M, idx, off, NC, N, B, mnorm = _setup(f, case)
    z = float(f[case + "z"])
    sure, amb = O.classify(f[case + "k_est"], f[case + "k_sd"], z, k)
    np.testing.assert_array_equal(amb, f[case + "k_amb"].astype(bool))
    ids = idx["order"][f[case + "k_pos"]]
    np.testing.assert_array_equal(ids, f[case + "k_ids"])
    score = O.stage3(idx["H16"], ids, amb, f["Q"][:B], f[case + "k_est"], sure)
    np.testing.assert_allclose(score, f[case + "k_score"], rtol=1e-5, atol=1e-6)
    I = O.final_topk(ids, f[case + "k_score"], k)
    np.testing.assert_array_equal(I, f[case + "out_I"])
    np.testing.assert_array_equal(amb.sum(1), f[case + "out_reads"])


@pytest.mark.parametrize("case", CASES)
def test_end_to_end_search(golden_i8, case):
    """the oracle's whole EngineI8 search (with the reference's routing and host products as inputs)."""
    f = golden_i8
    K, nprobe, k, M, idx, off, NC, N, B, mnorm = _setup(f, case)

    class Knobs(O.I8Knobs):
        MSZ = M

    out = O.search_i8(idx, f["Q"][:B], K, float(f[case + "z"]), nprobe, k, Knobs, QM=f[case + "QM"],
                      probe=_probe(f, case, nprobe), q8qs=(f[case + "k_q8"], f[case + "k_qs"]), Zq=f[case + "k_Zq"],
                      fallback=False)
    np.testing.assert_array_equal(out["ok"], f[case + "out_ok"])
    ok = out["ok"]
    np.testing.assert_array_equal(out["I"][ok], f[case + "out_I"][ok])
    np.testing.assert_array_equal(out["reads"][ok], f[case + "out_reads"][ok])
    np.testing.assert_array_equal(out["ids"][ok], f[case + "out_ids"][ok])


def test_fallback_path(golden_i8):
    """`_fallback` (rho 1.0, M 65536, fp32 LUT, no delta rule) on the rows the generator recomputed."""
    f, case = golden_i8, "A_"
    K, nprobe, k, M, idx, off, NC, N, B, mnorm = _setup(f, case)
    rows = f[case + "out_fb_rows"]
    Q = f["Q"][rows]
    QMr = f[case + "QM"][rows]
    q8, qs = f[case + "k_q8"][rows], f[case + "k_qs"][rows]
    Zq = f[case + "k_Zq"][rows]
    out = O._search_i8_core(idx, Q, K, float(f[case + "z"]), nprobe, k, O.I8Knobs, QMr,
                            torch.from_numpy(QMr).topk(nprobe, 1).indices.numpy(), (q8, qs), Zq, rho_override=1.0)
    np.testing.assert_array_equal(out["I"], f[case + "out_fb_I"])
    np.testing.assert_array_equal(out["reads"], f[case + "out_fb_reads"])

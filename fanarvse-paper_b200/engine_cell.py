"""Default-engine search (cell-residual trellis stage 1, tiered gather stage 2) on the B200 C library: the drop-in
for the reference's `EngineS` (`src/engine_cell.py:69-104`).

`search(Qb, K, z, nprobe, k) -> (I [B,k], reads [B], cand_ids [B,K])`, one CUDA graph per (B, K, z, nprobe, k), the
exactness flag as the only host synchronisation, and a recompute of flagged queries.  Host-side PyTorch keeps the
dense products the reference computes with cuBLAS (QM = fp16(Q) @ means16^T, q . c, Q @ W1, Q @ VP); routing
selection, pair lists, the trellis scan passes, threshold, stage-1 top-K, tiered gather scoring, classification,
exact re-rank and final top-k run in libfanar_b200.  There is no CPU path.
"""
from __future__ import annotations

import numpy as np
import torch

from . import _lib
from ._lib import ptr
from .engine import BN, EngineB200I8, cell_part_order, static_tiles


class IndexS:
    """Device-resident default-engine index in the reference's layout.

    s1   : off, order, c, means16, inv_mnorm, W1 [d,R] f32, tab [2^L] f32, words [N,W] int32, scale1 [N] fp16
           (`src/engine_cell.py:8-32`, `src/rev_fanardb.py:36-60`)
    code : Lloyd-Max tiered code: TS, planes, scale, sig, VP [d,D] f32 and cbf (per-tier codebook levels)
           (`src/tiered_fused.py:47-52`)
    H16  : fp16 full-precision store [N, d] in original-id order
    """

    def __init__(self, s1, code, H16, device="cuda", L=10, packed=True):
        dev = torch.device(device)
        self.device = dev
        f = lambda x, dt=None: torch.as_tensor(x).to(device=dev, dtype=dt).contiguous()
        self.off_np = np.asarray(s1["off"] if "off" in s1 else s1["off_t"].cpu().numpy(), np.int64)
        self.off = f(self.off_np, torch.int64)
        self.NC = len(self.off_np) - 1
        self.N = int(self.off_np[-1])
        self.order = f(s1["order"], torch.int32)
        self.c = f(s1["c"], torch.float32)
        self.means16 = f(s1["means16"], torch.float16)
        self.inv_mnorm = f(s1["inv_mnorm"], torch.float32)
        self.mnorm = None                      # pair constants are q . m_c itself (no normalised routing product)
        self.W1 = f(s1["W1"], torch.float32)
        self.R = self.W1.shape[1]
        self.L = int(s1.get("L", L))
        self.tab = f(s1["tab"], torch.float32)
        self.words = f(s1["words"], torch.int32)
        self.W = self.words.shape[1]
        self.scale1 = f(s1["scale1"], torch.float16)
        self.TS = [tuple(int(v) for v in t) for t in code["TS"]]
        self.T = len(self.TS)
        self.D = self.TS[-1][1]
        self.planes = [f(p, torch.uint8) for p in code["planes"]]
        self.cbf = [f(cb, torch.float32) for cb in code["cbf"]]
        self.scale = f(code["scale"], torch.float16)
        self.sig = f(code["sig"], torch.float16)
        self.VP = f(code["VP"], torch.float32)[:, :self.D].contiguous()
        self.H16 = f(H16, torch.float16)
        self.d = self.H16.shape[1]
        sizes = np.diff(self.off_np)
        # cells largest first: the order in which the cell-major scan hands cells out; as work-list entries, a large cell
        # as several parts
        order = np.argsort(-sizes, kind="stable").astype(np.int32)
        self.cell_order = f(order, torch.int32)
        self.cell_parts = f(cell_part_order(self.off_np, order, _lib.lib().fvs_cell_part_tiles()), torch.int32)
        self.NP = int(self.cell_parts.numel())
        tc, tr, self.MB = static_tiles(self.off_np, _lib.lib().fvs_trellis_tile_rows())
        self.tile_cell, self.tile_row0 = f(tc, torch.int32), f(tr, torch.int32)
        self.ntiles = len(tc)
        self._ts_s = _lib.i32_array([s for s, _, _ in self.TS])
        self._ts_e = _lib.i32_array([e for _, e, _ in self.TS])
        self._ts_b = _lib.i32_array([b for _, _, b in self.TS])
        self._ts_cb = _lib.ptr_array(self.cbf)
        self._ts_p = _lib.ptr_array(self.planes)
        self.rec = None
        if packed:
            from .index_build import pack_records
            self.rec, self.RB, self.soff, _ = pack_records(self.TS, self.planes, self.scale, self.sig)

    def nbytes_per_vector(self):
        return 4 * self.W + 2 + sum((e - s) * b for s, e, b in self.TS) / 8 + 4 * self.T


TRELLIS_CELLS_MAX_L = 10   # FVS_TRELLIS_CELLS_MAX_L: largest trellis window of the tcgen05 scan


class EngineB200S(EngineB200I8):
    """The reference's EngineS on libfanar_b200: (beta, rho) = (1.1, 0.75) for K <= 400 else (0.7, 0.5),
    M = max(4096, 16 K) (`src/engine_cell.py:78-79`, `src/s1cell.py:181`).  Graph capture, the flag read and the
    flagged-row recompute are inherited from EngineB200I8.

    SCAN = "cells" (the product path): batches above SMALL scan with the cell-major tcgen05 kernel
    (fvs_trellis_scan_cells); "mma" keeps the mma.sync tile kernel (fvs_trellis_scan) as the measured baseline, which
    also takes trellis windows above TRELLIS_CELLS_MAX_L."""
    M = None
    FB_M = 65536
    FB_INGRAPH = 0        # flagged rows are recomputed from the host (no in-graph recompute on this path)
    TINY, SMALL, CAP_SMALL = 8, 32, 8192      # `EngineC.TINY/SMALL`, `search_small`/`search_mask` CAP

    def __init__(self, index: IndexS):
        super().__init__(index)
        self.DELTA = None

    def route(self, Qb, nprobe):
        """QM = fp16(Q) @ means16^T (cuBLAS) and the nprobe cells of largest float(QM) / |m_c| (`src/engine_cell.py:40-42`)."""
        ix = self.ix
        QM = (Qb.half() @ ix.means16.T).contiguous()
        probe = torch.empty(Qb.shape[0], nprobe, dtype=torch.int64, device=Qb.device)
        self._call("route_topk", self.L.fvs_route_topk_scaled, ptr(QM), Qb.shape[0], ix.NC, nprobe, ptr(ix.inv_mnorm),
                   ptr(probe))
        return QM, probe

    def cells_scan(self):
        return self.SCAN == "cells" and self.ix.L <= TRELLIS_CELLS_MAX_L

    def _scan(self, mode, name, Qh, B, qid, coff, ccnt, qcp, t0, cnt, bval, bpos, M, bmc, mb=None, lists=None):
        ix = self.ix
        if lists is not None:
            lst, nl = lists
            self._call(name, self.L.fvs_trellis_scan_cells, mode, ptr(Qh), B, ix.R, ptr(qid), ptr(coff), ptr(ccnt),
                       ptr(qcp), ptr(lst), ptr(nl), ix.NP, ptr(ix.off), ix.NC, ptr(ix.words), ix.W, ptr(ix.tab), ix.L,
                       ptr(ix.scale1), ptr(t0), ptr(cnt), ptr(bval), ptr(bpos), M, ptr(bmc), ix.MB, ptr(self.sched),
                       ptr(self.status))
            return
        self._call(name, self.L.fvs_trellis_scan, mode, ptr(Qh), B, ix.R, ptr(qid), ptr(coff), ptr(ccnt), ptr(qcp),
                   ptr(ix.tile_cell), ptr(ix.tile_row0), ix.ntiles, ptr(ix.off), ix.NC, ptr(ix.words), ix.W,
                   ptr(ix.tab), ix.L, ptr(ix.scale1), ptr(t0), ptr(cnt), ptr(bval), ptr(bpos), M, ptr(bmc),
                   mb or ix.MB)

    def trellis_passes(self, K, nprobe, rho_override=None):
        """(rho, n1) of the batched trellis stage 1: (beta, rho) = (1.1, 0.75) for K <= 400 else (0.7, 0.5), (1.5,
        rho_override) for the recompute; n1 = the first pass's probe columns (`src/s1cell.py:176-184`)."""
        ix = self.ix
        beta, rho = (1.1, 0.75) if K <= 400 else (0.7, 0.5)
        if rho_override:
            beta, rho = 1.5, rho_override
        return rho, min(max(int(np.ceil(beta * K / (ix.N / ix.NC / BN + 1))), 1), nprobe)

    def route_pairs(self, QM, nprobe, n1):
        """`(QM.float() * inv_mnorm).topk(nprobe)` (`src/engine_cell.py:40-42`) and both passes' `_pairs_static` lists
        (`src/s1cell.py:170-175, 184, 192`) in two launches (fvs_route_pairs_scaled), with the scan's cell lists and
        cleared emit counters.  Returns probe and the pair tuple stage1_trellis takes."""
        ix = self.ix
        B = QM.shape[0]
        dev = QM.device
        work = self.__dict__.get("_rp_work")
        if work is None:
            work = self._rp_work = torch.zeros(2 * ix.NC + 1, dtype=torch.int32, device=dev)
        probe = torch.empty(B, nprobe, dtype=torch.int64, device=dev)
        n = B * nprobe
        qid = torch.empty(n, dtype=torch.int32, device=dev)
        qcp = torch.empty(n, device=dev)
        coff, ccnt, ccnt1 = (torch.empty(ix.NC, dtype=torch.int32, device=dev) for _ in range(3))
        list1, lst = (torch.empty(ix.NP, dtype=torch.int32, device=dev) for _ in range(2))
        slot = torch.empty(B * n1, dtype=torch.int32, device=dev)
        nl = torch.empty(2, dtype=torch.int32, device=dev)
        cnt = torch.empty(B, dtype=torch.int32, device=dev)
        self._call("route_pairs", self.L.fvs_route_pairs_scaled, ptr(QM), B, ix.NC, nprobe, n1, ptr(ix.inv_mnorm),
                   ptr(ix.mnorm), ptr(ix.cell_parts), ix.NP, ptr(probe), ptr(qid), ptr(qcp), ptr(coff), ptr(ccnt), ptr(ccnt1),
                   ptr(slot), ptr(list1), ptr(lst), ptr(nl), ptr(cnt), B, ptr(work))
        self.launches += 1   # two kernels
        return probe, (qid, coff, ccnt, ccnt1, qcp, slot, list1, lst, nl, cnt)

    def stage1_trellis(self, Qb, QM, probe, K, rho_override=None, M_override=None, Qh=None, pairs=None):
        """`s1cell.search_static` (`src/s1cell.py:176-195`) on the C library: returns pos [B,K] int64, ok [B] bool,
        est1 [B,K]."""
        ix, L = self.ix, self.L
        B = Qb.shape[0]
        dev = Qb.device
        if Qh is None:
            Qh = (Qb @ ix.W1).half().contiguous()
        M = M_override or self.M or max(4096, 16 * K)
        nprobe = probe.shape[1]
        rho, n1 = self.trellis_passes(K, nprobe, rho_override)
        probe = probe.contiguous()
        l1 = l2 = None
        if pairs is not None:             # from route_pairs: pair lists, cell lists, cleared counters
            qid, coff, ccnt, ccnt1, qcp, slot, list1, lst, nl, cnt = pairs
            l1, l2 = (list1, nl[0:1]), (lst, nl[1:2])
        else:
            # one pair list serves both passes: each cell's pairs from the first n1 probe columns come first
            qid, coff, ccnt, ccnt1, qcp, slot = self.pairs_split(probe, n1, QM)
            if self.cells_scan():
                cnt = torch.empty(B, dtype=torch.int32, device=dev)            # cleared by the list kernel
                list1, lst, nl = self.cell_lists(ccnt1, ccnt, cnt)
                l1, l2 = (list1, nl[0:1]), (lst, nl[1:2])
            else:
                cnt = torch.zeros(B, dtype=torch.int32, device=dev)
        bmc = torch.empty(qid.numel() * ix.MB, device=dev)   # block-maxima rows addressed by pair position
        self._scan(0, "trellis_scan_first", Qh, B, qid, coff, ccnt1, qcp, None, None, None, None, 0, bmc, lists=l1)
        t0 = torch.empty(B, device=dev)
        self._call("threshold", L.fvs_threshold, ptr(bmc), ix.MB, ptr(slot), ptr(probe), nprobe, n1, ptr(ix.off), B,
                   int(np.ceil(rho * K)), ptr(t0))
        bval = torch.empty(B, M, device=dev)
        bpos = torch.empty(B, M, dtype=torch.int32, device=dev)
        self._scan(1, "trellis_scan_emit", Qh, B, qid, coff, ccnt, qcp, t0, cnt, bval, bpos, M, None, lists=l2)
        pos = torch.empty(B, K, dtype=torch.int64, device=dev)
        est1 = torch.empty(B, K, device=dev)
        ok = torch.empty(B, dtype=torch.uint8, device=dev)
        self._call("select_topk", L.fvs_select_topk, ptr(bval), ptr(bpos), ptr(cnt), B, M, K, ptr(pos), ptr(est1),
                   ptr(ok), None, 0.0, 9)
        self._last = dict(t0=t0, cnt=cnt, n1=n1, M=M, bmc=bmc, Qh=Qh, ccnt=ccnt, ccnt1=ccnt1, npairs=int(qid.numel()),
                          bval=bval, bpos=bpos, slot=slot, scan_args=(qid, coff, qcp, l1, l2))
        return pos, ok.bool(), est1

    def stage1_small(self, Qb, QM, probe, K):
        """`EngineC._gpu` stage 1 for B <= 32 (`src/engine_cell.py:49-56`): `search_small` (B <= 8: fp32 estimate,
        streaming kernel straight from the probe list) or `search_mask` (fp16 tensor-core estimate through the pair
        lists); (beta, rho) = (1.1, 0.75), an 8192-entry buffer, first-pass maxima merged per global 32-row block and
        t0 = the r-th largest of them (`src/s1small_cell.py:38, 70`)."""
        ix, L = self.ix, self.L
        B = Qb.shape[0]
        dev = Qb.device
        beta, rho = 1.1, 0.75
        M = self.CAP_SMALL
        nprobe = probe.shape[1]
        n1 = min(max(int(np.ceil(beta * K / (ix.N / ix.NC / BN + 1))), 1), nprobe)
        r = int(np.ceil(rho * K))
        NBg = (ix.N + BN - 1) // BN
        probe = probe.contiguous()
        bm = torch.full((B, NBg), -1e30, device=dev)
        cnt = torch.zeros(B, dtype=torch.int32, device=dev)
        bval = torch.empty(B, M, device=dev)
        bpos = torch.empty(B, M, dtype=torch.int32, device=dev)
        t0 = torch.empty(B, device=dev)
        if B <= self.TINY:
            Qr = (Qb @ ix.W1).contiguous()
            common = lambda mode, ncols: (mode, ptr(Qr), B, ix.R, ptr(probe), nprobe, ncols, ptr(QM), ix.NC,
                                          ptr(ix.off), ptr(ix.words), ix.W, ptr(ix.tab), ix.L, ptr(ix.scale1))
            self._call("trellis_small_first", L.fvs_trellis_scan_small, *common(0, n1), None, None, None, None, 0,
                       ptr(bm), NBg, ix.MB)
            self._call("threshold", L.fvs_rth_largest, ptr(bm), B, NBg, NBg, r, ptr(t0))
            self._call("trellis_small_emit", L.fvs_trellis_scan_small, *common(1, nprobe), ptr(t0), ptr(cnt),
                       ptr(bval), ptr(bpos), M, None, NBg, ix.MB)
            q_used = Qr
        else:
            Qh = (Qb @ ix.W1).half().contiguous()
            qid, coff, ccnt, qcp, _ = self.pairs(probe, n1, QM, False)
            self._scan(2, "trellis_scan_first", Qh, B, qid, coff, ccnt, qcp, None, None, None, None, 0, bm, mb=NBg)
            self._call("threshold", L.fvs_rth_largest, ptr(bm), B, NBg, NBg, r, ptr(t0))
            qid, coff, ccnt, qcp, _ = self.pairs(probe, nprobe, QM, False)
            self._scan(1, "trellis_scan_emit", Qh, B, qid, coff, ccnt, qcp, t0, cnt, bval, bpos, M, None)
            q_used = Qh
        pos = torch.empty(B, K, dtype=torch.int64, device=dev)
        est1 = torch.empty(B, K, device=dev)
        ok = torch.empty(B, dtype=torch.uint8, device=dev)
        self._call("select_topk", L.fvs_select_topk, ptr(bval), ptr(bpos), ptr(cnt), B, M, K, ptr(pos), ptr(est1),
                   ptr(ok), None, 0.0, 9)
        self._last = dict(t0=t0, cnt=cnt, n1=n1, M=M, bm=bm, Qq=q_used, bval=bval, bpos=bpos)
        return pos, ok.bool(), est1

    def rotated_query(self, Qb):
        return (Qb @ self.ix.VP).contiguous()                              # `src/tiered_fused.py:57`

    def score_tiered(self, QC, pos, Zq):
        """`tiered_fused.score` (`src/tiered_fused.py:54-72`)."""
        ix = self.ix
        B, K = pos.shape
        est = torch.empty(B, K, device=pos.device)
        sd = torch.empty(B, K, device=pos.device)
        if ix.rec is not None:
            self._call("tiered_score", self.L.fvs_tiered_score_rec, ptr(pos), B, K, ptr(QC), ptr(Zq), Zq.shape[1],
                       ix.D, ix.T, ix._ts_s, ix._ts_e, ix._ts_b, ix._ts_cb, ptr(ix.rec), ix.RB, ix.soff, ix.N, ptr(est),
                       ptr(sd))
        else:
            self._call("tiered_score", self.L.fvs_tiered_score, ptr(pos), B, K, ptr(QC), ptr(Zq), Zq.shape[1], ix.D,
                       ix.T, ix._ts_s, ix._ts_e, ix._ts_b, ix._ts_cb, ix._ts_p, ptr(ix.scale), ptr(ix.sig), ix.N,
                       ptr(est), ptr(sd))
        return est, sd

    def _finish_s(self, Qb, QC, pos, z, k):
        Zq = self.rotated_query(Qb)
        est, sd = self.score_tiered(QC, pos, Zq)
        I, reads, ids, score_k = self.refine(Qb, pos, est, sd, z, k)
        self._last.update(est=est, sd=sd, Zq=Zq, score_k=score_k)
        return I, reads.long(), ids

    def _gpu(self, Qb, K, z, nprobe, k):
        """`EngineS._gpu` (`src/engine_cell.py:74-84`), with `EngineC._gpu` for batches up to 32."""
        if K <= k:
            raise ValueError("need K > k")
        QC = (Qb @ self.ix.c).contiguous()
        if len(Qb) > self.SMALL and self.cells_scan() and self.fused_routing(len(Qb), nprobe):
            QM = (Qb.half() @ self.ix.means16.T).contiguous()
            probe, pairs = self.route_pairs(QM, nprobe, self.trellis_passes(K, nprobe)[1])
            pos, ok, est1 = self.stage1_trellis(Qb, QM, probe, K, pairs=pairs)
        else:
            QM, probe = self.route(Qb, nprobe)
            if len(Qb) <= self.SMALL:
                pos, ok, est1 = self.stage1_small(Qb, QM, probe, K)
            else:
                pos, ok, est1 = self.stage1_trellis(Qb, QM, probe, K)
        self._last.update(probe=probe, QM=QM, QC=QC, est1=est1)
        I, reads, ids = self._finish_s(Qb, QC, pos, z, k)
        return ok, I, reads, ids

    def _fallback(self, Qb, K, z, nprobe, k):
        """Recompute of flagged rows: every block maximum of the first-pass cells above the K-th is kept (rho = 1,
        beta = 1.5), buffer 65536, so that at least K candidates are emitted."""
        QC = (Qb @ self.ix.c).contiguous()
        QM, probe = self.route(Qb, nprobe)
        pos, ok, est1 = self.stage1_trellis(Qb, QM, probe, K, rho_override=1.0, M_override=self.FB_M)
        return self._finish_s(Qb, QC, pos, z, k)

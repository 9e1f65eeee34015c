"""Throughput-mode search engine on the B200 C library: the drop-in for the reference's `EngineI8`.

Mirrors `throughput/enginei8.py` (class EngineI8 with the final knobs of `throughput/e_v3final.py:28-32`):
`search(Qb, K, z, nprobe, k) -> (I [B,k], reads [B], cand_ids [B,K])`, one CUDA graph per (B, K, z, nprobe, k), the
exactness flag as the only host synchronisation, and the reference's recompute path for flagged queries.

Host-side PyTorch keeps the dense products the reference computes with cuBLAS (routing product QM, the query
projections for quantisation and for the LUT, q . c); everything else -- top-n_p routing selection, the pair lists,
the int8 scan passes, threshold, stage-1 top-K with the delta rule, LUT scoring, classification, exact re-rank and
final top-k -- runs in libfanar_b200 through its C ABI.  There is no CPU path: without the shared library (or without a GPU) `search` raises.
"""
from __future__ import annotations

import numpy as np
import torch

from . import _lib
from ._lib import check, ptr

BN = 32


def cell_part_order(off, order, part_tiles, tile_rows=128):
    """Work-list order of the cell-major scans: the cells of `order` (largest first), each as its parts
    p = 0 .. ceil(tiles / part_tiles) - 1, entries `cell | p << 16` (FVS_CELL_PART_TILES; a cell's tiles of tile_rows
    rows start at its first 32-row block), so that several CTAs share a large cell.  int32 numpy array."""
    off = np.asarray(off, np.int64)
    order = np.asarray(order, np.int64)
    assert len(off) - 1 < 65536, "cell ids of the work lists are 16-bit"
    cs, ce = off[order], off[order + 1]
    ntiles = np.where(ce > cs, (ce - (cs & ~31) + tile_rows - 1) // tile_rows, 0)
    parts = np.maximum(1, (ntiles + part_tiles - 1) // part_tiles)
    within = np.arange(int(parts.sum())) - np.repeat(np.cumsum(parts) - parts, parts)
    return (np.repeat(order, parts) | (within << 16)).astype(np.int32)


def static_tiles(off, tile_rows):
    """Static work list of the int8 scan: for every non-empty cell, tiles of `tile_rows` rows starting on the cell's
    first global 32-row boundary (`src/s1cell.py:157-168` uses 32-row blocks; a tile here is tile_rows/32 of them).
    Returns (tile_cell, tile_row0) int32 numpy arrays and MB (max blocks per cell + 1)."""
    off = np.asarray(off, np.int64)
    s, e = off[:-1], off[1:]
    first = (s // BN) * BN
    ntile = np.where(e > s, (e - first + tile_rows - 1) // tile_rows, 0)
    cell = np.repeat(np.arange(len(s)), ntile)
    k = np.arange(len(cell)) - np.repeat(np.cumsum(ntile) - ntile, ntile)
    row0 = first[cell] + k * tile_rows
    MB = int((int((e - s).max()) + BN - 1) // BN + 1)
    return cell.astype(np.int32), row0.astype(np.int32), MB


class IndexI8:
    """Device-resident throughput-mode index in the reference's layout.

    s1   : dict with off (NC+1), order (int32 [N]), c, means16, inv_mnorm          (`src/engine_cell.py:26-32`)
    i8   : dict with Z (int8 [N,R]), zs (f32 [N]), Vr (f32 [d,R])                  (`throughput/enginei8.py:19-27`)
    code : uniform tiered code: TS, planes, scale, sig, deltas and VP or VP16 (or V + rots)  (`throughput/s2lut.py`)
    H16  : fp16 full-precision store [N, d] in original-id order (HBM-resident here; pinned host RAM in the reference)
    """

    def __init__(self, s1, i8, code, H16, device="cuda", packed=True):
        dev = torch.device(device)
        self.device = dev
        f = lambda x, dt=None: torch.as_tensor(x).to(device=dev, dtype=dt).contiguous()
        self.off_np = np.asarray(s1["off"] if "off" in s1 else s1["off_t"].cpu().numpy(), np.int64)
        self.off = f(self.off_np, torch.int64)
        self.NC = len(self.off_np) - 1
        self.N = int(self.off_np[-1])
        self.order = f(s1["order"], torch.int32)
        self.c = f(s1["c"], torch.float32)
        means16 = f(s1["means16"], torch.float16)
        inv_mnorm = f(s1["inv_mnorm"], torch.float32)
        self.meansN = (means16.float() * inv_mnorm[:, None]).half().contiguous()     # `throughput/enginei8.py:66`
        self.mnorm = (1.0 / inv_mnorm).float().contiguous()
        self.Z = f(i8["Z"], torch.int8)
        self.zs = f(i8["zs"], torch.float32)
        self.Vr = f(i8["Vr"], torch.float32)
        # Vr transposed (K-major for the tensor cores) and split into a TF32 part (rounded to nearest at 10 mantissa
        # bits) and the exact remainder: the two operands of the projection kernel's 3xTF32 products
        VrT = self.Vr.t().contiguous()
        self.VrT_big = ((VrT.view(torch.int32) + 0x1000) & ~0x1FFF).view(torch.float32).contiguous()
        self.VrT_small = (VrT - self.VrT_big).contiguous()
        self.R = self.Z.shape[1]
        self.TS = [tuple(int(v) for v in t) for t in code["TS"]]
        self.T = len(self.TS)
        self.D = self.TS[-1][1]
        self.planes = [f(p, torch.uint8) for p in code["planes"]]
        self.scale = f(code["scale"], torch.float16)
        self.sig = f(code["sig"], torch.float16)
        self.deltas = [float(code["deltas"][b]) for _, _, b in self.TS]
        if "VP16" in code:
            VP16 = f(code["VP16"], torch.float16)
        elif "VP" in code:
            VP16 = f(code["VP"], torch.float32).half()
        else:
            V = f(code["V"], torch.float32)
            Dm = torch.zeros(V.shape[0], V.shape[0], device=dev)
            for (s, e, _), P in zip(self.TS, code["rots"]):
                Dm[s:e, s:e] = f(P, torch.float32)
            VP16 = (V @ Dm).half()
        self.VP16 = VP16[:, :self.D].contiguous()
        self.H16 = f(H16, torch.float16)
        self.d = self.H16.shape[1]
        sizes = np.diff(self.off_np)
        # cells largest first: the order in which the cell-major scan hands cells out (big cells early, small at the end);
        # as work-list entries, a large cell as several parts
        order = np.argsort(-sizes, kind="stable").astype(np.int32)
        self.cell_order = f(order, torch.int32)
        self.cell_parts = f(cell_part_order(self.off_np, order, _lib.lib().fvs_cell_part_tiles()), torch.int32)
        self.NP = int(self.cell_parts.numel())
        tc, tr, self.MB = static_tiles(self.off_np, _lib.lib().fvs_i8_tile_rows())
        self.tile_cell, self.tile_row0 = f(tc, torch.int32), f(tr, torch.int32)
        self.ntiles = len(tc)
        self.LW = self.D // 4 * 16
        # host-side tier descriptors for the C ABI
        self._ts_s = _lib.i32_array([s for s, _, _ in self.TS])
        self._ts_e = _lib.i32_array([e for _, e, _ in self.TS])
        self._ts_b = _lib.i32_array([b for _, _, b in self.TS])
        self._ts_d = _lib.f32_array(self.deltas)
        self._ts_p = _lib.ptr_array(self.planes)
        # packed refinement records (one coalesced row per candidate in stage 2), the reference's `tiered_fused.pack`
        self.rec = None
        if packed:
            from .index_build import pack_records
            self.rec, self.RB, self.soff, _ = pack_records(self.TS, self.planes, self.scale, self.sig)

    def nbytes_per_vector(self):
        return self.R + 4 + sum((e - s) * b for s, e, b in self.TS) / 8 + 4 * self.T


class EngineB200I8:
    """The reference's EngineI8 (FanarVSE-T) on libfanar_b200.  Knobs as in `throughput/e_v3final.py:28-32`."""
    RHO = 0.6
    MSZ = 3072
    DELTA = 0.07
    LUTH = True
    BETA = None
    SCAN = "cells"   # "cells": cell-major tcgen05 scan (the product path); "tc": tile-major tcgen05 scan; "mma": the
    #                  mma.sync scan, kept as measured baselines
    SMALL = 32       # batches up to this size take the streaming scan (fvs_i8_scan_small) instead of the tile scan
    FB_INGRAPH = 48  # flagged rows recomputed inside the batch's own graph (batches of FB_MIN_BATCH or more)
    FB_MIN_BATCH = 256

    def __init__(self, index: IndexI8):
        self.ix = index
        self.graphs = {}
        self.graph_launches = {}
        self._async_slot = {}      # per search shape: the graph the next search_async replays (two alternate)
        self.nbad = 0
        self.nbad2 = 0
        self.launches = 0          # library kernel launches issued (eager) or captured
        self.timing = None         # dict name -> [(start, end) CUDA events] when timing library calls
        self.L = _lib.lib()
        self.status = torch.zeros(1, dtype=torch.int32, device=index.device)
        self.work = torch.zeros(index.NC, dtype=torch.int32, device=index.device)
        self._nflag = torch.zeros(1, dtype=torch.int32, device=index.device)   # rows flagged by the main pass
        # work counter of the cell-major scan (left at zero by every launch); like `status`, it belongs to one search
        # at a time: an engine's searches run one after another
        self.sched = torch.zeros(2, dtype=torch.int32, device=index.device)

    def pairs(self, probe, ncols, QM, want_slot):
        """pair list by cell over the first ncols probe columns (`throughput/enginei8.py:11-16`)."""
        ix = self.ix
        B, npr = probe.shape
        dev = probe.device
        n = B * ncols
        qid = torch.empty(n, dtype=torch.int32, device=dev)
        qcp = torch.empty(n, device=dev)
        coff = torch.empty(ix.NC, dtype=torch.int32, device=dev)
        ccnt = torch.empty(ix.NC, dtype=torch.int32, device=dev)
        slot = torch.empty(n, dtype=torch.int32, device=dev) if want_slot else None
        self._call("pairs", self.L.fvs_pairs, ptr(probe), B, npr, ncols, ix.NC, ptr(QM), ptr(ix.mnorm), ptr(qid),
                   ptr(coff), ptr(ccnt), ptr(qcp), ptr(slot), ptr(self.work))
        self.launches += 2   # fvs_pairs issues three kernels
        return qid, coff, ccnt, qcp, slot

    def pairs_split(self, probe, n1, QM):
        """both passes' pair lists as one list by cell, first-pass pairs first in each cell (`fvs_pairs_split`)."""
        ix = self.ix
        B, npr = probe.shape
        dev = probe.device
        n = B * npr
        qid = torch.empty(n, dtype=torch.int32, device=dev)
        qcp = torch.empty(n, device=dev)
        coff = torch.empty(ix.NC, dtype=torch.int32, device=dev)
        ccnt = torch.empty(ix.NC, dtype=torch.int32, device=dev)
        ccnt1 = torch.empty(ix.NC, dtype=torch.int32, device=dev)
        slot = torch.empty(B * n1, dtype=torch.int32, device=dev)
        work = self.__dict__.get("_work2")
        if work is None:
            work = self._work2 = torch.zeros(2 * ix.NC, dtype=torch.int32, device=dev)
        self._call("pairs", self.L.fvs_pairs_split, ptr(probe), B, npr, n1, ix.NC, ptr(QM), ptr(ix.mnorm), ptr(qid),
                   ptr(coff), ptr(ccnt), ptr(ccnt1), ptr(qcp), ptr(slot), ptr(work))
        self.launches += 2   # fvs_pairs_split issues three kernels
        return qid, coff, ccnt, ccnt1, qcp, slot

    def cell_lists(self, ccnt1, ccnt, zero=None):
        """the two passes' work lists for the cell-major scan: (list1, list, nlist [2] on the device); `zero` (the emit
        pass's counters) is cleared in the same launch."""
        ix = self.ix
        dev = ccnt.device
        list1 = torch.empty(ix.NP, dtype=torch.int32, device=dev)
        lst = torch.empty(ix.NP, dtype=torch.int32, device=dev)
        nl = torch.empty(2, dtype=torch.int32, device=dev)
        self._call("cell_lists", self.L.fvs_cell_lists, ptr(ix.cell_parts), ix.NP, ptr(ccnt1), ptr(ccnt), ptr(list1),
                   ptr(lst), ptr(nl), ptr(zero), 0 if zero is None else zero.numel())
        return list1, lst, nl

    def _scan(self, mode, name, q8, qs, B, qid, coff, ccnt, qcp, t0, cnt, bval, bpos, M, bmc, lists=None):
        ix = self.ix
        if self.SCAN == "cells":
            lst, nl = lists
            self._call(name, self.L.fvs_i8_scan_cells, mode, ptr(q8), ptr(qs), B, ix.R, ptr(qid), ptr(coff),
                       ptr(ccnt), ptr(qcp), ptr(lst), ptr(nl), ix.NP, ptr(ix.off), ix.NC, ptr(ix.Z), ix.N, ptr(ix.zs),
                       ptr(t0), ptr(cnt), ptr(bval), ptr(bpos), M, ptr(bmc), ix.MB, ptr(self.sched),
                       ptr(self.status))
        elif self.SCAN == "tc":
            self._call(name, self.L.fvs_i8_scan_tc, mode, ptr(q8), ptr(qs), B, ix.R, ptr(qid), ptr(coff), ptr(ccnt),
                       ptr(qcp), ptr(ix.tile_cell), ptr(ix.tile_row0), ix.ntiles, ptr(ix.off), ix.NC, ptr(ix.Z), ix.N,
                       ptr(ix.zs), ptr(t0), ptr(cnt), ptr(bval), ptr(bpos), M, ptr(bmc), ix.MB, ptr(self.status))
        else:
            self._call(name, self.L.fvs_i8_scan, mode, ptr(q8), ptr(qs), B, ix.R, ptr(qid), ptr(coff), ptr(ccnt),
                       ptr(qcp), ptr(ix.tile_cell), ptr(ix.tile_row0), ix.ntiles, ptr(ix.off), ix.NC, ptr(ix.Z),
                       ptr(ix.zs), ptr(t0), ptr(cnt), ptr(bval), ptr(bpos), M, ptr(bmc), ix.MB)

    _tag = ""        # prefix of the timing names (the in-graph recompute times its calls separately)

    def _call(self, name, fn, *args):
        """Call one C-ABI entry point on the current stream; count it; optionally bracket it with CUDA events."""
        name = self._tag + name
        if self.timing is not None:
            a = torch.cuda.Event(enable_timing=True)
            b = torch.cuda.Event(enable_timing=True)
            a.record()
            rc = fn(_lib.stream_handle(), *args)
            b.record()
            self.timing.setdefault(name, []).append((a, b))
        else:
            rc = fn(_lib.stream_handle(), *args)
        check(rc, name)
        self.launches += 1

    # ------------------------------------------------------------------ stage 1
    def query_prep(self, Qb):
        """QC = Qb @ c and Qh = fp16(Qb) (`throughput/enginei8.py:63, 67`) in one pass over the fp32 queries."""
        B, d = Qb.shape
        c = self.ix.c
        if Qb.dtype != torch.float32 or d % 4 or Qb.stride(1) != 1 or Qb.stride(0) % 4 or Qb.data_ptr() % 16:
            return (Qb @ c).contiguous(), Qb.half()          # shapes the vectorised kernel does not take
        Qh = torch.empty(B, d, dtype=torch.float16, device=Qb.device)
        QC = torch.empty(B, device=Qb.device)
        self._call("query_prep", self.L.fvs_query_prep, ptr(Qb), B, d, Qb.stride(0), ptr(c), ptr(Qh), ptr(QC))
        return QC, Qh

    KS_MAX = 16      # K-splits of the projection kernel (its partial-sum buffer is KS_MAX x B x R floats)

    def quantize(self, Qb):
        """q8, qs (`throughput/enginei8.py:38`): z = Qb @ Vr in fp32 accuracy (3xTF32 on the tensor cores, split over
        K), then the reference's quantisation, in `fvs_project_quantize`."""
        ix = self.ix
        B, d = Qb.shape
        R = ix.Vr.shape[1]
        q8 = torch.empty(B, R, dtype=torch.int8, device=Qb.device)
        qs = torch.empty(B, device=Qb.device)
        if Qb.dtype != torch.float32 or Qb.stride(1) != 1 or Qb.stride(0) % 4 or Qb.data_ptr() % 16 or R != 256:
            z = (Qb @ ix.Vr).contiguous()            # shapes the projection kernel does not take
            self._call("quantize", self.L.fvs_quantize, ptr(z), B, R, R, ptr(q8), ptr(qs))
            return q8, qs
        part = torch.empty(self.KS_MAX * B * R, device=Qb.device)
        self._call("quantize", self.L.fvs_project_quantize, ptr(Qb), B, d, Qb.stride(0), ptr(ix.VrT_big),
                   ptr(ix.VrT_small), R, ptr(q8), ptr(qs), ptr(part), self.KS_MAX, ptr(self.status))
        return q8, qs

    def first_pass_cells(self, K, nprobe, rho_override=None):
        beta = (1.1 if K <= 400 else 0.7) if not self.BETA else self.BETA
        if rho_override:
            beta = 1.5
        return min(max(int(np.ceil(beta * K / (self.ix.N / self.ix.NC / BN + 1))), 1), nprobe)

    def fused_routing(self, B, nprobe):
        """whether routing and pairing run as the two launches of fvs_route_pairs (batches that take the cell-major scan;
        shapes the fused kernels take)"""
        NC = self.ix.NC
        return self.SCAN == "cells" and B > self.SMALL and NC % 8 == 0 and NC <= 16384 and nprobe <= 512

    def route_pairs(self, QM, nprobe, n1):
        """`QM.topk(nprobe)` and both passes' pair lists (`throughput/enginei8.py:11-16, 67-70`) in two launches; also
        the scan's cell lists and cleared emit counters.  Returns probe and the pair tuple stage1_i8 takes."""
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
        self._call("route_pairs", self.L.fvs_route_pairs, ptr(QM), B, ix.NC, nprobe, n1, ptr(ix.mnorm),
                   ptr(ix.cell_parts), ix.NP, ptr(probe), ptr(qid), ptr(qcp), ptr(coff), ptr(ccnt), ptr(ccnt1), ptr(slot),
                   ptr(list1), ptr(lst), ptr(nl), ptr(cnt), B, ptr(work))
        self.launches += 1   # two kernels
        return probe, (qid, coff, ccnt, ccnt1, qcp, slot, list1, lst, nl, cnt)

    def stage1_i8(self, Qb, QM, probe, K, rho_override=None, M_override=None, q8qs=None, small=None, pairs=None):
        """`throughput/enginei8.py:36-60` on the C library: returns pos [B,K] int64, ok [B] bool, est1 [B,K], n1."""
        ix, L = self.ix, self.L
        B = Qb.shape[0]
        dev = Qb.device
        q8, qs = q8qs if q8qs is not None else self.quantize(Qb)
        M = M_override or self.MSZ or max(4096, 16 * K)
        rho = rho_override if rho_override else (self.RHO or (0.75 if K <= 400 else 0.5))
        n1 = self.first_pass_cells(K, probe.shape[1], rho_override)
        probe = probe.contiguous()
        if (B <= self.SMALL and self.SCAN != "mma") if small is None else small:
            return self._stage1_small(q8, qs, B, QM, probe, K, M, rho, n1, rho_override)
        l1 = l2 = None
        if pairs is not None:             # from route_pairs: pair lists, cell lists, cleared counters
            qid, coff, ccnt, ccnt1, qcp, slot, list1, lst, nl, cnt = pairs
            l1, l2 = (list1, nl[0:1]), (lst, nl[1:2])
        else:
            # one pair list serves both passes: each cell's pairs from the first n1 probe columns come first
            qid, coff, ccnt, ccnt1, qcp, slot = self.pairs_split(probe, n1, QM)
            if self.SCAN == "cells":
                cnt = torch.empty(B, dtype=torch.int32, device=dev)            # cleared by the list kernel
                list1, lst, nl = self.cell_lists(ccnt1, ccnt, cnt)
                l1, l2 = (list1, nl[0:1]), (lst, nl[1:2])
            else:
                cnt = torch.zeros(B, dtype=torch.int32, device=dev)
        bmc = torch.empty(qid.numel() * ix.MB, device=dev)   # block-maxima rows addressed by pair position
        self._scan(0, "i8_scan_first", q8, qs, B, qid, coff, ccnt1, qcp, None, None, None, None, 0, bmc, l1)
        t0 = torch.empty(B, device=dev)
        self._call("threshold", L.fvs_threshold, ptr(bmc), ix.MB, ptr(slot), ptr(probe), probe.shape[1], n1,
                   ptr(ix.off), B, int(np.ceil(rho * K)), ptr(t0))
        bval = torch.empty(B, M, device=dev)
        bpos = torch.empty(B, M, dtype=torch.int32, device=dev)
        self._scan(1, "i8_scan_emit", q8, qs, B, qid, coff, ccnt, qcp, t0, cnt, bval, bpos, M, None, l2)
        pos = torch.empty(B, K, dtype=torch.int64, device=dev)
        est1 = torch.empty(B, K, device=dev)
        ok = torch.empty(B, dtype=torch.uint8, device=dev)
        use_delta = self.DELTA is not None and not rho_override
        ncnt = torch.empty(B, dtype=torch.int32, device=dev) if use_delta else None
        self._call("select_topk", L.fvs_select_topk, ptr(bval), ptr(bpos), ptr(cnt), B, M, K, ptr(pos), ptr(est1),
                   ptr(ok), ptr(ncnt), float(self.DELTA or 0.0), 9)
        self._last = dict(t0=t0, cnt=cnt, n1=n1, M=M, bmc=bmc, q8=q8, qs=qs, ccnt=ccnt, ccnt1=ccnt1,
                          npairs=int(qid.numel()), bval=bval, bpos=bpos, slot=slot, ncnt=ncnt,
                          scan_args=(qid, coff, qcp, l1, l2))
        return pos, ok.view(torch.bool), est1, ncnt

    def _ident(self, n):
        """slot[i] = i (the streaming scan's pair slots), cached.  A captured graph keeps the address of the tensor it
        was given, so a tensor handed out is never released (a larger one is added when needed): releasing it would
        let the allocator reuse its memory under a graph that still reads it."""
        keep = self.__dict__.setdefault("_ident_keep", [])
        if not keep or keep[-1].numel() < n:
            keep.append(torch.arange(max(n, 1024), dtype=torch.int32, device=self.ix.device))
        return keep[-1]

    def _stage1_small(self, q8, qs, B, QM, probe, K, M, rho, n1, rho_override):
        """stage 1 for small batches: streaming scan straight from the probe list (no pair sort)."""
        ix, L = self.ix, self.L
        dev = q8.device
        npr = probe.shape[1]
        common = lambda mode, ncols: (mode, ptr(q8), ptr(qs), B, ix.R, ptr(probe), npr, ncols, ptr(QM), ix.NC,
                                      ptr(ix.mnorm), ptr(ix.off), ptr(ix.Z), ptr(ix.zs))
        bmc = torch.empty(B * n1 * ix.MB, device=dev)
        self._call("i8_scan_first", L.fvs_i8_scan_small, *common(0, n1), None, None, None, None, 0, ptr(bmc), ix.MB)
        t0 = torch.empty(B, device=dev)
        slot = self._ident(B * n1)
        self._call("threshold", L.fvs_threshold, ptr(bmc), ix.MB, ptr(slot), ptr(probe), npr, n1, ptr(ix.off), B,
                   int(np.ceil(rho * K)), ptr(t0))
        cnt = torch.zeros(B, dtype=torch.int32, device=dev)
        bval = torch.empty(B, M, device=dev)
        bpos = torch.empty(B, M, dtype=torch.int32, device=dev)
        self._call("i8_scan_emit", L.fvs_i8_scan_small, *common(1, npr), ptr(t0), ptr(cnt), ptr(bval), ptr(bpos), M,
                   None, ix.MB)
        pos = torch.empty(B, K, dtype=torch.int64, device=dev)
        est1 = torch.empty(B, K, device=dev)
        ok = torch.empty(B, dtype=torch.uint8, device=dev)
        use_delta = self.DELTA is not None and not rho_override
        ncnt = torch.empty(B, dtype=torch.int32, device=dev) if use_delta else None
        self._call("select_topk", L.fvs_select_topk, ptr(bval), ptr(bpos), ptr(cnt), B, M, K, ptr(pos), ptr(est1),
                   ptr(ok), ptr(ncnt), float(self.DELTA or 0.0), 9)
        self._last = dict(t0=t0, cnt=cnt, n1=n1, M=M, bmc=bmc, q8=q8, qs=qs, ccnt=None, npairs=B * npr, bval=bval,
                          bpos=bpos, slot=slot[:B * n1], probe=probe)
        return pos, ok.view(torch.bool), est1, ncnt

    # ------------------------------------------------------------------ stages 2-3
    def luts(self, Qb, half, Zq=None):
        ix = self.ix
        B = Qb.shape[0]
        if Zq is None:
            Zq = (Qb.half() @ ix.VP16).float().contiguous()                # `throughput/s2lut.py:122`
        Lt = torch.empty(B, ix.LW, device=Qb.device, dtype=torch.float16 if half else torch.float32)
        qsum = torch.empty(ix.T, B, device=Qb.device)
        qn2 = torch.empty(ix.T, B, device=Qb.device)
        self._call("lut_build", self.L.fvs_lut_build, ptr(Zq), B, ix.D, ix.D, int(half), ptr(Lt), ix.T, ix._ts_s,
                   ix._ts_e, ptr(qsum), ptr(qn2))
        return Lt, qsum, qn2, Zq

    def score_lut(self, QC, pos, pre, ncnt, half):
        ix = self.ix
        B, K = pos.shape
        Lt, qsum, qn2 = pre[:3]
        est = torch.empty(B, K, device=pos.device)
        sd = torch.empty(B, K, device=pos.device)
        self._call("lut_score", self.L.fvs_lut_score, ptr(pos), B, K, ptr(QC), ptr(Lt), int(half), ix.LW, ix.T,
                   ix._ts_s, ix._ts_e, ix._ts_b, ix._ts_d, ix._ts_p, ptr(ix.scale), ptr(ix.sig), ix.N, ptr(qsum),
                   ptr(qn2), ptr(ncnt), ptr(est), ptr(sd))
        return est, sd

    def score_lut_zq(self, QC, pos, Zq, ncnt, half):
        """fused table build + LUT scoring (`throughput/s2lut.py:92-126` in one launch)."""
        ix = self.ix
        B, K = pos.shape
        est = torch.empty(B, K, device=pos.device)
        sd = torch.empty(B, K, device=pos.device)
        zh = int(Zq.dtype == torch.float16)          # the fp16 product itself, or f32
        if ix.rec is not None:
            self._call("lut_score", self.L.fvs_lut_score_rec, ptr(pos), B, K, ptr(QC), ptr(Zq), Zq.shape[1], zh, ix.D,
                       int(half), ix.T, ix._ts_s, ix._ts_e, ix._ts_b, ix._ts_d, ptr(ix.rec), ix.RB, ix.soff, ix.N,
                       ptr(ncnt), ptr(est), ptr(sd))
        else:
            self._call("lut_score", self.L.fvs_lut_score_zq, ptr(pos), B, K, ptr(QC), ptr(Zq), Zq.shape[1], zh, ix.D,
                       int(half), ix.T, ix._ts_s, ix._ts_e, ix._ts_b, ix._ts_d, ix._ts_p, ptr(ix.scale), ptr(ix.sig),
                       ix.N, ptr(ncnt), ptr(est), ptr(sd))
        return est, sd

    def rotated_query(self, Qb, Qh=None):
        """Zq = fp16(Qb) @ VP16 (`throughput/s2lut.py:122`), kept in fp16: the LUT kernels read the product itself and
        take the same values as its .float()."""
        Qh = Qb.half() if Qh is None else Qh
        return (Qh @ self.ix.VP16).contiguous()

    def refine(self, Qb, pos, est, sd, z, k):
        ix = self.ix
        B, K = pos.shape
        ids = torch.empty(B, K, dtype=torch.int32, device=pos.device)
        I = torch.empty(B, k, dtype=torch.int32, device=pos.device)
        reads = torch.empty(B, dtype=torch.int32, device=pos.device)
        score_k = torch.empty(B, k, device=pos.device)
        Qf = Qb.float().contiguous()
        self._call("refine", self.L.fvs_refine, ptr(ix.H16), ix.d, ptr(ix.order), ptr(pos), ptr(est), ptr(sd), B, K,
                   float(z), k, ptr(Qf), Qf.shape[1], ptr(ids), ptr(I), ptr(reads), ptr(score_k))
        return I, reads, ids, score_k

    def _finish(self, Qb, QC, pos, ok, ncnt, K, z, k, half=None, Qh=None, Zq=None):
        """`throughput/enginei8.py:80-95`."""
        half = self.LUTH if half is None else half
        if Zq is None:
            Zq = self.rotated_query(Qb, Qh)
        est, sd = self.score_lut_zq(QC, pos, Zq, ncnt, half)
        I, reads, ids, score_k = self.refine(Qb, pos, est, sd, z, k)
        self._last.update(est=est, sd=sd, Zq=Zq, score_k=score_k)
        return ok, I, reads.long(), ids

    def route(self, Qb, nprobe, Qh=None):
        """QM = fp16(Q) @ meansN^T (cuBLAS) and the nprobe best cells per query (`throughput/enginei8.py:67-68`)."""
        Qh = Qb.half() if Qh is None else Qh
        QM = (Qh @ self.ix.meansN.T).contiguous()
        probe = torch.empty(Qb.shape[0], nprobe, dtype=torch.int64, device=Qb.device)
        self._call("route_topk", self.L.fvs_route_topk, ptr(QM), Qb.shape[0], self.ix.NC, nprobe, ptr(probe))
        return QM, probe

    def _gpu(self, Qb, K, z, nprobe, k):
        """`throughput/enginei8.py:61-70` (NROUTE branch)."""
        if K <= k or K < 10:
            raise ValueError("need K > k and K >= 10 (the delta rule reads the 10th stage-1 estimate)")
        QC, Qh = self.query_prep(Qb)         # one fp16 copy of the queries for the routing and rotation products
        pairs = None
        if self.fused_routing(len(Qb), nprobe):
            QM = (Qh @ self.ix.meansN.T).contiguous()
            probe, pairs = self.route_pairs(QM, nprobe, self.first_pass_cells(K, nprobe))
        else:
            QM, probe = self.route(Qb, nprobe, Qh)
        q8, qs = self.quantize(Qb)
        pos, ok, est1, ncnt = self.stage1_i8(Qb, QM, probe, K, q8qs=(q8, qs), pairs=pairs)
        fb = None
        if self.FB_INGRAPH and len(Qb) >= self.FB_MIN_BATCH:
            # the recompute of the flagged rows needs only the stage-1 flags: it runs on a second stream, beside the
            # main pass's LUT and re-rank stages, and joins before its results are scattered
            main, side = torch.cuda.current_stream(), self._side_stream(Qb.device)
            side.wait_stream(main)
            with torch.cuda.stream(side):
                fb = self._fallback_ingraph(Qb, QC, QM, probe, q8, qs, ok, K, z, k)
        out = self._finish(Qb, QC, pos, ok, ncnt, K, z, k, Qh=Qh)
        if fb is None:
            return out
        main.wait_stream(side)
        return self._fallback_scatter(fb, *out)

    def _side_stream(self, dev):
        side = self.__dict__.get("_side")
        if side is None:
            side = self._side = torch.cuda.Stream(device=dev)
        return side

    def _fallback_ingraph(self, Qb, QC, QM, probe, q8, qs, ok, K, z, k):
        """The recompute of `throughput/enginei8.py:112-120` for up to FB_INGRAPH flagged rows, inside the batch's own
        graph (no host round trip): `fvs_flagged_gather` compacts the flagged rows on the GPU (stable order; unused
        slots repeat row 0) and gathers their query, routing product, probe list and query codes; they rerun with
        rho 1.0 (beta 1.5), M 65536, fp32 LUT, no delta rule.  `_fallback_scatter` writes the results back and marks
        them done.  Rows beyond the capacity stay flagged for the host."""
        B, FB, dev = len(Qb), self.FB_INGRAPH, Qb.device
        rows = torch.empty(FB, dtype=torch.int32, device=dev)
        bufs = [torch.empty((FB,) + tuple(t.shape[1:]), dtype=t.dtype, device=dev) for t in (Qb, QM, probe, q8, qs, QC)]
        srcs = [Qb, QM, probe, q8, qs, QC]
        rb = [t[0].numel() * t.element_size() for t in srcs]
        self._call("fallback_gather", self.L.fvs_flagged_gather, ptr(ok), B, FB, ptr(rows), ptr(self._nflag),
                   len(srcs), _lib.ptr_array(srcs), _lib.ptr_array(bufs), _lib.i32_array(rb))
        Qf, QMf, probef, q8f, qsf, QCf = bufs
        main_last, self._tag = self._last, "fallback_"
        try:
            pos, okf, est1, _ = self.stage1_i8(Qf, QMf, probef, K, rho_override=1.0, M_override=65536,
                                               q8qs=(q8f, qsf), small=True)
            est, sd = self.score_lut_zq(QCf, pos, self.rotated_query(Qf), None, False)
            If, rf, idsf, _ = self.refine(Qf, pos, est, sd, z, k)
        finally:
            self._last, self._tag = main_last, ""
        return rows, If, rf.long(), idsf

    def _fallback_scatter(self, fb, ok, I, reads, ids):
        rows, If, rf, idsf = fb
        self._last["fallback_rows"] = rows
        outs, res = [I, reads, ids], [If, rf, idsf]
        self._call("fallback_scatter", self.L.fvs_rows_scatter, ptr(rows), rows.numel(), len(ok), ptr(ok), 3,
                   _lib.ptr_array(res), _lib.ptr_array(outs),
                   _lib.i32_array([t[0].numel() * t.element_size() for t in outs]))
        return ok, I, reads, ids

    def _fallback(self, Qb, K, z, nprobe, k):
        """`throughput/enginei8.py:112-120`: rho 1.0 (beta 1.5), M 65536, fp32 LUT, no delta rule."""
        QC = (Qb @ self.ix.c).contiguous()
        QM, probe = self.route(Qb, nprobe)
        pos, ok, est1, _ = self.stage1_i8(Qb, QM, probe, K, rho_override=1.0, M_override=65536)
        est, sd = self.score_lut_zq(QC, pos, self.rotated_query(Qb), None, False)
        I, reads, ids, _ = self.refine(Qb, pos, est, sd, z, k)
        return I, reads.long(), ids

    def knobs(self):
        """everything a captured graph bakes in besides the call's arguments (a knob change captures anew)."""
        return (self.RHO, self.MSZ, self.DELTA, self.LUTH, self.BETA, self.SCAN, self.SMALL, self.FB_INGRAPH,
                self.FB_MIN_BATCH, getattr(self, "M", None), getattr(self, "OVER", None))

    def search(self, Qb, K, z, nprobe, k, ret_est=False):
        """`throughput/enginei8.py:96-111`: returns (I [B,k] int32, reads [B] int64, cand_ids [B,K] int32)."""
        h = self._launch(Qb, K, z, nprobe, k, 0)
        if isinstance(h, tuple):
            return h
        res = h.result()
        if h.reads_done is not None:
            h.reads_done.synchronize()
        return res

    def search_async(self, Qb, K, z, nprobe, k):
        """`search` split in two for serving loops: launches the search of Qb (one graph replay) and returns a handle
        whose `result()` waits for that search alone and returns what `search` returns.  Searches of one shape
        alternate between two graphs with their own buffers, so one search can be in flight while the host collects
        the previous one (call `result()` of a handle before launching the search after the next).  Qb must stay
        unchanged until `result()` has returned and, when the handle's `reads_done` is an event (flagged rows beyond
        the graph's recompute capacity were recomputed from Qb on the current stream), until that event."""
        key = (len(Qb), K, z, nprobe, k, self.knobs())
        slot = self._async_slot.get(key, 0)
        self._async_slot[key] = slot ^ 1
        h = self._launch(Qb, K, z, nprobe, k, slot)
        return _Done(h) if isinstance(h, tuple) else h

    def _launch(self, Qb, K, z, nprobe, k, slot):
        if not Qb.is_cuda:
            raise RuntimeError("EngineB200I8.search needs CUDA queries (the B200 library has no CPU path)")
        if K <= k:
            raise ValueError("need K > k")
        B = len(Qb)
        if B == 0:
            dev = Qb.device
            return (torch.empty(0, k, dtype=torch.int32, device=dev), torch.empty(0, dtype=torch.int64, device=dev),
                    torch.empty(0, K, dtype=torch.int32, device=dev))
        key = (B, K, z, nprobe, k, self.knobs()) + ((("slot", slot),) if slot else ())
        if key not in self.graphs:
            qs = Qb.clone()
            st = torch.cuda.Stream()
            st.wait_stream(torch.cuda.current_stream())
            with torch.cuda.stream(st):
                for _ in range(3):
                    self._gpu(qs, K, z, nprobe, k)
            torch.cuda.current_stream().wait_stream(st)
            g = torch.cuda.CUDAGraph()
            n0 = self.launches
            hok = torch.empty(B, dtype=torch.uint8, pin_memory=True)
            hst = torch.empty(2, dtype=torch.int32, pin_memory=True)
            with torch.cuda.graph(g):
                ok, I, nr, ids = self._gpu(qs, K, z, nprobe, k)
                # the results as one int32 block (reads as int64 first, then I, then the candidate ids), so that a
                # replay's results leave the graph's buffers in one copy
                packed = torch.cat([nr.view(torch.int32), I.reshape(-1), ids.reshape(-1)])
                # exactness flags, status word and flagged count land in pinned host memory inside the graph
                hok.copy_(ok.view(torch.uint8), non_blocking=True)
                hst[0:1].copy_(self.status, non_blocking=True)
                hst[1:2].copy_(self._nflag, non_blocking=True)
            self.graph_launches[key] = self.launches - n0
            self.graphs[key] = (g, qs, packed, (I.shape[1], ids.shape[1]), hok.numpy(), hst.numpy())
        g, qs, packed, dims, hok, hst = self.graphs[key]
        qs.copy_(Qb)
        g.replay()
        self.replayed_launches = getattr(self, "replayed_launches", 0) + self.graph_launches[key]
        P = packed.clone()
        done = torch.cuda.Event()
        done.record()
        return _Pending(self, Qb, K, z, nprobe, k, P, dims, hok, hst, done)

    def _collect(self, Qb, K, z, nprobe, k, P, dims, hok, hst):
        """after a replay has completed: status, flagged-row accounting and the host recompute of rows beyond the
        graph's capacity; returns the results and whether that recompute ran"""
        B = len(Qb)
        kk, KK = dims
        nr = P[:2 * B].view(torch.int64)
        I = P[2 * B:2 * B + B * kk].view(B, kk)
        ids = P[2 * B + B * kk:].view(B, KK)
        if int(hst[0]) != 0:
            self.status.zero_()                                   # the next search starts clean
            raise _lib.FvsError("stage-1 scan: a bounded device wait expired (status flag set)")
        in_graph = self.FB_INGRAPH and B >= self.FB_MIN_BATCH
        if in_graph:
            self.nbad += int(hst[1])                   # recomputed inside the graph (or below, beyond capacity)
        if not bool(hok.all()):
            bad = torch.from_numpy(np.nonzero(hok == 0)[0])
            if not in_graph:
                self.nbad += len(bad)
            a, b, c = self._fallback_graphed(Qb, bad, K, z, nprobe, k)
            badd = bad.to(Qb.device)
            I[badd], nr[badd] = a, b
            ids[badd] = c[:, :ids.shape[1]]
            return (I, nr, ids), True
        return (I, nr, ids), False

    def search_host(self, Qb, K, z, nprobe, k):
        """Latency-mode search returning the top-k ids as a host numpy array [B, k] (`EngineT.search_host`,
        `src/engine_cell.py:121-137`): the graph also copies the exactness flags, the status word and the ids into
        pinned host memory, so a search is one replay and one stream synchronisation; flagged rows are recomputed."""
        if not Qb.is_cuda:
            raise RuntimeError("EngineB200I8.search_host needs CUDA queries (the B200 library has no CPU path)")
        B = len(Qb)
        if B == 0:
            return np.empty((0, k), np.int32)
        key = ("host", B, K, z, nprobe, k, self.knobs())
        if key not in self.graphs:
            qs = Qb.clone()
            host = torch.empty((B, k + 2), dtype=torch.int32, pin_memory=True)
            st = torch.cuda.Stream()
            st.wait_stream(torch.cuda.current_stream())

            def body():
                ok, I, nr, ids = self._gpu(qs, K, z, nprobe, k)
                packed = torch.cat([ok.to(torch.int32)[:, None], self.status.expand(B, 1), I.to(torch.int32)], 1)
                host.copy_(packed, non_blocking=True)

            with torch.cuda.stream(st):
                for _ in range(3):
                    body()
            torch.cuda.current_stream().wait_stream(st)
            torch.cuda.synchronize()
            g = torch.cuda.CUDAGraph()
            n0 = self.launches
            with torch.cuda.graph(g):
                body()
            self.graph_launches[key] = self.launches - n0
            self.graphs[key] = (g, qs, host.numpy())
        g, qs, h = self.graphs[key]
        qs.copy_(Qb)
        g.replay()
        torch.cuda.current_stream().synchronize()
        self.replayed_launches = getattr(self, "replayed_launches", 0) + self.graph_launches[key]
        if h[0, 1] != 0:
            self.status.zero_()
            raise _lib.FvsError("stage-1 scan: a bounded device wait expired (status flag set)")
        out = h[:, 2:].copy()
        if not h[:, 0].all():
            bad = np.nonzero(h[:, 0] == 0)[0]
            self.nbad += len(bad)
            a, _, _ = self._fallback_graphed(Qb, torch.from_numpy(bad), K, z, nprobe, k)
            out[bad] = a.cpu().numpy()
        return out

    FALLBACK_BUCKETS = (8, 16, 32, 64, 128, 256)

    def _fallback_graphed(self, Qb, bad, K, z, nprobe, k):
        """`_fallback` on the flagged rows, replayed from a CUDA graph captured per padded batch size (the rows are
        padded with copies of the first flagged row; their results are discarded)."""
        nb = len(bad)
        bucket = next((b for b in self.FALLBACK_BUCKETS if b >= nb), None)
        if bucket is None:                                                 # very many flagged rows: eager, chunked
            outs = [self._fallback(Qb[bad[i:i + 256].to(Qb.device)], K, z, nprobe, k) for i in range(0, nb, 256)]
            return tuple(torch.cat(x) for x in zip(*outs))
        key = ("fb", bucket, K, z, nprobe, k, self.knobs())
        if key not in self.graphs:
            qs = Qb[:1].repeat(bucket, 1).contiguous()
            st = torch.cuda.Stream()
            st.wait_stream(torch.cuda.current_stream())
            with torch.cuda.stream(st):
                for _ in range(2):
                    self._fallback(qs, K, z, nprobe, k)
            torch.cuda.current_stream().wait_stream(st)
            g = torch.cuda.CUDAGraph()
            n0 = self.launches
            with torch.cuda.graph(g):
                outs = self._fallback(qs, K, z, nprobe, k)
            self.graph_launches[key] = self.launches - n0
            self.graphs[key] = (g, qs, outs)
        g, qs, (a, b, c) = self.graphs[key]
        idx = torch.cat([bad, bad[:1].repeat(bucket - nb)]).to(Qb.device)
        qs.copy_(Qb[idx])
        g.replay()
        self.replayed_launches = getattr(self, "replayed_launches", 0) + self.graph_launches[key]
        return a[:nb].clone(), b[:nb].clone(), c[:nb].clone()

    def prewarm(self, Qb, K, z, nprobe, k, buckets=None):
        """Capture the recompute graphs of every padded batch size up front (a capture costs milliseconds; a timed
        or latency-critical search should only replay)."""
        for b in buckets or self.FALLBACK_BUCKETS:
            if b <= len(Qb):
                self._fallback_graphed(Qb, torch.arange(b), K, z, nprobe, k)
        torch.cuda.synchronize()

    def search_eager(self, Qb, K, z, nprobe, k):
        """One search without graph capture (same kernels); returns the intermediates for parity tests."""
        ok, I, nr, ids = self._gpu(Qb, K, z, nprobe, k)
        return dict(ok=ok, I=I, reads=nr, ids=ids, **self._last)


class _Pending:
    """A launched search (`EngineB200I8.search_async`): result() waits for its replay (its own event, not the whole
    stream) and collects it; the rows' host recompute, when needed, runs on the caller's current stream."""

    def __init__(self, eng, Qb, K, z, nprobe, k, P, dims, hok, hst, done):
        self._args = (Qb, K, z, nprobe, k, P, dims, hok, hst)
        self._eng, self._done, self._res = eng, done, None
        self.reads_done = None   # after result(): an event once the host recompute has read Qb, or None (none ran)

    def result(self):
        if self._res is None:
            self._done.synchronize()                             # the only synchronisation
            self._res, recomputed = self._eng._collect(*self._args)
            if recomputed:
                self.reads_done = torch.cuda.Event()
                self.reads_done.record()
        return self._res


class _Done:
    """An empty batch's result, in the handle form of search_async."""

    def __init__(self, res):
        self._res = res
        self.reads_done = None

    def result(self):
        return self._res

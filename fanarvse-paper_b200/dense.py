"""Routing-free int8 stage 1 on libfanar_b200: the drop-in for the reference's `Brute` (`throughput/brute.py:41-63`).

Every query code is contracted with every row code ([B x R] x [R x N] int8 -> int32 on the tensor cores, R up to 8192
in multiples of 128, e.g. R = 1536 = the full dimension), the per-query threshold is the r-th best score of a fixed
row sample (r = round(over * K * sample fraction)), and every row scoring at least that is emitted; `search` returns
the stage-1 top-K, its estimates, the exactness flag K <= cnt <= M and the counts, as the reference does.
`EngineB200Dense` continues with the throughput engine's LUT stage 2, classification and exact re-rank.
"""
from __future__ import annotations

import numpy as np
import torch

from . import _lib
from ._lib import check, ptr
from .engine import EngineB200I8


def dense_codes(X16, mu, V, R, chunk=65536):
    """int8 row codes and fp16 row scales, the reference's expression (`throughput/brute.py:43-46`) on the GPU."""
    dev = X16.device
    N = X16.shape[0]
    Vr = V[:, :R].contiguous().float()
    Z = torch.empty(N, R, dtype=torch.int8, device=dev)
    zs = torch.empty(N, dtype=torch.float16, device=dev)
    with torch.no_grad():
        for j in range(0, N, chunk):
            z = (X16[j:j + chunk].float() - mu) @ Vr
            a = z.abs().amax(1).clamp(min=1e-12) / 127
            Z[j:j + chunk] = torch.round(z / a[:, None]).clamp(-127, 127).to(torch.int8)
            zs[j:j + chunk] = a.half()
    return Z, zs


class DenseB200:
    """`Brute` on the B200 library.  Build from the fp16 store (`DenseB200(X16, mu, V, R)`) or from existing codes
    (`DenseB200.from_codes(Z, zs, mu, V)`)."""

    def __init__(self, X16=None, mu=None, V=None, R=128, sample_every=20, Z=None, zs=None):
        self.R = R
        self.mu = mu.float().contiguous()
        self.V = V[:, :R].float().contiguous()
        if Z is None:
            Z, zs = dense_codes(X16, self.mu, V, R)
        self.Z, self.zs = Z.contiguous(), zs.to(torch.float16).contiguous()
        self.N = self.Z.shape[0]
        dev = self.Z.device
        self.sidx = torch.arange(0, self.N, sample_every, device=dev)
        self.Zs, self.zss = self.Z[self.sidx].contiguous(), self.zs[self.sidx].contiguous()
        self.frac = len(self.sidx) / self.N
        self.L = _lib.lib()
        self.status = torch.zeros(1, dtype=torch.int32, device=dev)
        self.timing = None
        self.launches = 0

    @classmethod
    def from_codes(cls, Z, zs, mu, V, sample_every=20):
        return cls(None, mu, V, Z.shape[1], sample_every, Z=Z, zs=zs)

    def _call(self, name, fn, *args):
        if self.timing is not None:
            a, b = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
            a.record()
            rc = fn(_lib.stream_handle(), *args)
            b.record()
            self.timing.setdefault(name, []).append((a, b))
        else:
            rc = fn(_lib.stream_handle(), *args)
        check(rc, name)
        self.launches += 1

    def qcode(self, Qb):
        """q8, qs (`throughput/brute.py:48-50`): fp32 projection by cuBLAS, quantisation in the library."""
        z = ((Qb - self.mu) @ self.V).contiguous()
        B = z.shape[0]
        q8 = torch.empty(B, self.R, dtype=torch.int8, device=z.device)
        qs = torch.empty(B, device=z.device)
        self._call("quantize", self.L.fvs_quantize, ptr(z), B, self.R, self.R, ptr(q8), ptr(qs))
        return q8, qs

    def scores(self, q8, qs, Z, zs):
        """dense est [B, n] (`_scan` MODE 0)."""
        B, n = q8.shape[0], Z.shape[0]
        out = torch.empty(B, n, device=Z.device)
        self._call("dense_scores", self.L.fvs_dense_scan_tc, 0, ptr(q8), ptr(qs), B, self.R, ptr(Z), ptr(zs), n, None,
                   None, None, None, 0, ptr(out), n, ptr(self.status))
        return out

    def search(self, Qb, K, over=2.0, M=None, q8qs=None):
        """`Brute.search`: returns pos [B,K] int64, est [B,K], ok [B] bool, cnt [B] int32."""
        q8, qs = q8qs if q8qs is not None else self.qcode(Qb)
        B = q8.shape[0]
        dev = q8.device
        M = M or max(4096, 8 * K)
        r = max(1, int(round(over * K * self.frac)))
        sc = self.scores(q8, qs, self.Zs, self.zss)
        r = min(r, sc.shape[1])
        t0 = torch.empty(B, device=dev)
        self._call("sample_threshold", self.L.fvs_rth_largest, ptr(sc), B, sc.shape[1], sc.shape[1], r, ptr(t0))
        cnt = torch.zeros(B, dtype=torch.int32, device=dev)
        bval = torch.empty(B, M, device=dev)
        bpos = torch.empty(B, M, dtype=torch.int32, device=dev)
        self._call("dense_scan_emit", self.L.fvs_dense_scan_tc, 1, ptr(q8), ptr(qs), B, self.R, ptr(self.Z),
                   ptr(self.zs), self.N, ptr(t0), ptr(cnt), ptr(bval), ptr(bpos), M, None, 0, ptr(self.status))
        pos = torch.empty(B, K, dtype=torch.int64, device=dev)
        est = torch.empty(B, K, device=dev)
        ok = torch.empty(B, dtype=torch.uint8, device=dev)
        self._call("select_topk", self.L.fvs_select_topk, ptr(bval), ptr(bpos), ptr(cnt), B, M, K, ptr(pos), ptr(est),
                   ptr(ok), None, 0.0, 9)
        self._last = dict(q8=q8, qs=qs, sample=sc, t0=t0, cnt=cnt, bval=bval, bpos=bpos, M=M, r=r)
        return pos, est, ok.bool(), cnt

    def check_status(self):
        if int(self.status.item()) != 0:
            self.status.zero_()
            raise _lib.FvsError("dense scan: a bounded device wait expired (status flag set)")


class EngineB200Dense(EngineB200I8):
    """Routing-free search: dense int8 stage 1 (`DenseB200.search`, positions are rows of the index's sorted order),
    then the throughput engine's LUT stage 2, classification, exact re-rank and final top-k.  Flagged queries rerun
    stage 1 with 4x the oversampling and a 65,536-entry buffer."""
    OVER = 2.0
    FB_INGRAPH = 0        # flagged rows are recomputed from the host

    def __init__(self, index, dense: DenseB200):
        super().__init__(index)
        self.dense = dense

    def _gpu(self, Qb, K, z, nprobe, k):
        QC = (Qb @ self.ix.c).contiguous()
        pos, est1, ok, cnt = self.dense.search(Qb, K, over=self.OVER, M=self.MSZ)
        self._last = dict(self.dense._last)
        I, reads, ids = self._finish_plain(Qb, QC, pos, z, k)
        return ok, I, reads, ids

    def _finish_plain(self, Qb, QC, pos, z, k):
        Zq = self.rotated_query(Qb)
        est, sd = self.score_lut_zq(QC, pos, Zq, None, self.LUTH)
        I, reads, ids, score_k = self.refine(Qb, pos, est, sd, z, k)
        self._last.update(est=est, sd=sd, Zq=Zq, score_k=score_k)
        return I, reads.long(), ids

    def _fallback(self, Qb, K, z, nprobe, k):
        QC = (Qb @ self.ix.c).contiguous()
        pos, est1, ok, cnt = self.dense.search(Qb, K, over=4 * self.OVER, M=65536)
        return self._finish_plain(Qb, QC, pos, z, k)

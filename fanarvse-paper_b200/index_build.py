"""Index construction in the reference's exact on-device layout (build time, not the query path).

The query kernels consume the dicts the reference builds (same keys, dtypes, byte layouts).  The reference builds them
with CUDA, torch and faiss (`src/rev_fanardb.py:33-61`, `src/ideas_engine2.py:23-40`, `src/engine_cell.py:8-32`,
`throughput/enginei8.py:19-27`, `throughput/s2lut.py:9-29`, `src/tiered.py:15-44`).  faiss is not available here, so the
two places it is used (the 1-D Lloyd-Max codebooks behind `tiered.DIST`/`tiered.CB`, `src/tiered.py:6-10`) are computed
from the Gaussian density directly (the Lloyd-Max quantiser of N(0,1), then the reference's own sampled MSE on its
1M samples); every other step follows the reference's recipe.  Layout produced:

s1   : c [d] f32, off (numpy int64 [NC+1]), off_t int64 [NC+1], order int32 [N] (sorted position -> original id),
       means16 [NC,d] f16, inv_mnorm [NC] f32, cen (= inv_mnorm)                              (`src/engine_cell.py:23,26-32`)
i8   : Z int8 [N,R], zs f32 [N], Vr f32 [d,R], all in sorted-position order                  (`throughput/enginei8.py:19-27`)
code : TS [(s,e,b)], rots [w x w f32], planes[t] uint8 [b,N,w/8] (bit 7-k of byte j = bit of coordinate 8j+k),
       scale/sig f16 [T,N], V f32 [d,d], deltas {b: step}, cb_uniform {b: levels}            (`src/tiered.py:29-44`)
trellis (optional): W1 f32 [d,R], tab f32 [2^L], alpha, words int32 [N,W], scale1 f16 [N]     (`src/rev_fanardb.py:33-61`)
"""
from __future__ import annotations

import math

import numpy as np
import torch

G = 32  # coordinates per allocation group (`src/tiered.py:13`)


# ----------------------------------------------------------------------------------------------- scalar quantisers
def _phi(x):
    return np.exp(-0.5 * x * x) / math.sqrt(2 * math.pi)


def _Phi(x):
    from scipy.special import ndtr
    return ndtr(x)


def lloyd_max(bits: int, iters: int = 20000):
    """Lloyd-Max levels and MSE for a standard Gaussian (what `src/tiered.py:6-10` fits with faiss 1-D k-means)."""
    n = 2 ** bits
    from scipy.special import ndtri
    lv = ndtri((np.arange(n) + 0.5) / n)
    for _ in range(iters):
        th = np.concatenate([[-np.inf], (lv[1:] + lv[:-1]) / 2, [np.inf]])
        p = _Phi(th[1:]) - _Phi(th[:-1])
        lv = (_phi(th[:-1]) - _phi(th[1:])) / np.maximum(p, 1e-300)
    return lv.astype(np.float32), _gauss_mse(lv)


def _gauss_mse(lv):
    """E[(X - Q(X))^2] for X ~ N(0,1) with nearest-level quantiser lv (sorted)."""
    lv = np.asarray(lv, np.float64)
    th = np.concatenate([[-np.inf], (lv[1:] + lv[:-1]) / 2, [np.inf]])
    a, b = th[:-1], th[1:]
    Pa, Pb = _Phi(a), _Phi(b)
    pa = np.where(np.isfinite(a), _phi(np.where(np.isfinite(a), a, 0)), 0.0)
    pb = np.where(np.isfinite(b), _phi(np.where(np.isfinite(b), b, 0)), 0.0)
    aa = np.where(np.isfinite(a), a, 0.0)
    bb = np.where(np.isfinite(b), b, 0.0)
    m0 = Pb - Pa                      # int phi
    m1 = pa - pb                      # int x phi
    m2 = (Pb - Pa) + aa * pa - bb * pb  # int x^2 phi
    return float(np.sum(m2 - 2 * lv * m1 + lv * lv * m0))


_LM_CACHE = {}


def lloyd_table(bits: int):
    """(levels, mse) of the Lloyd-Max quantiser, computed once per bit width."""
    if bits not in _LM_CACHE:
        _LM_CACHE[bits] = lloyd_max(bits)
    return _LM_CACHE[bits]


_DIST_SAMPLES = None
_DIST_CACHE = {}


def lloyd_levels_f32(bits: int):
    """The 1-D codebook of `bits` bits as the reference holds it: sorted float32 levels (`src/tiered.py:8`, faiss's 1-D
    k-means fit there; the Lloyd-Max quantiser of N(0,1) here)."""
    return np.sort(lloyd_table(bits)[0].astype(np.float32))


def dist(bits: int) -> float:
    """The reference's `tiered.DIST[bits]` (`src/tiered.py:6-9`): mean squared error of the codebook over its 1M
    standard-normal samples (numpy default_rng(1)), each sample taken to the level picked by the midpoints
    (np.searchsorted), in float32; DIST[0] = 1."""
    global _DIST_SAMPLES
    if bits == 0:
        return 1.0
    if bits not in _DIST_CACHE:
        if _DIST_SAMPLES is None:
            _DIST_SAMPLES = np.random.default_rng(1).standard_normal((1_000_000, 1)).astype(np.float32)
        g = _DIST_SAMPLES[:, 0]
        cb = lloyd_levels_f32(bits)
        th = (cb[1:] + cb[:-1]) / 2
        _DIST_CACHE[bits] = float(((g - cb[np.searchsorted(th, g)]) ** 2).mean())
    return _DIST_CACHE[bits]


def uniform_delta(bits: int) -> float:
    """Step of the MSE-best uniform quantiser on the reference's grid linspace(0.02, 2.5, 600) (`throughput/s2lut.py:9-16`),
    the MSE evaluated exactly on the Gaussian density (the reference estimates it from 2M samples of its device's
    generator: `uniform_delta_sampled`).  Used for host-built indexes."""
    mid = (2 ** bits - 1) / 2
    best = None
    for delta in np.linspace(0.02, 2.5, 600):
        m = _gauss_mse((np.arange(2 ** bits) - mid) * delta)
        if best is None or m < best[0]:
            best = (m, float(delta))
    return best[1]


def uniform_delta_sampled(bits: int, device, n: int = 2_000_000) -> float:
    """The reference's `uniform_cb` step (`throughput/s2lut.py:9-16`): n standard-normal samples from a generator of
    `device` seeded 3, levels (k - (2^b - 1)/2) * delta for each delta of linspace(0.02, 2.5, 600), samples taken to
    the level picked by the midpoints (bucketize), the first delta of least mean squared error.  On the reference's
    device (CUDA) this is its step; on the host it follows the host generator."""
    g = torch.randn(n, device=device, generator=torch.Generator(device=device).manual_seed(3))
    mid = (2 ** bits - 1) / 2
    k = torch.arange(2 ** bits, device=device).float()
    best = None
    for delta in np.linspace(0.02, 2.5, 600):
        lv = (k - mid) * delta
        th = (lv[1:] + lv[:-1]) / 2
        mse = ((g - lv[torch.bucketize(g, th)]) ** 2).mean().item()
        if best is None or mse < best[0]:
            best = (mse, float(delta))
    return best[1]


# ----------------------------------------------------------------------------------------------- building blocks
def spherical_kmeans(X16, nlist, seed=0, sample=200_000, iters=15, chunk=50_000):
    """Cell centroids as `src/ideas_engine2.py:27-33` (200k sample, random init, 15 iterations, argmax assignment)."""
    dev = X16.device
    N = X16.shape[0]
    g = torch.Generator().manual_seed(seed)
    samp = X16[torch.randperm(N, generator=g)[:min(sample, N)].to(dev)].float()
    cen = samp[torch.randperm(len(samp), generator=g)[:nlist].to(dev)].clone()
    for _ in range(iters):
        a = torch.cat([(samp[j:j + chunk] @ cen.T).argmax(1) for j in range(0, len(samp), chunk)])
        cen = torch.nn.functional.normalize(torch.zeros_like(cen).index_add_(0, a, samp) + 1e-9, dim=1)
    return cen


def assign_cells(X16, cen, chunk=100_000):
    """order (sorted position -> id) and off (cell boundaries) as `src/ideas_engine2.py:35-36`."""
    A = torch.cat([(X16[j:j + chunk].float() @ cen.T).argmax(1) for j in range(0, X16.shape[0], chunk)])
    order = torch.argsort(A, stable=True)
    off = torch.searchsorted(A[order], torch.arange(cen.shape[0] + 1, device=X16.device))
    return order, off


def cell_of_position(off_t, N):
    return torch.searchsorted(off_t, torch.arange(N, device=off_t.device), right=True) - 1


def cell_means(X16, order, off_t, chunk=65536):
    """fp32 mean of each cell (`src/engine_cell.py:11-14`)."""
    N, d = X16.shape
    NC = len(off_t) - 1
    cell = cell_of_position(off_t, N)
    means = torch.zeros(NC, d, device=X16.device)
    for j in range(0, N, chunk):
        means.index_add_(0, cell[j:j + chunk], X16[order[j:j + chunk]].float())
    means /= (off_t[1:] - off_t[:-1]).clamp(min=1).float()[:, None]
    return means


def pca_eigh(S):
    ev, V = torch.linalg.eigh(torch.cov(S.T))
    return ev.flip(0), V.flip(1).contiguous()


def build_i8_codes(X16, order, off_t, means16, V, R=256, chunk=65536):
    """int8 cell-residual codes (`throughput/enginei8.py:19-27`): Z = round(((x - m_c) @ Vr) / a), a = max|z| / 127."""
    N = len(order)
    means = means16.float()
    cell = cell_of_position(off_t, N)
    Vr = V[:, :R].contiguous()
    Z = torch.empty(N, R, dtype=torch.int8, device=X16.device)
    zs = torch.empty(N, device=X16.device)
    for j in range(0, N, chunk):
        x = X16[order[j:j + chunk]].float()
        z = (x - means[cell[j:j + chunk]]) @ Vr
        a = z.abs().amax(1).clamp(min=1e-12) / 127
        Z[j:j + chunk] = torch.round(z / a[:, None]).clamp(-127, 127).to(torch.int8)
        zs[j:j + chunk] = a
    return Z, zs, Vr


def allocate(lam, B, bmin=1, bmax=8, dist_table=None):
    """MSE water-filling bit allocation over 32-dim groups -> tiers (s, e, bits) (`src/tiered.py:19-27`).  dist_table
    (bits -> MSE) defaults to `dist`."""
    D = dist_table.__getitem__ if dist_table is not None else dist
    d = len(lam)
    NG = d // G
    lamg = lam.reshape(NG, G).sum(1).cpu().numpy()
    b = np.full(NG, bmin)
    left = B - bmin * d
    while left >= G:
        gain = [lamg[i] * (D(b[i]) - D(b[i] + 1)) if b[i] < bmax else -1 for i in range(NG)]
        i = int(np.argmax(gain))
        b[i] += 1
        left -= G
    T, st = [], 0
    for i in range(1, NG + 1):
        if i == NG or b[i] != b[st]:
            T.append((st * G, i * G, int(b[st])))
            st = i
    return T


def pack_bits(bit):
    """(n, w) bool -> (n, w/8) uint8, bit 7-k of byte j = coordinate 8j+k (`src/tiered.py:12`)."""
    sh = torch.arange(7, -1, -1, device=bit.device, dtype=torch.uint8)
    return ((bit.reshape(bit.shape[0], -1, 8).to(torch.uint8)) << sh).sum(2).to(torch.uint8)


def tiered_build(X16, order, c, V, TS, CB, seed=0, chunk=16384):
    """Tiered refinement code (`src/tiered.py:29-44`) with the codebook table CB[b] = (levels, thresholds)."""
    dev = X16.device
    N = len(order)
    gen = torch.Generator(device=dev).manual_seed(100 + seed)
    rots = [torch.linalg.qr(torch.randn(e - s, e - s, device=dev, generator=gen))[0] for s, e, _ in TS]
    planes = [torch.empty(bb, N, (e - s) // 8, dtype=torch.uint8, device=dev) for s, e, bb in TS]
    scale = torch.empty(len(TS), N, dtype=torch.float16, device=dev)
    sig = torch.empty(len(TS), N, dtype=torch.float16, device=dev)
    for j in range(0, N, chunk):
        Z = (X16[order[j:j + chunk]].float() - c) @ V
        n = len(Z)
        for t, ((s, e, bb), P) in enumerate(zip(TS, rots)):
            F = Z[:, s:e] @ P
            nf = F.norm(dim=1).clamp(min=1e-12)
            dt = e - s
            Fu = F / nf[:, None] * dt ** 0.5
            cb, th = CB[bb]
            q = torch.bucketize(Fu, th)
            Y = cb[q]
            yn = Y.norm(dim=1)
            ct = (Fu * Y).sum(1) / (yn * dt ** 0.5)
            for p in range(bb):
                planes[t][p, j:j + n] = pack_bits(((q >> (bb - 1 - p)) & 1).bool())
            scale[t, j:j + n] = (nf / (ct * yn)).half()
            sig[t, j:j + n] = (nf * torch.sqrt((1 - ct ** 2).clamp(min=0)) / (ct * (dt - 1) ** 0.5)).half()
    nbytes = sum((e - s) * bb for s, e, bb in TS) / 8 + 4 * len(TS)
    return dict(TS=TS, rots=rots, planes=planes, scale=scale, sig=sig, V=V, bytes=nbytes)


def block_rotation(code):
    """VP = V @ blockdiag(rots) (`throughput/s2lut.py:31-37`, `src/tiered_fused.py:46-52`)."""
    V = code["V"]
    d = V.shape[0]
    D = torch.zeros(d, d, device=V.device)
    for (s, e, _), P in zip(code["TS"], code["rots"]):
        D[s:e, s:e] = P
    return (V @ D).contiguous()


# ----------------------------------------------------------------------------------------------- whole index
def build_index(X16, nlist, R=256, refine_bits=None, seed=0, kmeans_sample=200_000, kmeans_iters=15,
                uniform=True, lloyd=False):
    """Build s1 + int8 codes + tiered refinement (uniform and/or Lloyd-Max codebooks) for base X16 [N,d] fp16.

    Mirrors the reference's recipe end to end: global centre c from the first 50k rows (`src/rev_fanardb.py:37`),
    spherical k-means cells (`src/ideas_engine2.py:27-36`), cell means and norms (`src/engine_cell.py:8-32`), int8 PCA
    codes (`throughput/e_brute.py:8-10`, `throughput/enginei8.py:19-27`), tiered code over the PCA basis of normalised
    residuals (`src/tiered.py:15-44`) with uniform codebooks (`throughput/s2lut.py:18-29`).
    """
    dev = X16.device
    N, d = X16.shape
    refine_bits = int(refine_bits or 2.5 * d)
    with torch.no_grad():
        c = X16[:50000].float().mean(0)
        cen = spherical_kmeans(X16, nlist, seed, kmeans_sample, kmeans_iters)
        order, off_t = assign_cells(X16, cen)
        means = cell_means(X16, order, off_t)
        means16 = means.half().contiguous()
        nrm = means16.float().norm(dim=1).clamp(min=1e-12)
        inv_mnorm = (1.0 / nrm).contiguous()
        s1 = dict(c=c, off=off_t.cpu().numpy(), off_t=off_t, order=order.to(torch.int32).contiguous(),
                  means16=means16, inv_mnorm=inv_mnorm, cen=inv_mnorm)
        # int8 stage-1 codes over the PCA basis of mean-centred rows (every 10th row, mean of the first 200k)
        mu = X16[:200000].float().mean(0)
        _, Vp = pca_eigh(X16[::10].float() - mu)
        Z, zs, Vr = build_i8_codes(X16, order, off_t, means16, Vp, R)
        i8 = dict(Z=Z, zs=zs, Vr=Vr)
        # tiered refinement: PCA of normalised residuals to c (first 50k rows)
        S = X16[:50000].float() - c
        S = S / S.norm(dim=1, keepdim=True)
        lam, V = pca_eigh(S)
        lam = lam.clamp(min=1e-12)
        TS = allocate(lam, refine_bits)
        codes = {}
        if uniform:
            # the reference's sampled step on a CUDA build device (its own device); the exact-density step on the host
            step = (lambda b: uniform_delta_sampled(b, dev)) if dev.type == "cuda" else uniform_delta
            deltas = {b: step(b) for b in sorted({bb for _, _, bb in TS})}
            CBu = {}
            for b, dl in deltas.items():
                lv = ((torch.arange(2 ** b, device=dev).float() - (2 ** b - 1) / 2) * dl)
                CBu[b] = (lv, (lv[1:] + lv[:-1]) / 2)
            cu = tiered_build(X16, order, c, V, TS, CBu, seed)
            cu["deltas"] = deltas
            cu["cb_uniform"] = {b: CBu[b][0] for b in deltas}
            cu["VP"] = block_rotation(cu)
            codes["uniform"] = cu
        if lloyd:
            CBl = {}
            for b in sorted({bb for _, _, bb in TS}):
                lv = lloyd_levels_f32(b)                          # levels and midpoints in float32 (`src/tiered.py:8-10`)
                CBl[b] = (torch.from_numpy(lv).to(dev), torch.from_numpy((lv[1:] + lv[:-1]) / 2).to(dev))
            cl = tiered_build(X16, order, c, V, TS, CBl, seed)
            cl["cbf"] = [CBl[bb][0].contiguous() for _, _, bb in TS]
            cl["VP"] = block_rotation(cl)
            codes["lloyd"] = cl
    return s1, i8, codes


# ------------------------------------------------------------------------------------------------ default engine code
def trellis_table(L: int, seed: int = 0):
    """Fixed Gaussian table of the bitshift trellis (`src/trellis.py:12-15`): T[s] = Phi^-1((perm[s] + 0.5) / 2^L),
    perm a permutation of the 2^L states drawn from numpy's default_rng(seed)."""
    from scipy.special import ndtri
    S = 1 << L
    perm = np.random.default_rng(seed).permutation(S)
    return torch.tensor(ndtri((perm + 0.5) / S), dtype=torch.float32)


def viterbi_encode(Zs, vals, L):
    """State paths [n, R] int32 of the rows of Zs (f32, CUDA) through the k = 1 trellis with emitted values vals
    (`src/trellis_scan.py:21-32`), on the GPU through the library's encoder."""
    from . import _lib
    Zs = Zs.float().contiguous()
    vals = vals.float().contiguous()
    path = torch.empty(Zs.shape, dtype=torch.int32, device=Zs.device)
    _lib.check(_lib.lib().fvs_viterbi_encode(_lib.stream_handle(), _lib.ptr(Zs), Zs.shape[0], Zs.shape[1],
                                             _lib.ptr(vals), L, _lib.ptr(path)), "viterbi_encode")
    return path


def paths_to_words(path, L):
    """Bit stream of state paths (`src/trellis_scan.py:10-18`) as int32 words [n, ceil((R+L-1)/32)]: the first state's
    L bits MSB-first, then the low bit of every later state, packed MSB-first."""
    path = path.long()
    n, r = path.shape
    nbits = r + L - 1
    W = (nbits + 31) // 32
    bits = torch.zeros(n, W * 32, dtype=torch.int64, device=path.device)
    bits[:, :L] = (path[:, :1] >> torch.arange(L - 1, -1, -1, device=path.device)) & 1
    bits[:, L:nbits] = path[:, 1:] & 1
    w = (bits.reshape(n, W, 32) << torch.arange(31, -1, -1, device=path.device)).sum(2)
    return (w & 0xFFFFFFFF).to(torch.int64).to(torch.int32)


def build_trellis(X16, s1, R=256, L=10, seed=0, chunk=65536):
    """Stage-1 trellis code of the cell residuals (the reference's default engine): rotation W1 = V[:, :R] @ Haar(R)
    over the covariance of the first 50k rows (`src/rev_fanardb.py:37-38`), step alpha from a grid by the MSE on
    Gaussian segments (`src/rev_fanardb.py:39-43`), Viterbi paths of the normalised projected residuals, words and the
    per-row scale nz / (fip * |y|) (`src/engine_cell.py:8-24`).  Needs CUDA (the encoder runs in the library).
    Returns dict(W1, tab, alpha, words, scale1, L)."""
    dev = X16.device
    if dev.type != "cuda":
        raise RuntimeError("build_trellis encodes on the GPU")
    N, d = X16.shape
    g = torch.Generator().manual_seed(seed)
    with torch.no_grad():
        S = X16[:50000].float()
        _, V = pca_eigh(S - S.mean(0))
        W1 = (V[:, :R] @ torch.linalg.qr(torch.randn(R, R, generator=g).to(dev))[0]).contiguous()
        Tt = trellis_table(L).to(dev)
        G = torch.randn(512, R, generator=g).to(dev)
        best = None
        for a in np.linspace(0.6, 1.3, 15):
            vals = (float(a) * Tt).contiguous()
            m = float(((G - vals[viterbi_encode(G, vals, L).long()]) ** 2).mean())
            if best is None or m < best[0]:
                best = (m, float(a))
        alpha = best[1]
        tab = (alpha * Tt).contiguous()
        off_t = torch.as_tensor(s1["off"], device=dev)
        cell = cell_of_position(off_t, N)
        order = s1["order"].long()
        means = s1["means16"].float()
        W = (R + L - 1 + 31) // 32
        words = torch.empty(N, W, dtype=torch.int32, device=dev)
        scale1 = torch.empty(N, dtype=torch.float16, device=dev)
        for j in range(0, N, chunk):
            Rr = X16[order[j:j + chunk]].float() - means[cell[j:j + chunk]]
            n = len(Rr)
            Z = Rr @ W1
            nz = Z.norm(dim=1).clamp(min=1e-6)
            Zs = Z / nz[:, None] * R ** 0.5
            path = viterbi_encode(Zs, tab, L).long()
            words[j:j + n] = paths_to_words(path, L)
            Y = tab[path]
            yn = Y.norm(dim=1)
            fip = (Zs * Y).sum(1) / (yn * R ** 0.5)
            scale1[j:j + n] = (nz / (fip * yn)).half()
    return dict(W1=W1, tab=tab, alpha=alpha, words=words, scale1=scale1, L=L)


def pack_records(TS, planes, scale, sig):
    """Packed refinement records, the layout of the reference's `tiered_fused.pack` (`src/tiered_fused.py:112-125`):
    [N, RB] uint8, tier t plane p at byte toff[t] + p*KB_t (KB_t = (e-s)/8), then the fp16 (scale, sigma) pair of
    every tier at soff + 4t; RB rounded up to 64 bytes.  Built on the device of the planes.  Returns
    (rec, RB, soff, toff)."""
    N = planes[0].shape[1]
    toff, o = [], 0
    for s, e, b in TS:
        toff.append(o)
        o += b * (e - s) // 8
    soff = o
    RB = (o + 4 * len(TS) + 63) // 64 * 64
    rec = torch.zeros(N, RB, dtype=torch.uint8, device=planes[0].device)
    for t, (s, e, b) in enumerate(TS):
        KB = (e - s) // 8
        rec[:, toff[t]:toff[t] + b * KB] = planes[t].permute(1, 0, 2).reshape(N, b * KB)
    ss = torch.stack([scale.to(torch.float16), sig.to(torch.float16)], 2)          # [T, N, 2]
    rec[:, soff:soff + 4 * len(TS)] = ss.permute(1, 0, 2).contiguous().view(torch.uint8).reshape(N, 4 * len(TS))
    return rec, RB, soff, toff

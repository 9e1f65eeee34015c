"""Seeded synthetic stand-ins for the reference's datasets.

The reference measures on real embedding sets (998k x 1536 DBpedia OpenAI-ada-002, 2.25M x 768 arXiv) prepared by
`src/prep_1m.py:1-20`: rows L2-normalised and stored fp16, 2000 held-out fp32 queries, exact fp32 top-10/top-100
ground truth.  Those files are not available here, so this module draws Gaussian-mixture data with the same shapes:

* C mixture components with unit-norm isotropic Gaussian centres and Dirichlet(1) weights;
* within-cluster noise with a power-law spectrum lambda_i ~ i^-alpha in a random orthonormal basis, scaled so that the
  expected cosine between a point and its centre is about 0.7 (sum(lambda) = 1/0.49 - 1);
* rows L2-normalised; the base stored fp16, the queries kept fp32 (`src/prep_1m.py:11-19`);
* queries are fresh draws of the same generator.

Everything is generated with torch on the target device from a seeded generator, so a CUDA box and a CPU box draw
different (but individually reproducible) data.
"""
from __future__ import annotations

import math
from dataclasses import dataclass

import torch


@dataclass(frozen=True)
class MixtureSpec:
    n: int
    d: int
    comps: int
    alpha: float = 0.8
    cos: float = 0.7
    nq: int = 2000
    seed: int = 0


# BASELINE configs (shapes only); the index parameters live with the engines.
CONFIGS = {
    "c1_100k_768": MixtureSpec(n=100_000, d=768, comps=256, alpha=0.8, nq=1000),
    "c2_1m_1536": MixtureSpec(n=1_000_000, d=1536, comps=1024, alpha=0.8, nq=2000),
    "c4_2m25_768": MixtureSpec(n=2_250_000, d=768, comps=2048, alpha=1.0, nq=2000),
    "c5_shard_2m_1536": MixtureSpec(n=2_000_000, d=1536, comps=4096, alpha=0.8, nq=2000),
}


class Mixture:
    """A frozen draw of the mixture parameters; `sample` produces rows."""

    def __init__(self, spec: MixtureSpec, device="cpu"):
        self.spec, self.device = spec, torch.device(device)
        g = torch.Generator(device=self.device).manual_seed(spec.seed)
        d, C = spec.d, spec.comps
        self.centres = torch.nn.functional.normalize(torch.randn(C, d, generator=g, device=self.device), dim=1)
        # Dirichlet(1) weights = normalised Exp(1) draws
        e = -torch.log(torch.rand(C, generator=g, device=self.device, dtype=torch.float64).clamp_min(1e-300))
        self.weights = (e / e.sum()).float()
        lam = torch.arange(1, d + 1, device=self.device, dtype=torch.float64) ** (-spec.alpha)
        lam = lam * ((1.0 / spec.cos ** 2 - 1.0) / lam.sum())
        self.sqrt_lam = lam.sqrt().float()
        self.basis = torch.linalg.qr(torch.randn(d, d, generator=g, device=self.device))[0].contiguous()
        self._g = g

    def sample(self, n: int, gen: torch.Generator, chunk: int = 65536) -> torch.Tensor:
        """n L2-normalised fp32 rows."""
        out = torch.empty(n, self.spec.d, device=self.device)
        for j in range(0, n, chunk):
            m = min(chunk, n - j)
            comp = torch.multinomial(self.weights, m, replacement=True, generator=gen)
            eps = (torch.randn(m, self.spec.d, generator=gen, device=self.device) * self.sqrt_lam) @ self.basis.T
            out[j:j + m] = torch.nn.functional.normalize(self.centres[comp] + eps, dim=1)
        return out


def make_dataset(spec: MixtureSpec, device="cpu", gt_k: int = 100, with_gt: bool = True, shard: int = 0):
    """Returns dict(base16 [n,d] fp16, queries [nq,d] fp32, gt [nq,gt_k] int64 or None) on `device`.

    `shard` selects an independent stream of base rows from the same mixture (row-sharded multi-GPU data: every shard
    shares the mixture and the queries)."""
    mix = Mixture(spec, device)
    gb = torch.Generator(device=mix.device).manual_seed(spec.seed + 1 + 1000 * shard)
    gq = torch.Generator(device=mix.device).manual_seed(spec.seed + 2)
    base16 = torch.empty(spec.n, spec.d, dtype=torch.float16, device=mix.device)
    for j in range(0, spec.n, 262144):
        m = min(262144, spec.n - j)
        base16[j:j + m] = mix.sample(m, gb).half()
    queries = mix.sample(spec.nq, gq)
    gt = brute_force_topk(base16, queries, gt_k) if with_gt else None
    return dict(base16=base16, queries=queries, gt=gt, spec=spec, mixture=mix)


def extra_queries(ds, n: int, seed: int):
    """n more queries from the dataset's mixture (timing batches beyond the recall batch)."""
    mix = ds["mixture"]
    return mix.sample(n, torch.Generator(device=mix.device).manual_seed(seed))


def brute_force_topk(base16: torch.Tensor, queries: torch.Tensor, k: int, chunk: int = 131072) -> torch.Tensor:
    """Exact fp32 inner-product top-k (ids, ties by lower id first), as `src/prep_1m.py:14-18` computes ground truth."""
    best_v = best_i = None
    for j in range(0, base16.shape[0], chunk):
        s = queries @ base16[j:j + chunk].float().T
        kk = min(k, s.shape[1])
        v, ix = s.topk(kk, 1)
        ix = ix + j
        if best_v is None:
            best_v, best_i = v, ix
        else:
            vv = torch.cat([best_v, v], 1)
            ii = torch.cat([best_i, ix], 1)
            t = vv.topk(min(k, vv.shape[1]), 1)
            best_v, best_i = t.values, ii.gather(1, t.indices)
    return best_i


def recall(I, gt, k: int) -> float:
    """Mean |I[:, :k] & gt[:, :k]| / k, as `src/rev_fanardb.py:134-136`."""
    I = I[:, :k].tolist()
    G = gt[:, :k].tolist()
    return float(sum(len(set(a) & set(b)) for a, b in zip(I, G)) / (k * len(I)))


def default_nlist(n: int) -> int:
    """Cells per index size as the reference chose them (`src/v19_final.py:18`): 512 at 100k, 4096 at 1M, 8192 at 2M+."""
    if n <= 150_000:
        return 512
    if n <= 1_500_000:
        return 4096
    return 8192


def spectrum_check(spec: MixtureSpec) -> float:
    """Expected cosine of a point to its centre implied by the spectrum (about spec.cos)."""
    return 1.0 / math.sqrt(1.0 + (1.0 / spec.cos ** 2 - 1.0))

"""The allocation-free pair builder (fvs_pairs_noalloc) gives the same pair lists as fvs_pairs, on two calls in a row.

It exists for callers that cannot allocate device memory (a host program binding the library through a foreign-
function interface without a CUDA allocator, or a plugin inside an application whose device memory belongs to that
application's own pool): its per-cell scratch is a device array inside the library instead of a caller buffer.
This file is collected last so that a failure here does not stop the rest of a -x run."""
import numpy as np
import pytest
import torch

from conftest import pkg

pytestmark = pytest.mark.gpu
DEV = "cuda"


def _pairs(lib, L, fn, probe, QM, mnorm, ncols, NC, with_work):
    B, npr = probe.shape
    n = B * ncols
    qid = torch.empty(n, dtype=torch.int32, device=DEV)
    qcp = torch.empty(n, device=DEV)
    coff = torch.empty(NC, dtype=torch.int32, device=DEV)
    ccnt = torch.empty(NC, dtype=torch.int32, device=DEV)
    slot = torch.empty(n, dtype=torch.int32, device=DEV)
    args = [L.stream_handle(), L.ptr(probe), B, npr, ncols, NC, L.ptr(QM), L.ptr(mnorm), L.ptr(qid), L.ptr(coff),
            L.ptr(ccnt), L.ptr(qcp), L.ptr(slot)]
    if with_work:
        args.append(L.ptr(torch.empty(NC, dtype=torch.int32, device=DEV)))
    L.check(fn(*args), "pairs")
    torch.cuda.synchronize()
    return [x.cpu().numpy() for x in (qid, coff, ccnt, qcp, slot)]


def _same(a, b, NC, ncols, B):
    qa, oa, ca, pa, sa = a
    qb, ob, cb, pb, sb = b
    np.testing.assert_array_equal(oa, ob)
    np.testing.assert_array_equal(ca, cb)
    for c in range(NC):                     # the query order inside a cell is unspecified: compare sets
        s, e = oa[c], oa[c] + ca[c]
        np.testing.assert_array_equal(np.sort(qa[s:e]), np.sort(qb[s:e]))
    # the pair behind each slot: same query and same pair constant (exact)
    np.testing.assert_array_equal(qa[sa], qb[sb])
    np.testing.assert_array_equal(pa[sa], pb[sb])
    np.testing.assert_array_equal(qa[sa], np.repeat(np.arange(B), ncols))


def test_pairs_noalloc_matches_pairs_twice():
    pkg("build").build()
    L = pkg("_lib")
    lib = L.lib()
    rng = np.random.default_rng(11)
    B, NC, npr, ncols = 257, 4096, 96, 40
    probe = torch.from_numpy(np.stack([rng.permutation(NC)[:npr] for _ in range(B)]).astype(np.int64)).to(DEV)
    QM = torch.from_numpy((rng.standard_normal((B, NC)) * 0.3).astype(np.float16)).to(DEV)
    mnorm = torch.from_numpy((rng.random(NC) + 0.5).astype(np.float32)).to(DEV)
    want = _pairs(lib, L, lib.fvs_pairs, probe, QM, mnorm, ncols, NC, True)
    for _ in range(2):   # the shared scratch keeps the previous call's contents; each call must clear what it uses
        got = _pairs(lib, L, lib.fvs_pairs_noalloc, probe, QM, mnorm, ncols, NC, False)
        _same(got, want, NC, ncols, B)


def test_pairs_noalloc_rejects_too_many_cells():
    L = pkg("_lib")
    lib = L.lib()
    d = torch.zeros(16, device=DEV)
    rc = lib.fvs_pairs_noalloc(L.stream_handle(), L.ptr(d), 1, 1, 1, 65537, L.ptr(d), None, L.ptr(d), L.ptr(d),
                               L.ptr(d), L.ptr(d), None)
    assert rc == -2

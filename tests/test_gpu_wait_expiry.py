"""Bounded waits of the tcgen05 kernels: when a pipeline wait runs out of polls, the kernel stops, drains the copies and
MMAs it issued, frees its tensor memory, sets `status` and returns; the engine raises, and the next call on the same
device runs normally (its TMEM allocation would wait forever if an earlier CTA had kept its columns).

The expiry is made on purpose by lowering the poll budget of the pipeline waits (`fvs_set_wait_limit`): 0 makes every
such wait give up at once; small budgets make some waits give up while copies and MMAs are in flight, which is the
drain path.  No fault, trap or endless wait is involved: every wait stays bounded, and the drain waits keep the full
budget."""
import numpy as np
import pytest
import torch

from conftest import pkg

pytestmark = pytest.mark.gpu
DEV = "cuda"


@pytest.fixture(scope="module")
def setup():
    pkg("build").build()
    synth, ib, eng = pkg("synth"), pkg("index_build"), pkg("engine")
    ds = synth.make_dataset(synth.MixtureSpec(n=20000, d=256, comps=16, nq=300, seed=21), DEV, gt_k=10)
    s1, i8, codes = ib.build_index(ds["base16"], 64, R=256, refine_bits=640, seed=21, kmeans_sample=20000)
    ix = eng.IndexI8(s1, i8, codes["uniform"], ds["base16"], DEV)
    return ds, ix, eng


def _engine(eng, ix, scan="cells"):
    E = eng.EngineB200I8(ix)
    E.SCAN = scan        # a tcgen05 scan (cell-major or tile-major) at every batch size
    E.SMALL = 0
    E.FB_INGRAPH = 0
    return E


def _with_limit(polls, fn):
    L = pkg("_lib")
    lib = L.lib()
    prev = lib.fvs_set_wait_limit(polls)
    try:
        return fn()
    finally:
        lib.fvs_set_wait_limit(prev)


@pytest.mark.parametrize("scan", ["cells", "tc"])
def test_expired_wait_raises_and_device_stays_usable(setup, scan):
    ds, ix, eng = setup
    L = pkg("_lib")
    Q = ds["queries"]
    K, z, nprobe, k = 40, 1.5, 16, 10
    mk = lambda e, i: _engine(e, i, scan)
    I0, nr0, ids0 = mk(eng, ix).search(Q, K, z, nprobe, k)
    torch.cuda.synchronize()
    prev = L.lib().fvs_set_wait_limit(0)
    assert L.lib().fvs_set_wait_limit(prev) == 0 and prev == 4194304          # the default, restored

    # every pipeline wait gives up at once: the search raises (graph path) and the eager scan reports through status
    E = mk(eng, ix)
    with pytest.raises(L.FvsError, match="bounded device wait"):
        _with_limit(0, lambda: E.search(Q, K, z, nprobe, k))
    E2 = mk(eng, ix)
    _with_limit(0, lambda: E2.search_eager(Q, K, z, nprobe, k))
    torch.cuda.synchronize()
    assert int(E2.status) == 1

    # small budgets: some waits give up with copies / MMAs in flight (drain path), others finish; every call returns
    for polls in (1, 4, 32, 256):
        E3 = mk(eng, ix)
        _with_limit(polls, lambda: E3.search_eager(Q, K, z, nprobe, k))
        torch.cuda.synchronize()
        assert int(E3.status) in (0, 1)

    # the same device afterwards: a normal search gives the results of before, status clear
    E4 = mk(eng, ix)
    I4, nr4, ids4 = E4.search(Q, K, z, nprobe, k)
    torch.cuda.synchronize()
    assert int(E4.status) == 0
    np.testing.assert_array_equal(I4.cpu().numpy(), I0.cpu().numpy())
    np.testing.assert_array_equal(ids4.cpu().numpy(), ids0.cpu().numpy())


def test_expired_wait_dense_scan(setup):
    ds, ix, eng = setup
    L = pkg("_lib")
    dense = pkg("dense")
    g = torch.Generator(device=DEV).manual_seed(3)
    N, R, B = 20000, 256, 200
    Z = torch.randint(-127, 128, (N, R), device=DEV, dtype=torch.int8, generator=g)
    zs = (torch.rand(N, device=DEV, generator=g) + 0.5).half()
    mu = torch.zeros(ds["queries"].shape[1], device=DEV)
    V = torch.randn(ds["queries"].shape[1], R, device=DEV, generator=g)
    D = dense.DenseB200.from_codes(Z, zs, mu, V)
    Q = ds["queries"][:B].contiguous()
    pos0, est0, ok0, cnt0 = D.search(Q, 50)
    torch.cuda.synchronize()
    D.check_status()
    _with_limit(0, lambda: D.search(Q, 50))
    torch.cuda.synchronize()
    with pytest.raises(L.FvsError, match="bounded device wait"):
        D.check_status()
    assert int(D.status) == 0                       # cleared by the raise
    pos1, est1, ok1, cnt1 = D.search(Q, 50)
    torch.cuda.synchronize()
    D.check_status()
    np.testing.assert_array_equal(pos1.cpu().numpy(), pos0.cpu().numpy())
    np.testing.assert_array_equal(cnt1.cpu().numpy(), cnt0.cpu().numpy())

"""Single-GPU check of the graphed sharded step (local search, exact scores of the winners, merge, flag sum) against
its parts run eagerly; the NCCL exchange itself runs in the multi-GPU bench (one process per GPU)."""
import numpy as np
import pytest
import torch

from conftest import pkg
from oracle import fvs_oracle as O

pytestmark = pytest.mark.gpu
DEV = "cuda"


def test_graphed_sharded_step_matches_parts():
    pkg("build").build()
    synth, ib, eng, sh = pkg("synth"), pkg("index_build"), pkg("engine"), pkg("sharded")
    ds = synth.make_dataset(synth.MixtureSpec(n=30000, d=384, comps=24, nq=300, seed=21), DEV, gt_k=10)
    s1, i8, codes = ib.build_index(ds["base16"], 96, R=256, refine_bits=960, seed=21, kmeans_sample=30000)
    ix = eng.IndexI8(s1, i8, codes["uniform"], ds["base16"], DEV)
    E = eng.EngineB200I8(ix)
    E.MSZ = 300                                   # some flagged rows (recomputed inside the graph)
    off = 5_000_000
    S = sh.ShardedSearch(E, off)
    Q = ds["queries"]
    K, z, nprobe, k = 40, 1.5, 16, 10
    Ig, Sg, reads = S.search(Q, K, z, nprobe, k)
    Ig2, Sg2, _ = S.search(Q, K, z, nprobe, k)     # replay
    I, _, _ = E.search(Q, K, z, nprobe, k)
    ex = sh.exact_scores(E, Q, I)
    want_i, want_s = O.merge_topk((I.long() + off).cpu().numpy()[None], ex.cpu().numpy()[None], k)
    np.testing.assert_array_equal(Ig.cpu().numpy(), want_i)
    np.testing.assert_array_equal(Sg.cpu().numpy(), want_s)
    np.testing.assert_array_equal(Ig2.cpu().numpy(), want_i)
    assert E.nbad > 0
    S.close()


@pytest.mark.parametrize("recompute", [False, True])
def test_sharded_search_async_matches_search(recompute):
    """two steps in flight (the two graphs of one shape alternate), then a third that replays the first graph again:
    each handle's results equal those of the synchronous search on the same queries; with `recompute`, flagged rows
    exceed the graph's recompute capacity, so result() takes the host recompute and the exchange again"""
    pkg("build").build()
    synth, ib, eng, sh = pkg("synth"), pkg("index_build"), pkg("engine"), pkg("sharded")
    ds = synth.make_dataset(synth.MixtureSpec(n=30000, d=384, comps=24, nq=300, seed=22), DEV, gt_k=10)
    s1, i8, codes = ib.build_index(ds["base16"], 96, R=256, refine_bits=960, seed=22, kmeans_sample=30000)
    ix = eng.IndexI8(s1, i8, codes["uniform"], ds["base16"], DEV)
    E = eng.EngineB200I8(ix)
    if recompute:
        E.MSZ, E.FB_INGRAPH = 300, 1
    S = sh.ShardedSearch(E, 1_000_000)
    Q = ds["queries"]
    Qs = [Q, Q.flip(0).contiguous(), Q.roll(7, 0).contiguous()]
    K, z, nprobe, k = 40, 1.5, 16, 10
    want = [S.search(q, K, z, nprobe, k) for q in Qs]
    h0 = S.search_async(Qs[0], K, z, nprobe, k)
    h1 = S.search_async(Qs[1], K, z, nprobe, k)
    r0 = h0.result()
    h2 = S.search_async(Qs[2], K, z, nprobe, k)
    for h, w in zip((h0, h1, h2), want):
        for a, b in zip(h.result(), w):
            np.testing.assert_array_equal(a.cpu().numpy(), b.cpu().numpy())
    assert r0 is h0.result()
    if recompute:
        assert S.eager_steps > 0
    S.close()

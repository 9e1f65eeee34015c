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

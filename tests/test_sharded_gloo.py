"""Row-sharded search, host side, on CPU ranks (gloo, world size 2).

The per-shard engine and the two device steps (exact scores of the local winners, cross-shard merge) are replaced by
the oracle's restatements so that the plumbing -- row offsets, the all-gather of [B, k] (global id, score) pairs, the
merge by (score desc, id asc) -- runs without a GPU.  A second test kills one rank before the exchange: the other rank
must fail with an error from the process group instead of waiting forever."""
import datetime
import os
import socket
import sys
import tempfile
import traceback

import numpy as np
import pytest
import torch
import torch.distributed as dist
import torch.multiprocessing as mp

REPO = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))


def _free_port():
    s = socket.socket()
    s.bind(("127.0.0.1", 0))
    p = s.getsockname()[1]
    s.close()
    return p


def _shard(rank, n=2500, d=256, nq=24):
    sys.path.insert(0, REPO)
    import importlib
    synth = importlib.import_module("fanarvse-paper_b200.synth")
    ib = importlib.import_module("fanarvse-paper_b200.index_build")
    import __graft_entry__ as ge
    ds = synth.make_dataset(synth.MixtureSpec(n=n, d=d, comps=8, nq=nq, seed=4), "cpu", gt_k=10, shard=rank)
    s1, i8, codes = ib.build_index(ds["base16"], 24, R=256, refine_bits=640, seed=4, kmeans_sample=n)
    return ds, ge.oracle_index(s1, i8, codes["uniform"], ds["base16"])


class _OracleLocal:
    """stands in for the shard's EngineB200I8 (same search signature and outputs)."""

    def __init__(self, oi):
        from oracle import fvs_oracle as O
        self.O, self.oi = O, oi

    def search(self, Qb, K, z, nprobe, k):
        out = self.O.search_i8(self.oi, Qb.numpy(), K, z, nprobe, k, self.O.I8Knobs, fallback=True)
        return torch.from_numpy(out["I"].astype(np.int32)), torch.from_numpy(out["reads"]), torch.from_numpy(out["ids"])


def _worker(rank, world, port, outdir, fail_rank):
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
    sys.path.insert(0, REPO)
    import importlib
    sharded = importlib.import_module("fanarvse-paper_b200.sharded")
    from oracle import fvs_oracle as O
    dist.init_process_group("gloo", rank=rank, world_size=world, timeout=datetime.timedelta(seconds=8))
    ds, oi = _shard(rank)
    n = len(oi["order"])
    H = oi["H16"].astype(np.float32)

    def exact(Qb, I):
        return torch.from_numpy((H[I.numpy()] * Qb.numpy()[:, None, :]).sum(2).astype(np.float32))

    def merge(ids_g, s_g, k):
        a, b = O.merge_topk(ids_g.numpy(), s_g.numpy(), k)
        return torch.from_numpy(a), torch.from_numpy(b)

    S = sharded.ShardedSearch(_OracleLocal(oi), rank * n, exact=exact, merge=merge)
    Q = ds["queries"]
    if rank == fail_rank:
        os._exit(3)                       # dies before its first exchange
    try:
        I, Sc, reads = S.search(Q, 40, 1.25, 10, 10)
        Il, _, _ = S.local.search(Q, 40, 1.25, 10, 10)
        Ia, Sa, _ = S.search_async(Q, 40, 1.25, 10, 10).result()      # the handle form takes the same exchange
        assert torch.equal(Ia, I) and torch.equal(Sa, Sc), "search_async differs from search"
        np.savez(os.path.join(outdir, f"r{rank}.npz"), I=I.numpy(), S=Sc.numpy(), local=Il.numpy() + rank * n,
                 local_s=exact(Q, Il).numpy())
        status = "ok"
    except Exception as e:  # a peer vanished: the collective must raise, not hang
        status = "raised: " + type(e).__name__ + ": " + str(e).splitlines()[0][:200]
    open(os.path.join(outdir, f"r{rank}.status"), "w").write(status)
    try:
        dist.destroy_process_group()
    except Exception:
        pass


def _run(world, fail_rank, timeout=240):
    outdir = tempfile.mkdtemp()
    port = _free_port()
    ctx = mp.get_context("spawn")
    ps = [ctx.Process(target=_worker, args=(r, world, port, outdir, fail_rank)) for r in range(world)]
    for p in ps:
        p.start()
    for p in ps:
        p.join(timeout)
    alive = [p for p in ps if p.is_alive()]
    for p in alive:
        p.kill()
    assert not alive, "a rank did not finish"
    return outdir, [p.exitcode for p in ps]


def test_sharded_merge_two_ranks():
    outdir, codes = _run(2, fail_rank=-1)
    assert codes == [0, 0]
    from oracle import fvs_oracle as O
    r = [np.load(os.path.join(outdir, f"r{i}.npz")) for i in range(2)]
    for i in range(2):
        assert open(os.path.join(outdir, f"r{i}.status")).read() == "ok"
    # both ranks hold the same global result ...
    np.testing.assert_array_equal(r[0]["I"], r[1]["I"])
    # ... which is the exact-score merge of the two shards' local top-k, in global ids
    ids_g = np.stack([r[0]["local"], r[1]["local"]]).astype(np.int64)
    s_g = np.stack([r[0]["local_s"], r[1]["local_s"]])
    want_i, want_s = O.merge_topk(ids_g, s_g, 10)
    np.testing.assert_array_equal(r[0]["I"], want_i)
    np.testing.assert_array_equal(r[0]["S"], want_s)
    # every result row draws from both shards' id ranges only through the merge
    assert (r[0]["I"] >= 0).all() and (r[0]["I"] < 2 * 2500).all()


def test_dead_rank_is_detected():
    outdir, codes = _run(2, fail_rank=1)
    assert codes[1] == 3
    assert codes[0] == 0
    st = open(os.path.join(outdir, "r0.status")).read()
    assert st.startswith("raised"), st


class _ShortLocal:
    """a shard engine whose local top-k has fewer than k real rows for some queries (-1 = no result)."""

    def __init__(self, I):
        self.I = I

    def search(self, Qb, K, z, nprobe, k):
        return self.I.clone(), torch.zeros(len(self.I), dtype=torch.int64), None


def _short_worker(rank, world, port, outdir):
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
    sys.path.insert(0, REPO)
    import importlib
    sharded = importlib.import_module("fanarvse-paper_b200.sharded")
    from oracle import fvs_oracle as O
    dist.init_process_group("gloo", rank=rank, world_size=world, timeout=datetime.timedelta(seconds=8))
    rng = np.random.default_rng(rank)
    B, k, n = 6, 10, 1000
    I = rng.permutation(n)[:B * k].reshape(B, k).astype(np.int32)
    I[0, 3:] = -1                       # query 0: 3 rows on this shard
    I[1, :] = -1                        # query 1: none on this shard
    if rank == 1:
        I[2, 1:] = -1                   # query 2: 1 row on shard 1
    scores = rng.standard_normal((B, k)).astype(np.float32)

    def exact(Qb, Il):
        s = torch.from_numpy(scores.copy())
        s[Il < 0] = -1e30               # as fvs_exact_scores scores a -1 id
        return s

    def merge(ids_g, s_g, k):
        a, b = O.merge_topk(ids_g.numpy(), s_g.numpy(), k)
        return torch.from_numpy(a), torch.from_numpy(b)

    S = sharded.ShardedSearch(_ShortLocal(torch.from_numpy(I)), rank * n, exact=exact, merge=merge)
    Ig, Sg, _ = S.search(torch.zeros(B, 4), 40, 1.25, 10, k)
    np.savez(os.path.join(outdir, f"s{rank}.npz"), I=Ig.numpy(), S=Sg.numpy())
    dist.destroy_process_group()


def test_no_result_rows_stay_minus_one():
    """a -1 local id ("no result") is not offset into another shard's id range: it merges as -1, after every real
    row (global ids are row_offset + local id only for real rows)."""
    outdir = tempfile.mkdtemp()
    port = _free_port()
    ctx = mp.get_context("spawn")
    ps = [ctx.Process(target=_short_worker, args=(r, 2, port, outdir)) for r in range(2)]
    for p in ps:
        p.start()
    for p in ps:
        p.join(240)
    assert [p.exitcode for p in ps] == [0, 0]
    r = np.load(os.path.join(outdir, "s0.npz"))
    I = r["I"]
    assert (I[0, :6] >= 0).all() and (I[0, 6:] == -1).all()         # 3 + 3 real rows
    assert (I[1] == -1).all()                                         # no shard has a row
    assert (I[2, :k_real(I[2])] >= 0).all() and k_real(I[2]) == 10     # shard 0 fills it
    assert ((I == -1) | ((I >= 0) & (I < 2000))).all()


def k_real(row):
    return int((row >= 0).sum())

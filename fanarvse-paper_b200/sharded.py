"""Row-sharded search over the GPUs of one node (new; the reference is single-GPU).

Every rank holds its own index over a contiguous slice of the database rows [row_offset, row_offset + n) (built by the
reference's recipe on that slice alone), searches the same query batch with the local engine, and returns its local
top-k with EXACT scores (a "sure" candidate is ranked by est + 10 without a read, `src/engine3.py:144-145`, which is
not comparable across shards, so the k winners are re-read with `fvs_exact_scores`).  One all-gather of the [B, k]
(global id, score) pairs crosses NVLink (NCCL), and `fvs_merge_topk` keeps the global top-k by (score desc, id asc).

The exchange is the only collective; every rank takes it once per batch, in the same order, also when its local search
ran the recompute path.
"""
from __future__ import annotations

import torch
import torch.distributed as dist

from . import _lib


def exact_scores(engine, Qb, I):
    """fp32 <H[id], q> for the local ids I [B, k] (int32) on the engine's device."""
    ix = engine.ix
    B, k = I.shape
    S = torch.empty(B, k, device=I.device)
    Qf = Qb.float().contiguous()
    L = _lib.lib()
    _lib.check(L.fvs_exact_scores(_lib.stream_handle(), _lib.ptr(ix.H16), ix.d, _lib.ptr(I.contiguous()), B, k,
                                  _lib.ptr(Qf), Qf.shape[1], _lib.ptr(S)), "fvs_exact_scores")
    return S


def merge_topk(ids_g, score_g, k):
    """Global top-k of [G, B, kin] (ids int64, scores f32) on the GPU."""
    G, B, kin = ids_g.shape
    I = torch.empty(B, k, dtype=torch.int64, device=ids_g.device)
    S = torch.empty(B, k, device=ids_g.device)
    L = _lib.lib()
    _lib.check(L.fvs_merge_topk(_lib.stream_handle(), _lib.ptr(ids_g.contiguous()), _lib.ptr(score_g.contiguous()), G,
                                B, kin, k, _lib.ptr(I), _lib.ptr(S)), "fvs_merge_topk")
    return I, S


class ShardedSearch:
    """search(Qb, K, z, nprobe, k) -> (I [B,k] int64 global ids, S [B,k] exact scores, reads [B] local reads).

    `local` is the rank's engine (EngineB200I8 on its shard); `row_offset` the global id of its first row.  The local
    exact-score and merge steps can be replaced (CPU tests inject the oracle's restatements).

    On CUDA ranks the whole step -- local search (with its in-graph recompute of flagged rows), exact scores of the
    local winners, the all-gather, the merge, and a sum over ranks of the rows still flagged -- is one CUDA graph per
    (B, K, z, nprobe, k); the host reads that sum once.  Only when some rank has rows beyond its in-graph recompute
    capacity do all ranks take the eager path (the rank-local recompute, then the exchange again), so every rank makes
    the same collective calls in the same order.  `close()` releases the graphs (they hold NCCL calls) and must run
    before the process group is destroyed."""

    def __init__(self, local, row_offset, group=None, exact=None, merge=None):
        self.local, self.row_offset, self.group = local, int(row_offset), group
        self.exact = exact or (lambda Qb, I: exact_scores(self.local, Qb, I))
        self.merge = merge or merge_topk
        self.graphs = {}
        self._slot = {}            # per step shape: the graph the next search_async replays (two alternate)
        self.eager_steps = 0

    def close(self):
        self.graphs.clear()
        if torch.cuda.is_available():
            torch.cuda.synchronize()

    def _exchange(self, Qb, I, k):
        """exact scores of the local top-k, one all-gather, merge (every rank, same order)."""
        S = self.exact(Qb, I)
        I = I.long()
        gid = torch.where(I < 0, torch.full_like(I, -1), I + self.row_offset)   # -1 ("no result") stays -1
        G = dist.get_world_size(self.group) if dist.is_initialized() else 1
        if G == 1:
            ids_all, s_all = gid[None], S[None]
        else:
            # one collective: (id as two int32 words, score bits) per entry, gathered into [G, B, k, 3]
            B = gid.shape[0]
            rec = torch.cat([gid.contiguous().view(torch.int32).view(B, k, 2), S.contiguous().view(torch.int32)[..., None]], 2)
            out = torch.empty((G,) + tuple(rec.shape), dtype=torch.int32, device=rec.device)
            if out.device.type == "cuda":
                dist.all_gather_into_tensor(out, rec, group=self.group)
            else:
                dist.all_gather(list(out.unbind(0)), rec, group=self.group)
            ids_all = out[..., :2].contiguous().view(torch.int64).view(G, B, k)
            s_all = out[..., 2].contiguous().view(torch.float32)
        return self.merge(ids_all, s_all, k)

    def _graph_body(self, qs, K, z, nprobe, k):
        ok, I, reads, ids = self.local._gpu(qs, K, z, nprobe, k)
        Ig, Sg = self._exchange(qs, I, k)
        left = (~ok).sum().to(torch.int32).reshape(1)
        flags = torch.cat([left, self.local.status])
        if dist.is_initialized() and dist.get_world_size(self.group) > 1:
            dist.all_reduce(flags, op=dist.ReduceOp.SUM, group=self.group)
        flags = torch.cat([flags, self.local._nflag])          # + this rank's rows flagged by its main pass
        return ok, I, reads, ids, Ig, Sg, flags

    def search(self, Qb, K, z, nprobe, k):
        if not Qb.is_cuda or not hasattr(self.local, "_gpu"):
            I, reads, _ = self.local.search(Qb, K, z, nprobe, k)
            Ig, Sg = self._exchange(Qb, I, k)
            return Ig, Sg, reads
        h = self._launch(Qb, K, z, nprobe, k, 0)
        res = h.result()
        if h.reads_done is not None:
            h.reads_done.synchronize()
        return res

    def search_async(self, Qb, K, z, nprobe, k):
        """`search` split in two, as EngineB200I8.search_async: launches the step (one graph replay; the steps of one
        shape alternate between two graphs with their own buffers) and returns a handle whose `result()` waits for
        that step alone and returns what `search` returns.  Call `result()` of a handle before launching the step
        after the next.  Every rank must launch and collect its steps in the same order: the collectives inside the
        graphs, and those of a recompute beyond the graph's capacity (run inside `result()`, on all ranks together),
        then keep one order across ranks.  Qb stays unchanged until `result()` has returned and, when the handle's
        `reads_done` is an event, until that event."""
        if not Qb.is_cuda or not hasattr(self.local, "_gpu"):
            return _ShardDone(self.search(Qb, K, z, nprobe, k))
        key = (len(Qb), K, z, nprobe, k, self.local.knobs())
        slot = self._slot.get(key, 0)
        self._slot[key] = slot ^ 1
        return self._launch(Qb, K, z, nprobe, k, slot)

    def _launch(self, Qb, K, z, nprobe, k, slot):
        key = (len(Qb), K, z, nprobe, k, self.local.knobs()) + ((("slot", slot),) if slot else ())
        if key not in self.graphs:
            qs = Qb.clone()
            st = torch.cuda.Stream()
            st.wait_stream(torch.cuda.current_stream())
            with torch.cuda.stream(st):
                for _ in range(3):
                    self._graph_body(qs, K, z, nprobe, k)
            torch.cuda.current_stream().wait_stream(st)
            torch.cuda.synchronize()
            g = torch.cuda.CUDAGraph()
            n0 = self.local.launches
            hf = torch.empty(3, dtype=torch.int32, pin_memory=True)
            with torch.cuda.graph(g):
                ok, I, reads, _, Ig, Sg, flags = self._graph_body(qs, K, z, nprobe, k)
                # the step's results as one int32 block: reads and global ids as int64 words, the merged scores, and
                # for the recompute path the local ids and exactness flags; one copy takes them out of the graph's
                # buffers.  The flags summed over ranks go to pinned host memory.
                packed = torch.cat([reads.view(torch.int32), Ig.reshape(-1).view(torch.int32),
                                    Sg.reshape(-1).view(torch.int32), I.reshape(-1).to(torch.int32),
                                    ok.to(torch.int32)])
                hf.copy_(flags, non_blocking=True)
            self.graphs[key] = (g, qs, packed, hf.numpy(), self.local.launches - n0 + 2)  # + exact, merge
        g, qs, packed, f, nl = self.graphs[key]
        qs.copy_(Qb)
        g.replay()
        self.local.replayed_launches = getattr(self.local, "replayed_launches", 0) + nl
        P = packed.clone()
        done = torch.cuda.Event()
        done.record()
        return _ShardPending(self, (Qb, K, z, nprobe, k, P, f), done)

    def _collect(self, Qb, K, z, nprobe, k, P, f):
        """after a replay has completed: status, flagged-row accounting, and the eager recompute + exchange when some
        rank has flagged rows beyond its graph's capacity (every rank takes that path together); returns the results
        and whether the recompute ran"""
        B = len(Qb)
        n = B * k
        reads = P[:2 * B].view(torch.int64)
        Ig = P[2 * B:2 * B + 2 * n].view(torch.int64).view(B, k)
        Sg = P[2 * B + 2 * n:2 * B + 3 * n].view(torch.float32).view(B, k)
        self.local.nbad += int(f[2])
        if int(f[1]) != 0:
            raise _lib.FvsError("sharded search: a bounded device wait expired on some rank (status flag set)")
        if int(f[0]) == 0:
            return (Ig, Sg, reads), False
        # some rank has flagged rows left: every rank recomputes its own (possibly none) and exchanges again
        self.eager_steps += 1
        E = self.local
        I = P[2 * B + 3 * n:2 * B + 4 * n].view(B, k)
        ok = P[2 * B + 4 * n:] != 0
        bad = torch.nonzero(~ok).flatten().cpu()
        if len(bad):
            a, b, _ = E._fallback_graphed(Qb, bad, K, z, nprobe, k)
            badd = bad.to(Qb.device)
            I[badd], reads[badd] = a.to(I.dtype), b
        Ig, Sg = self._exchange(Qb, I, k)
        return (Ig, Sg, reads), True


class _ShardPending:
    """A launched sharded step (`ShardedSearch.search_async`): result() waits for its replay (its own event) and
    collects it; `reads_done` as in EngineB200I8.search_async."""

    def __init__(self, sh, args, done):
        self._sh, self._args, self._done, self._res = sh, args, done, None
        self.reads_done = None

    def result(self):
        if self._res is None:
            self._done.synchronize()                             # the only synchronisation
            self._res, recomputed = self._sh._collect(*self._args)
            if recomputed:
                self.reads_done = torch.cuda.Event()
                self.reads_done.record()
        return self._res


class _ShardDone:
    """An eager step's result, in the handle form of search_async."""

    def __init__(self, res):
        self._res = res
        self.reads_done = None

    def result(self):
        return self._res

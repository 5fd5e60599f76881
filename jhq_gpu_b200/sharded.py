"""Database-sharded JHQ search, one process per GPU (torch.distributed).

The reference is single-GPU only. For the 100M-vector configurations the
vectors are partitioned across ranks in contiguous id ranges (shard r holds
global ids [base_r, base_r + n_r)); every rank holds the same trained
artefacts (deterministic training or jhq_set_trained), so probe choices are
identical everywhere. A batch of queries is searched on every shard; each
rank returns its local top-k with global ids, the [k] lists are all-gathered
over NCCL (NVLink), and the device kernel behind jhq_merge_shards merges the
world_size lists per query by (distance, id) — missing entries (+inf, -1).

Because each shard keeps its own exact top-ck before the residual refine,
the sharded candidate set is a superset of the single-index one (recall is at
least the single-GPU recall); it is not bit-identical to a single index.
"""
from __future__ import annotations

from typing import Callable, Optional

import numpy as np


def contiguous_shard(n: int, world: int, rank: int):
    """Global id range [lo, hi) of `rank` when n vectors are split in `world`
    contiguous blocks (sizes differ by at most one)."""
    lo = n * rank // world
    hi = n * (rank + 1) // world
    return lo, hi


def merge_topk_numpy(D: np.ndarray, I: np.ndarray, k: int):
    """Host restatement of the device merge: D, I are [nshards][nq][k];
    order by (distance, id), missing = (+inf, -1). Used by tests only."""
    ns, nq, kk = D.shape
    outD = np.full((nq, k), np.inf, np.float32)
    outI = np.full((nq, k), -1, np.int32)
    for q in range(nq):
        d = D[:, q, :].ravel()
        i = I[:, q, :].ravel()
        ok = i >= 0
        d, i = d[ok], i[ok]
        order = np.lexsort((i, d))[:k]
        outD[q, :len(order)] = d[order]
        outI[q, :len(order)] = i[order]
    return outD, outI


class ShardedSearch:
    """Search one rank's shard and merge all ranks' results.

    `local_search(q_dev, nq, k, d_dev, i_dev, stream)` runs the local search
    into device buffers (normally JHQGpuIndex.search_device); `merge` is the
    device merge (jhq_gpu_b200.merge_shards) — both injectable so the
    gather/offset logic can be exercised on CPU ranks in tests."""

    def __init__(self, local_search: Callable, id_base, group=None,
                 merge: Optional[Callable] = None):
        """id_base: int (shard = global ids [id_base, ...)) or an int32 tensor on
        the device mapping local ids to global ids (streaming adds)."""
        import torch.distributed as dist
        self.dist = dist
        self.local_search = local_search
        self.id_base = id_base
        self.group = group
        self.world = dist.get_world_size(group)
        self.merge = merge if merge is not None else device_merge

    def search(self, q, k: int, stream=None):
        """q: [nq, d] float32 tensor on this rank's device. Returns (D, I)
        tensors [nq, k] with global ids, identical on every rank."""
        import torch
        nq = q.shape[0]
        dev = q.device
        Dl = torch.empty((nq, k), dtype=torch.float32, device=dev)
        Il = torch.empty((nq, k), dtype=torch.int32, device=dev)
        st = stream if stream is not None else (torch.cuda.current_stream(dev)
                                                if dev.type == "cuda" else None)
        self.local_search(q, nq, k, Dl, Il, st)
        if isinstance(self.id_base, int):
            Il = torch.where(Il >= 0, Il + self.id_base, Il)
        else:
            Il = torch.where(Il >= 0, self.id_base[Il.clamp(min=0).long()], Il)
        Dparts = [torch.empty_like(Dl) for _ in range(self.world)]
        Iparts = [torch.empty_like(Il) for _ in range(self.world)]
        self.dist.all_gather(Dparts, Dl.contiguous(), group=self.group)
        self.dist.all_gather(Iparts, Il.contiguous(), group=self.group)
        Dall = torch.stack(Dparts)
        Iall = torch.stack(Iparts)
        D = torch.empty((nq, k), dtype=torch.float32, device=dev)
        I = torch.empty((nq, k), dtype=torch.int32, device=dev)
        self.merge(Dall, Iall, self.world, nq, k, D, I, st)
        return D, I


def device_merge(Dall, Iall, world, nq, k, D, I, stream):
    """merge callable for ShardedSearch on CUDA tensors (jhq_merge_shards)."""
    from . import merge_shards
    merge_shards(Dall.data_ptr(), Iall.data_ptr(), world, nq, k, D.data_ptr(), I.data_ptr(),
                 stream.cuda_stream if stream is not None else 0)


class PartitionedCoarseSearch(ShardedSearch):
    """ShardedSearch whose coarse step (rotation + scores against all nlist
    centroids + top-nprobe) is split by queries: rank r computes the probe lists
    of its 1/world of the queries, the lists are all-gathered, and every rank
    then scans its shard with the full set. The coarse GEMM is the same on all
    ranks (replicated centroids), so the gathered lists equal the ones each rank
    would compute alone."""

    def __init__(self, index, id_base: int, group=None):
        super().__init__(None, id_base, group)
        self.index = index

    def search(self, q, k: int, stream=None):
        import torch
        nq = q.shape[0]
        dev = q.device
        st = stream if stream is not None else torch.cuda.current_stream(dev)
        rank = self.dist.get_rank(self.group)
        np_ = self.index.params.nprobe
        per = -(-nq // self.world)
        lo, hi = min(nq, rank * per), min(nq, (rank + 1) * per)
        mine = torch.zeros((per, np_), dtype=torch.int32, device=dev)
        if hi > lo:
            self.index.probe_device(q[lo:hi].data_ptr(), hi - lo, mine.data_ptr(), st.cuda_stream)
        parts = [torch.empty_like(mine) for _ in range(self.world)]
        self.dist.all_gather(parts, mine, group=self.group)
        probes = torch.cat(parts)[:nq].contiguous()
        idx = self.index

        def local(qq, n, kk, D, I, s):
            idx.search_device_probes(qq.data_ptr(), probes.data_ptr(), n, kk, D.data_ptr(),
                                     I.data_ptr(), s.cuda_stream)
        self.local_search = local
        return super().search(q, k, st)


def index_local_search(index):
    """local_search callable for ShardedSearch backed by a JHQGpuIndex."""
    def run(q, nq, k, D, I, stream):
        index.search_device(q.data_ptr(), nq, k, D.data_ptr(), I.data_ptr(),
                            stream.cuda_stream if stream is not None else 0)
    return run

"""Sharded search: the gather / id-offset / merge logic on world_size-2 gloo
ranks (CPU), and the device merge kernel on one GPU with two shard indexes."""
import os
import socket

import numpy as np
import pytest


def _free_port():
    s = socket.socket()
    s.bind(("127.0.0.1", 0))
    p = s.getsockname()[1]
    s.close()
    return p


def _shard_world(rank, world, port, n, d, M, k, out_path):
    import torch
    import torch.distributed as dist
    from jhq_gpu_b200.sharded import ShardedSearch, contiguous_shard, merge_topk_numpy
    from oracle import Oracle
    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    dist.init_process_group("gloo", rank=rank, world_size=world)
    o = Oracle()
    rng = np.random.default_rng(0)
    x = rng.standard_normal((n, d), dtype=np.float32)
    q = rng.standard_normal((9, d), dtype=np.float32)
    P = np.linalg.qr(rng.standard_normal((d, d)))[0].astype(np.float32).T.copy().ravel()
    c1d = o.c1d(1.0, 4)
    y = o.rotate(P, x)
    codes = o.encode_primary(y, M, 8, c1d)
    res = o.kmeans1d((y - o.reconstruct(codes, d, M, 8, c1d)).ravel(), 16)
    lo, hi = contiguous_shard(n, world, rank)

    def local(qt, nq, kk, D, I, stream):                 # oracle over this rank's shard
        ys = y[lo:hi]
        pc = o.encode_primary(ys, M, 8, c1d)
        rc, co = o.encode_residual(ys, pc, M, 8, c1d, res, 4)
        Dd, Ii = o.search(o.rotate(P, qt.numpy()), M=M, B=8, Br=4, c1d=c1d, res_c1d=res,
                          codes=pc, res=rc, corr=co, assign=np.zeros(hi - lo, np.int32),
                          cents=np.zeros((1, d), np.float32), k=kk, alpha=4.0, nprobe=1)
        D.copy_(torch.from_numpy(Dd))
        I.copy_(torch.from_numpy(Ii))

    def merge(Dall, Iall, ws, nq, kk, D, I, stream):
        md, mi = merge_topk_numpy(Dall.numpy(), Iall.numpy(), kk)
        D.copy_(torch.from_numpy(md))
        I.copy_(torch.from_numpy(mi))

    ss = ShardedSearch(local, lo, merge=merge)
    D, I = ss.search(torch.from_numpy(q), k)
    if rank == 0:
        np.savez(out_path, D=D.numpy(), I=I.numpy())
    dist.barrier()
    dist.destroy_process_group()


def test_sharded_gather_merge_on_gloo_ranks(tmp_path, oracle):
    import torch.multiprocessing as mp
    from jhq_gpu_b200.sharded import contiguous_shard, merge_topk_numpy
    n, d, M, k, world = 3001, 32, 8, 7, 2
    out = str(tmp_path / "res.npz")
    mp.spawn(_shard_world, args=(world, _free_port(), n, d, M, k, out), nprocs=world, join=True)
    got = np.load(out)
    # expected: every shard searched alone (global ids), merged by (dist, id)
    o = oracle
    rng = np.random.default_rng(0)
    x = rng.standard_normal((n, d), dtype=np.float32)
    q = rng.standard_normal((9, d), dtype=np.float32)
    P = np.linalg.qr(rng.standard_normal((d, d)))[0].astype(np.float32).T.copy().ravel()
    c1d = o.c1d(1.0, 4)
    y = o.rotate(P, x)
    codes = o.encode_primary(y, M, 8, c1d)
    res = o.kmeans1d((y - o.reconstruct(codes, d, M, 8, c1d)).ravel(), 16)
    Ds, Is = [], []
    for r in range(world):
        lo, hi = contiguous_shard(n, world, r)
        pc = o.encode_primary(y[lo:hi], M, 8, c1d)
        rc, co = o.encode_residual(y[lo:hi], pc, M, 8, c1d, res, 4)
        Dd, Ii = o.search(o.rotate(P, q), M=M, B=8, Br=4, c1d=c1d, res_c1d=res, codes=pc, res=rc,
                          corr=co, assign=np.zeros(hi - lo, np.int32),
                          cents=np.zeros((1, d), np.float32), k=k, alpha=4.0, nprobe=1)
        Ds.append(Dd)
        Is.append(np.where(Ii >= 0, Ii + lo, Ii))
    eD, eI = merge_topk_numpy(np.stack(Ds), np.stack(Is), k)
    assert np.array_equal(got["I"], eI)
    assert np.array_equal(got["D"], eD)


def test_contiguous_shards_cover_ids():
    from jhq_gpu_b200.sharded import contiguous_shard
    for n in (0, 1, 7, 100_000_000):
        for w in (1, 2, 3, 8):
            spans = [contiguous_shard(n, w, r) for r in range(w)]
            assert spans[0][0] == 0 and spans[-1][1] == n
            assert all(a[1] == b[0] for a, b in zip(spans, spans[1:]))


@pytest.mark.gpu
def test_device_merge_two_shards(jhq, oracle):
    import torch
    from jhq_gpu_b200.sharded import contiguous_shard, merge_topk_numpy
    d, M, n, k = 64, 16, 6000, 10
    rng = np.random.default_rng(1)
    x = rng.standard_normal((n, d), dtype=np.float32)
    q = rng.standard_normal((77, d), dtype=np.float32)
    p = jhq.Params(M=M, nlist=16, nprobe=4, batch_size=32)
    first = jhq.JHQGpuIndex(d, p)
    first.train(x[:3000])
    t = first.get_trained()
    Ds, Is = [], []
    for r in range(2):
        lo, hi = contiguous_shard(n, 2, r)
        idx = first if r == 0 else jhq.JHQGpuIndex(d, p)
        if r:
            idx.set_trained(t["Pi"], t["c1d"], t["res_c1d"], t["cents"], t["sigma"])
        idx.add(x[lo:hi])
        Dd, Ii = idx.search(q, k)
        Ds.append(Dd)
        Is.append(np.where(Ii >= 0, Ii + lo, Ii).astype(np.int32))
    Dall = torch.from_numpy(np.stack(Ds)).cuda()
    Iall = torch.from_numpy(np.stack(Is)).cuda()
    D = torch.empty((77, k), dtype=torch.float32, device="cuda")
    I = torch.empty((77, k), dtype=torch.int32, device="cuda")
    jhq.merge_shards(Dall.data_ptr(), Iall.data_ptr(), 2, 77, k, D.data_ptr(), I.data_ptr())
    torch.cuda.synchronize()
    eD, eI = merge_topk_numpy(np.stack(Ds), np.stack(Is), k)
    assert np.array_equal(I.cpu().numpy(), eI)
    assert np.array_equal(D.cpu().numpy(), eD)


@pytest.mark.gpu
@pytest.mark.parametrize("nlist,nprobe", [(1, 1), (64, 8)])
def test_single_process_sharded_index_equals_merged_shards(nlist, nprobe):
    """jhq_sharded_*: round-robin placement over 3 shards (all on GPU 0 here),
    two add() calls, query-split coarse step, device merge == searching one
    index per shard (same artefacts, rows g % 3 == s) and merging on the host."""
    import jhq_gpu_b200 as J
    from jhq_gpu_b200.sharded import merge_topk_numpy
    rng = np.random.default_rng(51)
    d, M, S = 64, 16, 3
    x = rng.standard_normal((9001, d)).astype(np.float32)
    q = rng.standard_normal((300, d)).astype(np.float32)
    p = J.Params(M=M, nlist=nlist, nprobe=nprobe, batch_size=128)
    sh = J.JHQShardedIndex(d, p, devices=[0] * S)
    sh.train(x[:4000])
    sh.add(x[:5000])
    sh.add(x[5000:])
    assert sh.ntotal == 9001
    D, I = sh.search(q, 10)
    ref = J.JHQGpuIndex(d, p)
    ref.train(x[:4000])
    t = ref.get_trained()
    Ds, Is = [], []
    for s in range(S):
        idx = J.JHQGpuIndex(d, p)
        idx.set_trained(t["Pi"], t["c1d"], t["res_c1d"], t["cents"], t["sigma"])
        idx.add(x[s::S])
        ds, is_ = idx.search(q, 10)
        Ds.append(ds)
        Is.append(np.where(is_ >= 0, is_ * S + s, -1).astype(np.int32))
    D2, I2 = merge_topk_numpy(np.stack(Ds), np.stack(Is), 10)
    assert np.array_equal(I, I2), np.argwhere(I != I2)[:5]
    assert np.array_equal(D, D2)
    # fewer vectors than shards: empty shards take no part
    sh2 = J.JHQShardedIndex(d, p, devices=[0] * S)
    sh2.train(x[:4000])
    sh2.add(x[:2])
    D3, I3 = sh2.search(q[:5], 4)
    assert set(I3.ravel()) <= {-1, 0, 1} and (I3[:, 2:] == -1).all()
    if nlist == 1:                         # flat: both vectors are always found
        assert (np.sort(I3[:, :2], axis=1) == [0, 1]).all()


@pytest.mark.gpu
def test_single_process_sharded_index_over_gpus():
    """jhq_sharded_* over every visible GPU (peer copies between devices):
    equals one index per shard merged on the host."""
    import torch
    import jhq_gpu_b200 as J
    from jhq_gpu_b200.sharded import merge_topk_numpy
    ng = torch.cuda.device_count()
    if ng < 2:
        pytest.skip("needs 2 or more GPUs")
    S = min(ng, 8)
    rng = np.random.default_rng(61)
    d = 64
    x = rng.standard_normal((12000, d)).astype(np.float32)
    q = rng.standard_normal((500, d)).astype(np.float32)
    p = J.Params(M=16, nlist=32, nprobe=6, batch_size=128)
    sh = J.JHQShardedIndex(d, p, devices=list(range(S)))
    sh.train(x[:5000])
    sh.add(x)
    D, I = sh.search(q, 10)
    ref = J.JHQGpuIndex(d, p)
    ref.train(x[:5000])
    t = ref.get_trained()
    Ds, Is = [], []
    for s in range(S):
        idx = J.JHQGpuIndex(d, p)
        idx.set_trained(t["Pi"], t["c1d"], t["res_c1d"], t["cents"], t["sigma"])
        idx.add(x[s::S])
        ds, is_ = idx.search(q, 10)
        Ds.append(ds)
        Is.append(np.where(is_ >= 0, is_ * S + s, -1).astype(np.int32))
    D2, I2 = merge_topk_numpy(np.stack(Ds), np.stack(Is), 10)
    assert np.array_equal(I, I2) and np.array_equal(D, D2)

"""GPU parity of the CUDA path against the oracle (bit for bit) and against the
reference's own CPU code (tolerance). All calls go through the C-ABI
(libjhq_b200.so) via the jhq_gpu_b200 ctypes mirror."""
import os

import numpy as np
import pytest

pytestmark = pytest.mark.gpu


def _data(n, d, seed, scale=1.0):
    rng = np.random.default_rng(seed)
    return (rng.standard_normal((n, d)) * scale).astype(np.float32)


def _oracle_index(oracle, idx, x):
    """Everything the oracle needs, recomputed from the product's trained artefacts."""
    t = idx.get_trained()
    p = idx.params
    y = oracle.rotate(t["Pi"], x)
    codes = oracle.encode_primary(y, p.M, p.B, t["c1d"])
    rc, corr = oracle.encode_residual(y, codes, p.M, p.B, t["c1d"], t["res_c1d"], p.Br)
    norms = oracle.cent_norms(t["cents"])
    assign = oracle.assign(y, t["cents"], norms) if p.nlist > 1 else np.zeros(len(x), np.int32)
    return t, y, codes, rc, corr, assign


def _oracle_search(oracle, idx, ox, q, k):
    t, _, codes, rc, corr, assign = ox
    p = idx.params
    qr = idx.rotate_queries(q)             # the search path's own query rotation
    return oracle.search(qr, M=p.M, B=p.B, Br=p.Br, c1d=t["c1d"], res_c1d=t["res_c1d"],
                         codes=codes, res=rc, corr=corr, assign=assign, cents=t["cents"], k=k,
                         alpha=p.alpha, nprobe=min(p.nprobe, p.nlist))


def _build(jhq, d, params, x_train, x_add):
    idx = jhq.JHQGpuIndex(d, params)
    idx.train(x_train)
    idx.add(x_add)
    return idx


def _assert_same(D, I, D2, I2):
    assert np.array_equal(I, I2), np.argwhere(I != I2)[:5]
    assert np.array_equal(D, D2, equal_nan=True)


def test_rotation_bit_exact(jhq, oracle):
    x = _data(3000, 128, 1)
    idx = _build(jhq, 128, jhq.Params(M=32, nlist=1, batch_size=64), x[:1000], x[:100])
    t = idx.get_trained()
    for n in (7, 300, 3000):                       # skinny and tiled GEMM paths
        assert np.array_equal(idx.rotate(x[:n]), oracle.rotate(t["Pi"], x[:n]))


@pytest.mark.parametrize("d,M,B,Br", [(128, 32, 8, 4), (1024, 128, 8, 4), (104, 26, 8, 4),
                                      (64, 64, 8, 4), (64, 16, 4, 8), (128, 16, 8, 4)])
def test_encode_bit_exact(jhq, oracle, d, M, B, Br):
    x = _data(1500, d, 2)
    idx = _build(jhq, d, jhq.Params(M=M, B=B, Br=Br, nlist=1), x[:1000], x[:10])
    t = idx.get_trained()
    y = oracle.rotate(t["Pi"], x)
    pc, rc, co = idx.encode(y)
    opc = oracle.encode_primary(y, M, B, t["c1d"])
    orc, oco = oracle.encode_residual(y, opc, M, B, t["c1d"], t["res_c1d"], Br)
    assert np.array_equal(pc, opc)
    assert np.array_equal(rc, orc)
    assert np.array_equal(co, oco)


def test_train_matches_oracle(jhq, oracle):
    d, M, nlist = 64, 16, 16
    x = _data(4000, d, 3, 2.0)
    idx = jhq.JHQGpuIndex(d, jhq.Params(M=M, nlist=nlist, nprobe=4, ivf_iters=5))
    idx.train(x)
    t = idx.get_trained()
    s = oracle.sigma(x)
    assert t["sigma"] == s
    assert np.array_equal(t["c1d"], oracle.c1d(s, 4))
    y = oracle.rotate(t["Pi"], x)
    assert np.array_equal(t["cents"], oracle.train_ivf(y, nlist, 5))
    codes = oracle.encode_primary(y, M, 8, t["c1d"])
    yhat = oracle.reconstruct(codes, d, M, 8, t["c1d"])
    assert np.array_equal(t["res_c1d"], oracle.kmeans1d((y - yhat).ravel(), 16))


def test_add_codes_and_assignment(jhq, oracle):
    d, M = 64, 16
    x = _data(6000, d, 4)
    idx = _build(jhq, d, jhq.Params(M=M, nlist=24, nprobe=5, add_batch=1000), x[:3000], x)
    pc, rc, co, asg = idx.get_codes()
    _, _, codes, orc, oco, oasg = _oracle_index(oracle, idx, x)
    assert np.array_equal(pc, codes)
    assert np.array_equal(rc, orc)
    assert np.array_equal(co, oco)
    assert np.array_equal(asg, oasg)


@pytest.mark.parametrize("cfg", [
    dict(d=128, M=32, nlist=1, nprobe=1, n=10000, nq=100, batch=64),           # C0 shape
    dict(d=128, M=32, nlist=32, nprobe=6, n=8000, nq=130, batch=50),
    dict(d=104, M=26, nlist=16, nprobe=3, n=3000, nq=40, batch=256),            # C4 shape
    dict(d=256, M=32, nlist=1, nprobe=1, n=2500, nq=33, batch=16, B=8, Br=8),
    dict(d=64, M=64, nlist=8, nprobe=8, n=2000, nq=20, batch=7),                # Ds=1, K1D=256
    dict(d=64, M=16, nlist=1, nprobe=1, n=3000, nq=17, batch=64, B=4),          # B < 8
    dict(d=1024, M=128, nlist=1, nprobe=1, n=4000, nq=70, batch=64),            # C1 shape
])
def test_search_bit_exact_vs_oracle(jhq, oracle, cfg):
    d, n = cfg["d"], cfg["n"]
    x = _data(n, d, 5)
    q = _data(cfg["nq"], d, 6)
    p = jhq.Params(M=cfg["M"], B=cfg.get("B", 8), Br=cfg.get("Br", 4), nlist=cfg["nlist"],
                   nprobe=cfg["nprobe"], batch_size=cfg["batch"])
    idx = _build(jhq, d, p, x[:min(n, 2000)], x)
    ox = _oracle_index(oracle, idx, x)
    for k in (10, 1, 25):
        D, I = idx.search(q, k)
        D2, I2 = _oracle_search(oracle, idx, ox, q, k)
        _assert_same(D, I, D2, I2)


@pytest.mark.parametrize("order", ["list", "query"])
@pytest.mark.parametrize("cfg", [
    dict(d=128, M=32, nlist=64, nprobe=8, n=20000, nq=300, batch=100),        # C3 shape, small lists
    dict(d=104, M=26, nlist=128, nprobe=16, n=9000, nq=50, batch=64),         # C4 shape
    dict(d=64, M=16, nlist=300, nprobe=40, n=2000, nq=40, batch=13),          # many empty lists
    dict(d=32, M=8, nlist=5000, nprobe=64, n=12000, nq=30, batch=16),         # nlist > 4096 probe path
])
def test_ivf_scan_orders_bit_exact(jhq, oracle, monkeypatch, cfg, order):
    """Both SIMT scan work orders (list-major units / query-major warp items)
    give the oracle's results bit for bit (JHQ_IVF=simt: the C3 / C4 shapes
    would otherwise take the tensor-core scan)."""
    monkeypatch.setenv("JHQ_SCAN_ORDER", order)
    monkeypatch.setenv("JHQ_IVF", "simt")
    d, n = cfg["d"], cfg["n"]
    x = _data(n, d, 21)
    q = _data(cfg["nq"], d, 22)
    p = jhq.Params(M=cfg["M"], nlist=cfg["nlist"], nprobe=cfg["nprobe"], batch_size=cfg["batch"])
    idx = _build(jhq, d, p, x[:min(n, max(4000, cfg["nlist"]))], x)
    ox = _oracle_index(oracle, idx, x)
    for k in (10, 3):
        _assert_same(*idx.search(q, k), *_oracle_search(oracle, idx, ox, q, k))


def test_edge_cases(jhq, oracle):
    d, M = 32, 8
    x = _data(300, d, 7)
    idx = _build(jhq, d, jhq.Params(M=M, nlist=4, nprobe=2, batch_size=8), x, x[:5])
    ox = _oracle_index(oracle, idx, x[:5])
    q = _data(13, d, 8)
    D, I = idx.search(q, 10)                        # k > ntotal: padded with (+inf, -1)
    D2, I2 = _oracle_search(oracle, idx, ox, q, 10)
    _assert_same(D, I, D2, I2)
    assert (I[:, 5:] == -1).all() and np.isinf(D[:, 5:]).all()
    D, I = idx.search(q[:0], 10)                    # nq = 0
    assert D.shape == (0, 10)
    with pytest.raises(ValueError):
        idx.search(q, 0)
    with pytest.raises(ValueError):
        idx.search(q, 100)                          # ck = 400 > 256
    empty = jhq.JHQGpuIndex(d, jhq.Params(M=M, nlist=4))
    with pytest.raises(RuntimeError, match="train"):
        empty.add(x)
    with pytest.raises(RuntimeError, match="empty"):
        empty.search(q, 10)
    empty.train(x)
    with pytest.raises(RuntimeError, match="empty"):
        empty.search(q, 10)
    with pytest.raises(ValueError):
        jhq.JHQGpuIndex(d, jhq.Params(M=M, nlist=400)).train(x)   # n_train < nlist


def test_empty_lists_and_many_probes(jhq, oracle):
    d, M = 32, 8
    x = _data(700, d, 9)
    idx = _build(jhq, d, jhq.Params(M=M, nlist=300, nprobe=40, batch_size=32), x, x[:150])
    ox = _oracle_index(oracle, idx, x[:150])
    q = _data(50, d, 10)
    _assert_same(*idx.search(q, 10), *_oracle_search(oracle, idx, ox, q, 10))


def test_streaming_add_equals_single_add(jhq, oracle):
    d, M = 64, 16
    x = _data(5000, d, 11)
    q = _data(40, d, 12)
    p = jhq.Params(M=M, nlist=16, nprobe=4, batch_size=16, add_batch=700)
    a = _build(jhq, d, p, x[:2000], x)
    b = jhq.JHQGpuIndex(d, p)
    b.train(x[:2000])
    for s in range(0, 5000, 1234):
        b.add(x[s:s + 1234])
    assert b.ntotal == 5000
    _assert_same(*a.search(q, 10), *b.search(q, 10))


def test_device_search_equals_host_search(jhq):
    import torch
    d, M = 128, 32
    x = _data(5000, d, 13)
    q = _data(300, d, 14)
    idx = _build(jhq, d, jhq.Params(M=M, nlist=8, nprobe=3, batch_size=64), x[:2000], x)
    D, I = idx.search(q, 10)
    tq = torch.from_numpy(q).cuda()
    tD = torch.empty((300, 10), dtype=torch.float32, device="cuda")
    tI = torch.empty((300, 10), dtype=torch.int32, device="cuda")
    idx.search_device(tq.data_ptr(), 300, 10, tD.data_ptr(), tI.data_ptr(),
                      torch.cuda.current_stream().cuda_stream)
    torch.cuda.synchronize()
    _assert_same(D, I, tD.cpu().numpy(), tI.cpu().numpy())


@pytest.mark.parametrize("nlist,nprobe", [(1, 1), (40, 6)])
def test_probe_then_search_equals_search(jhq, nlist, nprobe):
    """jhq_probe_device + jhq_search_device_probes (query-partitioned coarse step
    of the sharded search) == jhq_search_device."""
    import torch
    d, M = 64, 16
    x = _data(6000, d, 31)
    q = _data(333, d, 32)
    idx = _build(jhq, d, jhq.Params(M=M, nlist=nlist, nprobe=nprobe, batch_size=100), x[:3000], x)
    tq = torch.from_numpy(q).cuda()
    s = torch.cuda.current_stream().cuda_stream
    D1 = torch.empty((333, 10), dtype=torch.float32, device="cuda")
    I1 = torch.empty((333, 10), dtype=torch.int32, device="cuda")
    idx.search_device(tq.data_ptr(), 333, 10, D1.data_ptr(), I1.data_ptr(), s)
    pr = torch.empty((333, nprobe), dtype=torch.int32, device="cuda")
    idx.probe_device(tq[:200].data_ptr(), 200, pr.data_ptr(), s)          # two partial calls
    idx.probe_device(tq[200:].data_ptr(), 133, pr[200:].data_ptr(), s)
    D2 = torch.empty_like(D1)
    I2 = torch.empty_like(I1)
    idx.search_device_probes(tq.data_ptr(), pr.data_ptr(), 333, 10, D2.data_ptr(), I2.data_ptr(), s)
    torch.cuda.synchronize()
    assert torch.equal(I1, I2) and torch.equal(D1, D2)


def test_save_load_roundtrip(jhq, tmp_path):
    d, M = 64, 16
    x = _data(3000, d, 15)
    q = _data(25, d, 16)
    idx = _build(jhq, d, jhq.Params(M=M, nlist=8, nprobe=3), x[:2000], x)
    path = str(tmp_path / "idx.jhq")
    idx.save(path)
    idx2 = jhq.JHQGpuIndex.load(path)
    assert idx2.ntotal == 3000
    _assert_same(*idx.search(q, 10), *idx2.search(q, 10))
    open(path + ".bad", "wb").write(open(path, "rb").read()[:100])
    with pytest.raises(jhq.JHQError):
        jhq.JHQGpuIndex.load(path + ".bad")


def test_set_trained_uses_reference_artefacts(jhq, oracle):
    """Identical training across builds: the product imports the reference cpu/
    artefacts (rotation, sigma, c1d, residual codebook) and its returned
    distances are checked against the reference's OWN v14 CUDA search over the
    reference's own rotated rows (oracle/_ref/libref_v14.so, fed by ref_gpu_pin)."""
    from oracle import REF_SO, RefCPU, RefGPU
    if not os.path.exists(REF_SO):
        pytest.skip("oracle/_ref not built")
    try:
        rg = RefGPU("v14")
    except FileNotFoundError:
        pytest.skip("oracle/_ref/libref_v14.so not built")
    r = RefCPU()
    d, M = 128, 32
    x = _data(3000, d, 17)
    s = r.sigma(x)
    Pi = r.rotation(d, 42)
    c1d = r.c1d(d, M, 8, s)
    y = r.apply(d, 42, x)                           # the reference's cblas rotation
    codes = r.encode(d, M, 8, s, y)
    yhat = r.reconstruct(d, M, 8, s, codes)
    res = r.kmeans1d((y - yhat).ravel(), 16)
    idx = jhq.JHQGpuIndex(d, jhq.Params(M=M, nlist=1, nprobe=1))
    idx.set_trained(Pi, c1d, res, np.zeros((1, d), np.float32), s)
    idx.add(x)
    pc, _, _, _ = idx.get_codes()
    # codes bit-exact given identical y; end-to-end mismatches only at codeword midpoints
    assert np.array_equal(idx.encode(y)[0], codes)
    assert (pc != codes).mean() < 1e-3
    q = _data(20, d, 18)
    D, I = idx.search(q, 10)
    qr = r.apply(d, 42, q)
    _, _, _, Dr, Ir = rg.pin(y, qr, M=M, c1d=c1d, res_c1d=res, cents=None, sigma=s, k=10)
    shared = 0
    for qi in range(20):
        ref = dict(zip(Ir[qi].tolist(), Dr[qi].tolist()))
        scale = float((qr[qi].astype(np.float64) ** 2).sum())
        for i, dv in zip(I[qi].tolist(), D[qi].tolist()):
            if i in ref:
                shared += 1
                assert abs(dv - ref[i]) <= 1e-4 * max(abs(dv), abs(ref[i]), scale)
    assert shared >= 0.9 * 20 * 10


def _probe_lists(jhq, d, nlist, nprobe, cents, q):
    """probe_device lists of an index whose centroids are `cents` (identity rotation)."""
    import torch
    idx = jhq.JHQGpuIndex(d, jhq.Params(M=d // 4, nlist=nlist, nprobe=nprobe, batch_size=512))
    rng = np.random.default_rng(5)
    c1d = np.sort(rng.standard_normal(idx.K1D)).astype(np.float32)
    res = np.sort(rng.standard_normal(idx.Kr) * 0.1).astype(np.float32)
    idx.set_trained(np.eye(d, dtype=np.float32), c1d, res, cents, 1.0)
    idx.add(_data(500, d, 6))
    tq = torch.from_numpy(q).cuda()
    pr = torch.empty((len(q), nprobe), dtype=torch.int32, device="cuda")
    idx.probe_device(tq.data_ptr(), len(q), pr.data_ptr(), torch.cuda.current_stream().cuda_stream)
    torch.cuda.synchronize()
    idx.synchronize()                      # raises if a tensor-core wait gave up
    return pr.cpu().numpy()


def _unit(n, d, seed):
    c = _data(n, d, seed)
    return (c / np.linalg.norm(c, axis=1, keepdims=True)).astype(np.float32)


@pytest.mark.parametrize("case", ["gauss_dups", "sphere_zero_query", "sphere_tiny_query",
                                  "wide_small_nlist", "c3_shape"])
def test_coarse_tensor_core_probes_equal_fp32(jhq, monkeypatch, case):
    """Tensor-core coarse scores + margin selection give the same probe lists as
    the fp32 SIMT GEMM + exact selection (itself bit-exact against the oracle),
    including exact ties (duplicate centroids, all-equal scores) that send rows
    through the full-rescore path."""
    if case == "gauss_dups":
        d, nlist, nprobe = 104, 5000, 64
        cents = _data(nlist, d, 40)
        cents[100:300] = cents[:200]
        q = _data(700, d, 41)
    elif case == "sphere_zero_query":
        d, nlist, nprobe = 64, 8192, 32
        cents = _unit(nlist, d, 42)
        q = np.zeros((130, d), np.float32)
    elif case == "sphere_tiny_query":
        d, nlist, nprobe = 64, 8192, 32
        cents = _unit(nlist, d, 43)
        q = _data(257, d, 44, scale=1e-4)
    elif case == "wide_small_nlist":
        d, nlist, nprobe = 1024, 300, 16
        cents = _data(nlist, d, 45)
        q = _data(129, d, 46)
    else:
        d, nlist, nprobe = 128, 65536, 64
        cents = _data(nlist, d, 47)
        q = cents[:1000] + _data(1000, d, 48, scale=0.3)
    monkeypatch.delenv("JHQ_COARSE", raising=False)
    tc = _probe_lists(jhq, d, nlist, nprobe, cents, q)
    monkeypatch.setenv("JHQ_COARSE", "simt")
    ref = _probe_lists(jhq, d, nlist, nprobe, cents, q)
    assert np.array_equal(tc, ref), np.argwhere(tc != ref)[:5]


def test_flat_pilot_pruning_is_exact(jhq, monkeypatch, tmp_path):
    """Flat index: the pilot-cluster bound plus the scan's early page exit give
    the same ids and distances as the unpruned scan (clustered data, where most
    pages exit early), also after save/load (the pilot clusters are stored)."""
    from jhq_gpu_b200 import datasets
    d, M = 256, 64
    x = datasets.normalized_mixture(20000, d, 64, seed=3, sub=1)
    q = datasets.normalized_mixture(300, d, 64, seed=3, sub=2)
    p = jhq.Params(M=M, nlist=1, nprobe=1, batch_size=64)
    monkeypatch.delenv("JHQ_PILOT", raising=False)
    a = _build(jhq, d, p, x[:6000], x)
    monkeypatch.setenv("JHQ_PILOT", "0")
    b = _build(jhq, d, p, x[:6000], x)
    Da, Ia = a.search(q, 10)
    Db, Ib = b.search(q, 10)
    _assert_same(Da, Ia, Db, Ib)
    path = str(tmp_path / "flat.jhq")
    a.save(path)
    c = jhq.JHQGpuIndex.load(path)
    _assert_same(*c.search(q, 10), Da, Ia)


@pytest.mark.parametrize("cfg", [
    dict(d=128, M=32, nlist=1, nprobe=1, n=6000, nq=70, batch=64, R=20),       # flat + pilot
    dict(d=1024, M=128, nlist=1, nprobe=1, n=3000, nq=33, batch=16, R=40),
    dict(d=104, M=26, nlist=32, nprobe=6, n=8000, nq=90, batch=50, R=25),      # IVF, C4 shape
])
def test_exact_rerank_bit_exact_vs_oracle(jhq, oracle, cfg):
    """jhq_set_rerank(R): the JHQ stage returns the best max(R, k) candidates
    (the oracle's search with k = R), re-scored by exact L2 over the stored
    vectors (oracle_rerank) — ids and distances bit for bit."""
    d, n, R = cfg["d"], cfg["n"], cfg["R"]
    x = _data(n, d, 41)
    q = _data(cfg["nq"], d, 42)
    p = jhq.Params(M=cfg["M"], nlist=cfg["nlist"], nprobe=cfg["nprobe"], batch_size=cfg["batch"])
    idx = jhq.JHQGpuIndex(d, p)
    idx.train(x[:min(n, 3000)])
    idx.set_rerank(R)
    idx.add(x[:n // 2])
    idx.add(x[n // 2:])                            # vectors kept across repeated adds
    assert idx.rerank == R
    ox = _oracle_index(oracle, idx, x)
    for k in (10, 1, R):
        D, I = idx.search(q, k)
        _, Ic = _oracle_search(oracle, idx, ox, q, max(R, k))
        D2, I2 = oracle.rerank(q, x, Ic, k)
        _assert_same(D, I, D2, I2)
    idx.set_rerank(0)                              # back to the reference's JHQ search
    _assert_same(*idx.search(q, 10), *_oracle_search(oracle, idx, ox, q, 10))


def test_exact_rerank_state_and_persistence(jhq, tmp_path):
    d = 64
    x = _data(2000, d, 43)
    q = _data(20, d, 44)
    idx = _build(jhq, d, jhq.Params(M=16, nlist=4, nprobe=2), x, x)
    with pytest.raises(RuntimeError):
        idx.set_rerank(20)                         # vectors were not kept
    with pytest.raises(ValueError):
        idx.set_rerank(-1)
    idx = jhq.JHQGpuIndex(d, jhq.Params(M=16, nlist=4, nprobe=2))
    idx.train(x)
    idx.set_rerank(30)
    idx.add(x)
    with pytest.raises(ValueError):
        idx.search(q, 70)                          # ck = 280 > 256
    path = str(tmp_path / "rr.jhq")
    idx.save(path)
    idx2 = jhq.JHQGpuIndex.load(path)
    assert idx2.rerank == 30
    _assert_same(*idx.search(q, 10), *idx2.search(q, 10))


def test_exact_rerank_reaches_recall_gate_on_c1_generator(jhq):
    """C1 generator (normalised GMM, D=1024, M=128) at 20k rows: the JHQ distance
    alone stays near the method's cap; with R = 40 the exact rerank reaches
    recall@10 >= 0.95."""
    from jhq_gpu_b200 import datasets
    x, q = datasets.make("c1", seed=0, n=20000, nq=200)
    gt = datasets.ground_truth_torch(x, q, 10)
    idx = jhq.JHQGpuIndex(1024, jhq.Params(M=128, nlist=1, nprobe=1, batch_size=64))
    idx.train(x)
    idx.set_rerank(40)
    idx.add(x)
    _, I = idx.search(q, 10)
    rec = datasets.recall_at_k(I, gt, 10)
    idx.set_rerank(0)
    _, I0 = idx.search(q, 10)
    rec0 = datasets.recall_at_k(I0, gt, 10)
    print(f"recall@10 JHQ {rec0:.4f}, with exact rerank R=40 {rec:.4f}")
    assert rec >= 0.95 and rec > rec0


@pytest.mark.parametrize("gen,d,M,nlist,nprobe", [
    ("c3", 128, 32, 2048, 32),       # uint8 generator: exact distance ties are common
    ("c4", 104, 26, 1024, 24),       # int8 Student-t generator, D=100 zero-padded to 104
])
def test_integer_generators_bit_exact_vs_oracle(jhq, oracle, gen, d, M, nlist, nprobe):
    """The C3 / C4 data generators (not i.i.d. normal) at 60k rows with nlist in the
    thousands, the tensor-core scan (two and three planes) and both SIMT scan orders: ids and distances
    equal the oracle's, and every result row is ordered by (distance, id) — the
    tie rule applied everywhere."""
    from jhq_gpu_b200 import datasets
    g = datasets.rows_c3 if gen == "c3" else datasets.rows_c4
    x = np.concatenate(list(g(0, 60000)))
    q = np.concatenate(list(g(0, 150, sub=2)))
    p = jhq.Params(M=M, nlist=nlist, nprobe=nprobe, batch_size=64)
    idx = _build(jhq, d, p, x[:20000], x)
    ox = _oracle_index(oracle, idx, x)
    D2, I2 = _oracle_search(oracle, idx, ox, q, 10)
    ties = 0
    D, I = idx.search(q, 10)                        # the default (tensor-core) scan
    _assert_same(D, I, D2, I2)
    os.environ["JHQ_IVF_TC_3PLANES"] = "1"          # tensor-core scan with the L&H plane kept
    try:
        idx.set_nprobe(nprobe)
        D, I = idx.search(q, 10)
    finally:
        del os.environ["JHQ_IVF_TC_3PLANES"]
    _assert_same(D, I, D2, I2)
    for order in ("query", "list"):                 # both SIMT orders
        os.environ["JHQ_SCAN_ORDER"] = order
        os.environ["JHQ_IVF"] = "simt"
        try:
            idx.set_nprobe(nprobe)                  # re-plan with the forced order
            D, I = idx.search(q, 10)
        finally:
            del os.environ["JHQ_SCAN_ORDER"]
            del os.environ["JHQ_IVF"]
        _assert_same(D, I, D2, I2)
    for row_d, row_i in zip(D, I):
        keys = list(zip(row_d.tolist(), row_i.tolist()))
        assert keys == sorted(keys)
        ties += sum(1 for a, b in zip(row_d[:-1], row_d[1:]) if a == b)
    print(f"{gen}: {ties} exactly tied neighbours in the returned lists")


def test_c1_generator_flat_pilot_bit_exact_vs_oracle(jhq, oracle):
    """The C1 normalised-mixture generator (where the pilot bound prunes hardest),
    flat index with pilot clusters: bit-exact against the oracle, which has no
    pruning at all."""
    from jhq_gpu_b200 import datasets
    x, q = datasets.make("c1", seed=0, n=30000, nq=128)
    idx = _build(jhq, 1024, jhq.Params(M=128, nlist=1, nprobe=1, batch_size=64), x, x)
    ox = _oracle_index(oracle, idx, x)
    for k in (10, 40):
        _assert_same(*idx.search(q, k), *_oracle_search(oracle, idx, ox, q, k))


@pytest.mark.parametrize("d,M,nlist,n", [(128, 32, 1, 20000), (64, 16, 64, 6000),
                                         (64, 16, 500, 1500), (1024, 128, 16, 8000)])
def test_device_training_equals_host_training(jhq, monkeypatch, d, M, nlist, n):
    """train() runs the IVF Lloyd update and the residual 1-D k-means on the device
    (index-order double folds after a stable sort by cluster); JHQ_TRAIN_HOST=1
    runs the host restatement of the reference's loops. Artefacts must be equal
    bit for bit, including lists left empty (reseeded, nlist 500 on 1,500 rows)."""
    x = _data(n, d, 51, 1.5)
    p = jhq.Params(M=M, nlist=nlist, nprobe=min(8, nlist), ivf_iters=6)
    a = jhq.JHQGpuIndex(d, p)
    a.train(x)
    monkeypatch.setenv("JHQ_TRAIN_HOST", "1")
    b = jhq.JHQGpuIndex(d, p)
    b.train(x)
    ta, tb = a.get_trained(), b.get_trained()
    for key in ("c1d", "res_c1d", "cents"):
        assert np.array_equal(ta[key].view(np.uint32), tb[key].view(np.uint32)), key


@pytest.mark.parametrize("cfg", [
    dict(d=128, M=32, nlist=1, nprobe=1, n=6000, Br=4),
    dict(d=104, M=26, nlist=32, nprobe=6, n=8000, Br=4),
    dict(d=64, M=8, nlist=8, nprobe=3, n=3000, Br=8),
])
def test_per_subspace_residual_codebooks_bit_exact(jhq, oracle, cfg, tmp_path):
    """M per-subspace residual codebooks: codebook m is the 1-D k-means of the
    residuals of subspace m's dims in (row, dim) order; encode, corr and the
    full search equal the oracle's per-subspace restatement bit for bit; the
    choice survives save/load."""
    d, M, n = cfg["d"], cfg["M"], cfg["n"]
    x = _data(n, d, 61)
    q = _data(45, d, 62)
    p = jhq.Params(M=M, Br=cfg["Br"], nlist=cfg["nlist"], nprobe=cfg["nprobe"], batch_size=32)
    idx = jhq.JHQGpuIndex(d, p)
    idx.set_residual_codebooks(True)
    idx.train(x[:3000])
    with pytest.raises(RuntimeError):
        idx.set_residual_codebooks(False)
    idx.add(x)
    t = idx.get_trained()
    assert t["res_c1d"].shape == (M, idx.Kr)
    Ds = d // M
    y = oracle.rotate(t["Pi"], x[:3000])
    codes = oracle.encode_primary(y, M, 8, t["c1d"])
    r = y - oracle.reconstruct(codes, d, M, 8, t["c1d"])
    for m in (0, M // 2, M - 1):
        exp = oracle.kmeans1d(r[:, m * Ds:(m + 1) * Ds].ravel(), idx.Kr)
        assert np.array_equal(t["res_c1d"][m][:len(exp)], exp), m
    yall = oracle.rotate(t["Pi"], x)
    pc, rc, co, asg = idx.get_codes()
    orc, oco = oracle.encode_residual(yall, pc, M, 8, t["c1d"], t["res_c1d"], cfg["Br"],
                                      per_sub=True)
    assert np.array_equal(rc, orc) and np.array_equal(co, oco)
    qr = idx.rotate_queries(q)
    D2, I2 = oracle.search(qr, M=M, B=8, Br=cfg["Br"], c1d=t["c1d"], res_c1d=t["res_c1d"],
                           codes=pc, res=rc, corr=co, assign=asg, cents=t["cents"], k=10,
                           alpha=4.0, nprobe=min(cfg["nprobe"], cfg["nlist"]), per_sub=True)
    _assert_same(*idx.search(q, 10), D2, I2)
    path = str(tmp_path / "ps.jhq")
    idx.save(path)
    idx2 = jhq.JHQGpuIndex.load(path)
    assert idx2.residual_per_subspace
    _assert_same(*idx2.search(q, 10), D2, I2)


@pytest.mark.parametrize("pool_pages,rerank", [(10**6, 0), (120, 0), (160, 16)])
def test_list_paging_equals_resident_index(jhq, pool_pages, rerank):
    """Out-of-core lists: codes in mapped host memory, staged per batch into a
    device page pool (several waves when the pool is small); the results equal
    the resident index's bit for bit, through the host and the device search,
    with and without the exact rerank over host-resident vectors."""
    import torch
    d, M, nlist = 64, 16, 64
    x = _data(20000, d, 71)
    q = _data(300, d, 72)
    p = jhq.Params(M=M, nlist=nlist, nprobe=6, batch_size=100, add_batch=7000)
    ref = jhq.JHQGpuIndex(d, p)
    ref.train(x[:5000])
    pg = jhq.JHQGpuIndex(d, p)
    pg.set_trained(**{kk: v for kk, v in ref.get_trained().items()})
    page_bytes = 16 * 32 + 128                               # Mp = 16: 16 bytes per slot + slot id
    pg.set_list_paging(pool_pages * page_bytes)
    if rerank:
        ref.set_rerank(rerank)
        pg.set_rerank(rerank)
    ref.add(x[:12000]); ref.add(x[12000:])
    pg.add(x[:12000]); pg.add(x[12000:])
    for k in (10, 4):
        _assert_same(*pg.search(q, k), *ref.search(q, k))
    tq = torch.from_numpy(q).cuda()
    D = torch.empty((300, 10), dtype=torch.float32, device="cuda")
    I = torch.empty((300, 10), dtype=torch.int32, device="cuda")
    pg.search_device(tq.data_ptr(), 300, 10, D.data_ptr(), I.data_ptr(),
                     torch.cuda.current_stream().cuda_stream)
    torch.cuda.synchronize()
    _assert_same(D.cpu().numpy(), I.cpu().numpy(), *ref.search(q, 10))
    if pool_pages < 1000:
        assert pg.paging_waves > 3 * 3                       # 3 batches per search, several waves each
    assert np.array_equal(pg.get_codes()[1], ref.get_codes()[1])


def test_list_paging_errors(jhq):
    d = 32
    x = _data(3000, d, 73)
    flat = jhq.JHQGpuIndex(d, jhq.Params(M=8, nlist=1))
    with pytest.raises(ValueError):
        flat.set_list_paging(1 << 20)
    idx = _build(jhq, d, jhq.Params(M=8, nlist=16, nprobe=4), x, x)
    with pytest.raises(RuntimeError):
        idx.set_list_paging(1 << 20)                         # after add
    tiny = jhq.JHQGpuIndex(d, jhq.Params(M=8, nlist=16, nprobe=16))
    tiny.train(x)
    tiny.set_list_paging(3 * (32 * 16 + 128))                # 3 pages < one query's 16 lists
    with pytest.raises(ValueError):
        tiny.add(x)                                          # largest list exceeds the pool


@pytest.mark.parametrize("refine", ["cta", "warp"])
@pytest.mark.parametrize("cfg", [
    dict(d=128, M=32, nlist=16, nprobe=4, R=0),       # short residual rows: lane per candidate
    dict(d=1024, M=128, nlist=1, nprobe=1, R=0),      # long rows: warp per candidate
    dict(d=128, M=32, nlist=16, nprobe=4, R=24),      # exact rerank, ck = 96
])
def test_refine_kernels_bit_exact(jhq, oracle, monkeypatch, refine, cfg):
    """Both refine kernels (one CTA per query / one warp per query) give the
    oracle's results bit for bit."""
    monkeypatch.setenv("JHQ_REFINE", refine)
    d = cfg["d"]
    x = _data(5000, d, 81)
    q = _data(77, d, 82)
    p = jhq.Params(M=cfg["M"], nlist=cfg["nlist"], nprobe=cfg["nprobe"], batch_size=40)
    idx = jhq.JHQGpuIndex(d, p)
    idx.train(x[:3000])
    if cfg["R"]:
        idx.set_rerank(cfg["R"])
    idx.add(x)
    ox = _oracle_index(oracle, idx, x)
    for k in (10, 3):
        D, I = idx.search(q, k)
        if cfg["R"]:
            _, Ic = _oracle_search(oracle, idx, ox, q, max(cfg["R"], k))
            D2, I2 = oracle.rerank(q, x, Ic, k)
        else:
            D2, I2 = _oracle_search(oracle, idx, ox, q, k)
        _assert_same(D, I, D2, I2)


@pytest.mark.parametrize("d,M", [(1024, 128), (128, 32), (104, 26)])
def test_tensor_core_query_rotation(jhq, monkeypatch, d, M):
    """Search-side query rotation on tcgen05 (bf16 three-term split): every output
    within 2^-15 ||x|| of the exact fp32 chain (Pi is orthonormal, so its columns
    have unit norm); JHQ_ROTATE=simt gives the exact chain itself. The end-to-end
    effect on the returned ids is measured and reported."""
    from jhq_gpu_b200 import datasets
    if d == 1024:
        x, q = datasets.make("c1", seed=0, n=12000, nq=200)
    else:
        x = _data(12000, d, 91)
        q = _data(200, d, 92)
    p = jhq.Params(M=M, nlist=1, nprobe=1, batch_size=1024)   # large batches rotate on tcgen05
    idx = _build(jhq, d, p, x[:6000], x)
    y_exact = idx.rotate(q)
    y_tc = idx.rotate_queries(q)
    bound = 2.0 ** -15 * np.linalg.norm(q.astype(np.float64), axis=1, keepdims=True)
    err = np.abs(y_tc.astype(np.float64) - y_exact)
    assert (err <= bound).all(), float((err / bound).max())
    D, I = idx.search(q, 10)
    monkeypatch.setenv("JHQ_ROTATE", "simt")
    idx2 = _build(jhq, d, p, x[:6000], x)
    assert np.array_equal(idx2.rotate_queries(q), idx2.rotate(q))
    D2, I2 = idx2.search(q, 10)
    same = np.mean([len(set(a) & set(b)) / 10.0 for a, b in zip(I, I2)])
    print(f"d={d}: max |err| / bound {float((err / bound).max()):.3f}, "
          f"returned ids shared with the fp32 rotation {same:.4f}")
    assert same >= 0.99


def test_coarse_wait_timeout_is_reported_and_the_index_recovers(jhq, monkeypatch):
    """The tcgen05 kernel's pipeline waits are bounded. A test-only setting
    (JHQ_TEST_TC_WAIT_CYCLES, read when the kernel is launched or captured)
    shortens them to zero cycles, so the first wait that is not already
    satisfied gives up: the kernel flags the error, drains its own copies and
    MMAs with full-length waits, frees its TMEM and returns. The search reports
    JHQ_ETIMEDOUT, and once the graph is captured again with the normal limit
    the next search is correct. No GPU fault is involved."""
    d = 128
    x = _data(8000, d, 95)
    q = _data(300, d, 96)
    idx = _build(jhq, d, jhq.Params(M=32, nlist=64, nprobe=8, batch_size=256), x[:4000], x)
    D0, I0 = idx.search(q, 10)
    monkeypatch.setenv("JHQ_TEST_TC_WAIT_CYCLES", "0")
    idx.set_nprobe(8)                                  # re-capture with the short waits
    with pytest.raises(jhq.JHQError) as e:
        idx.search(q, 10)
    assert e.value.code == jhq.JHQ_ETIMEDOUT
    monkeypatch.delenv("JHQ_TEST_TC_WAIT_CYCLES")
    idx.set_nprobe(8)
    _assert_same(*idx.search(q, 10), D0, I0)
    idx.check_device_status()                          # the flag was cleared by the report


@pytest.mark.parametrize("n,nq,batch,k,R", [(30000, 70, 64, 10, 0), (20000, 200, 130, 10, 0),
                                             (6000, 33, 32, 40, 0), (25000, 64, 64, 10, 24)])
def test_flat_tensor_core_scan_bit_exact(jhq, oracle, monkeypatch, n, nq, batch, k, R):
    """Flat index with 1-bit codes (C1: D=1024, M=128): the ADC scan as a tcgen05
    GEMM of the code bits with the queries, then the margin selection and exact
    rescoring — the same ids and distances as the oracle and as the SIMT scan
    (JHQ_FLAT=simt), with query blocks of 64, 128+2, and ck > the tile count."""
    from jhq_gpu_b200 import datasets
    x, q = datasets.make("c1", seed=1, n=n, nq=nq)
    p = jhq.Params(M=128, nlist=1, nprobe=1, batch_size=batch)
    idx = jhq.JHQGpuIndex(1024, p)
    idx.train(x[:min(n, 20000)])
    if R:
        idx.set_rerank(R)
    idx.add(x)
    ox = _oracle_index(oracle, idx, x)
    D, I = idx.search(q, k)
    if R:
        _, Ic = _oracle_search(oracle, idx, ox, q, max(R, k))
        D2, I2 = oracle.rerank(q, x, Ic, k)
    else:
        D2, I2 = _oracle_search(oracle, idx, ox, q, k)
    _assert_same(D, I, D2, I2)
    monkeypatch.setenv("JHQ_FLAT", "simt")
    idx.set_nprobe(1)                                  # re-plan on the SIMT scan
    _assert_same(*idx.search(q, k), D, I)


def test_flat_tensor_core_scores_within_the_bound(jhq, oracle):
    """The tensor-core flat scan's approximate scores s~ against the exact keys s*
    (the oracle's byte-LUT sums): after removing each query's constant shift,
    |s~ - s*| stays within the bound E the selection uses (the LUT-path rounding,
    the int16 quantisation residual R1 of the query and the roundings forming
    s~). Measured on tcgen05 integer arithmetic, and reported."""
    from jhq_gpu_b200 import datasets
    x, q = datasets.make("c1", seed=2, n=20000, nq=8)
    idx = _build(jhq, 1024, jhq.Params(M=128, nlist=1, nprobe=1, batch_size=64), x, x)
    s_tc = idx.debug_flat_scores(q).astype(np.float64)
    t = idx.get_trained()
    pc, _, _, _ = idx.get_codes()
    qr = idx.rotate_queries(q)
    c0, c1 = float(t["c1d"][0]), float(t["c1d"][1])
    worst = 0.0
    for i in range(len(q)):
        lut = oracle.byte_lut(qr[i], 128, 8, t["c1d"])
        s_ex = lut[np.arange(128)[None, :], pc].sum(1, dtype=np.float64)
        x64 = qr[i].astype(np.float64)
        V = ((np.abs(x64) + max(abs(c0), abs(c1))) ** 2).sum()
        L1 = np.abs(x64).sum()
        S0 = ((x64 - c0) ** 2).sum()
        # the kernel's quantisation: Q = rint(q / s), s = max|q| / 32000 (fp32)
        sc = np.float32(np.abs(qr[i]).max()) / np.float32(32000.0)
        Q = np.clip(np.rint(qr[i] / sc), -32000, 32000).astype(np.float64)
        R1 = np.abs(x64 - float(sc) * Q).sum()
        G = L1 + R1
        u = 2.0 ** -24
        E = 1.1 * (V * (2 * 128 + 16) * u + abs(c1 * c1 - c0 * c0) * 1024 * u +
                   2 * abs(c1 - c0) * (R1 + 2 * u * G) +
                   2 * u * (S0 + abs(c1 * c1 - c0 * c0) * 1024 + 2 * abs(c1 - c0) * G))
        diff = s_tc[i] - s_ex
        dev = np.abs(diff - np.median(diff)).max()
        print(f"query {i}: max |s~ - s* - shift| {dev:.3e}, E {E:.3e}, ratio {dev / E:.3f}, "
              f"shift {np.median(diff):.3e}, spread of s* {s_ex.std():.3e}")
        worst = max(worst, dev / E)
    assert worst <= 1.0


@pytest.mark.parametrize("gen,d,M,nlist,nprobe,nq,batch,k,R", [
    ("c3", 128, 32, 2048, 32, 150, 64, 10, 0),     # ragged last batch (150 = 2 x 64 + 22)
    ("c4", 104, 26, 1024, 24, 130, 128, 10, 0),    # d = 104 padded to 128 inside the planes
    ("c3", 128, 32, 4096, 8, 96, 96, 40, 0),       # ck = 160 > the tiles of most queries
    ("c3", 128, 32, 512, 16, 64, 64, 10, 24),      # exact rerank behind the scan
])
def test_ivf_tensor_core_scan_bit_exact(jhq, oracle, monkeypatch, gen, d, M, nlist, nprobe, nq,
                                        batch, k, R):
    """IVF with 2-bit-per-dimension codes (C3 uint8 / C4 int8 generators): the
    two-pass tensor-core scan (per-query tile minima of the int8 GEMM of the code
    bit planes with the queries, then exact rescoring of the tiles within the
    margin) returns the oracle's ids and distances, and the query-major SIMT
    scan's (JHQ_IVF=simt), bit for bit."""
    from jhq_gpu_b200 import datasets
    g = datasets.rows_c3 if gen == "c3" else datasets.rows_c4
    x = np.concatenate(list(g(0, 40000)))
    q = np.concatenate(list(g(0, nq, sub=2)))
    p = jhq.Params(M=M, nlist=nlist, nprobe=nprobe, batch_size=batch)
    idx = jhq.JHQGpuIndex(d, p)
    idx.train(x[:20000])
    if R:
        idx.set_rerank(R)
    idx.add(x)
    ox = _oracle_index(oracle, idx, x)
    D, I = idx.search(q, k)
    if R:
        _, Ic = _oracle_search(oracle, idx, ox, q, max(R, k))
        D2, I2 = oracle.rerank(q, x, Ic, k)
    else:
        D2, I2 = _oracle_search(oracle, idx, ox, q, k)
    _assert_same(D, I, D2, I2)
    monkeypatch.setenv("JHQ_IVF", "simt")
    idx.set_nprobe(nprobe)                          # re-plan on the SIMT scan
    _assert_same(*idx.search(q, k), D, I)

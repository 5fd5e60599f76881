"""Host-side logic of the product that needs no GPU: the C-ABI library loads and
exports every symbol include/jhq.h declares; the CPU training steps match the
reference's cpu/ (golden vectors); parameter validation mirrors the reference."""
import os
import re

import numpy as np
import pytest

from conftest import ROOT


def _declared_symbols():
    src = open(os.path.join(ROOT, "include", "jhq.h")).read()
    src = re.sub(r"/\*.*?\*/", "", src, flags=re.S)
    return sorted(set(re.findall(r"\b(jhq_[a-z0-9_]+)\s*\(", src)))


def test_library_exports_every_declared_symbol(jhq):
    L = jhq.load_library()
    declared = _declared_symbols()
    assert len(declared) >= 20
    for name in declared:
        assert hasattr(L, name), name
    assert sorted(jhq.EXPORTED) == declared


def test_rotation_matches_reference_lapack(jhq, golden):
    for d in (16, 104):
        P = jhq.jl_rotation(d, 42)
        R = golden[f"pi_d{d}"]
        np.testing.assert_allclose(P, R, atol=5e-6)      # same QR convention, fp rounding only
        Q = P.reshape(d, d).astype(np.float64)
        np.testing.assert_allclose(Q @ Q.T, np.eye(d), atol=1e-5)


def test_training_primitives_bit_exact(jhq, golden):
    s = jhq.estimate_sigma(golden["sigma_x"])
    assert np.float32(s) == golden["sigma"]
    for M, K in ((2, 2), (4, 4), (8, 16), (16, 256)):
        assert np.array_equal(jhq.lloyd_max_c1d(s, K), golden[f"c1d_d16_M{M}"])
    assert np.array_equal(jhq.kmeans_1d(golden["km_vals"], 16), golden["km_c16"])
    assert np.array_equal(jhq.kmeans_1d(golden["km_vals"][:3], 4), golden["km_c4_small"])


@pytest.mark.parametrize("d,kw,msg", [
    (0, {}, "d must be positive"),
    (128, dict(M=0), "M must be positive"),
    (128, dict(M=33), "divisible by M"),
    (128, dict(M=32, B=7), "divisible by Ds"),
    (128, dict(M=128, B=9), "B must be <= 8"),
    (128, dict(M=32, Br=5), "Br must be 4 or 8"),
    (128, dict(M=32, nlist=0), "nlist"),
    (128, dict(M=32, nprobe=0), "nprobe"),
    (128, dict(M=32, ivf_iters=0), "ivf_iters"),
    (128, dict(M=32, batch_size=0), "batch_size"),
    (128, dict(M=32, add_batch=0), "add_batch"),
    (128, dict(M=32, alpha=0.0), "alpha"),
    (4096, dict(M=2048, B=8), "M too large"),
    (1024, dict(M=1024, B=8), "M too large"),
])
def test_param_validation_like_reference(jhq, d, kw, msg):
    """JHQGpuIndex ctor throws std::invalid_argument (jhq_gpu_index.cu:110-121)."""
    with pytest.raises(ValueError, match=msg):
        jhq.JHQGpuIndex(d, jhq.Params(**kw))


def test_null_and_error_paths(jhq):
    L = jhq.load_library()
    assert L.jhq_index_destroy(None) == 0
    assert L.jhq_params_default(None) == jhq.JHQ_EINVAL
    p = jhq.CParams()
    assert L.jhq_params_default(p) == 0
    assert (p.M, p.B, p.Br, p.nlist, p.nprobe, p.batch_size, p.seed, p.add_batch) == \
        (96, 8, 4, 1024, 8, 256, 42, 65536)
    assert abs(p.alpha - 4.0) < 1e-7
    assert L.jhq_search(None, None, 0, 10, None, None) == jhq.JHQ_EINVAL
    assert b"null index" in L.jhq_last_error()
    assert L.jhq_load(b"/nonexistent/file.jhq", -1, None) == jhq.JHQ_EINVAL
    # sharded index: argument errors before any device is touched
    import ctypes as C
    h = C.c_void_p()
    assert L.jhq_sharded_create(64, None, 0, None, C.byref(h)) == jhq.JHQ_EINVAL
    assert L.jhq_sharded_create(64, None, 65, None, C.byref(h)) == jhq.JHQ_EINVAL
    assert L.jhq_sharded_destroy(None) == 0
    assert L.jhq_sharded_search(None, None, 0, 10, None, None) == jhq.JHQ_EINVAL
    assert L.jhq_sharded_ntotal(None) == -1


@pytest.mark.parametrize("d,M,nlist", [(128, 32, 1), (1024, 128, 1), (1024, 128, 1024),
                                       (128, 32, 65536), (104, 26, 65536), (768, 96, 1024)])
def test_benchmark_shapes_pass_validation(jhq, d, M, nlist):
    """BASELINE configs pass parameter validation (on a GPU-less host the
    constructor then fails at device selection with JHQ_EDEVICE, not EINVAL)."""
    try:
        idx = jhq.JHQGpuIndex(d, jhq.Params(M=M, nlist=nlist, nprobe=min(64, nlist)))
        idx.close()
    except jhq.JHQError as e:
        assert e.code == jhq.JHQ_EDEVICE


def _bf16_rne(x):
    """bf16 round-to-nearest-even of float32 x, as float32 (coarse_tc.cu bf16_rne)."""
    u = x.astype(np.float32).view(np.uint32).astype(np.uint64)
    r = ((u + 0x7FFF + ((u >> 16) & 1)) >> 16) << 16
    return r.astype(np.uint32).view(np.float32)


@pytest.mark.parametrize("case", ["normal", "offset", "uint8_like", "tiny_query"])
def test_coarse_margin_bound_holds(case):
    """The tensor-core coarse scores use x = hi + lo (bf16 RNE pieces) and the sum
    q_hi.c_hi + q_hi.c_lo + q_lo.c_hi over 3d products; select_probes_margin
    (ivf.cu) takes every list within 2E of the approximate nprobe-th score, with
    E = (2 eps |q| cmax + 2^-21 (cmax^2 + 2 |q| cmax)) * 1.01,
    eps = 6 * 2^-18 + d (3 * 2^-22 + 2^-23). Emulated here with fp32 sums in
    either order: |s~ - s| <= E must hold for every list."""
    rng = np.random.default_rng(7)
    d, n = 128, 3000
    if case == "normal":
        c = rng.standard_normal((n, d)).astype(np.float32); q = rng.standard_normal(d).astype(np.float32)
    elif case == "offset":
        c = (rng.standard_normal((n, d)) + 50).astype(np.float32); q = (rng.standard_normal(d) + 50).astype(np.float32)
    elif case == "uint8_like":
        c = rng.integers(0, 256, (n, d)).astype(np.float32); q = rng.integers(0, 256, d).astype(np.float32)
    else:
        c = rng.standard_normal((n, d)).astype(np.float32); q = (rng.standard_normal(d) * 1e-4).astype(np.float32)
    norms = (c.astype(np.float64) ** 2).sum(1).astype(np.float32)
    # exact fp32 chain score (gemm_rows EPI_COARSE order)
    acc = np.zeros(n, np.float32)
    for j in range(d):
        acc = (np.float64(q[j]) * c[:, j] + acc).astype(np.float32)      # one rounding: fma
    s = (norms - np.float32(2) * acc).astype(np.float32)
    # bf16 split products, summed in fp32 forwards and backwards
    qh = _bf16_rne(q); ql = _bf16_rne((q - qh).astype(np.float32))
    ch = _bf16_rne(c); cl = _bf16_rne((c - ch).astype(np.float32))
    terms = np.concatenate([qh[None, :] * ch, qh[None, :] * cl, ql[None, :] * ch], 1).astype(np.float32)
    worst = 0.0
    for order in (slice(None), slice(None, None, -1)):
        t = np.zeros(n, np.float32)
        for col in terms.T[order]:
            t = (t + col).astype(np.float32)
        st = (norms - np.float32(2) * t).astype(np.float32)
        worst = max(worst, float(np.max(np.abs(st.astype(np.float64) - s))))
    qn = float(np.sqrt((q.astype(np.float32) ** 2).sum())) * 1.001
    cmax = float(np.sqrt(norms.max())) * 1.0001
    eps = 6 * 2.0 ** -18 + d * (3 * 2.0 ** -22 + 2.0 ** -23)
    E = (2 * eps * qn * cmax + 2.0 ** -21 * (cmax * cmax + 2 * qn * cmax)) * 1.01
    assert worst <= E, (worst, E)


def test_recall_at_k_matches_reference_definition():
    """datasets.recall_at_k restates examples/demo_jhq_v14_streaming_add.cu:15-27:
    hits of the returned ids among the first gt_k ground-truth columns / (nq k)."""
    from jhq_gpu_b200.datasets import recall_at_k
    labels = np.array([[1, 2, 3], [7, 8, -1]], np.int32)
    gt = np.array([[3, 1, 9], [8, 0, 5]], np.int32)
    assert recall_at_k(labels, gt, 3) == 3 / 6          # 1, 3 found; 8 found
    assert recall_at_k(labels, gt[:, :1], 3) == 2 / 6   # gt_k = 1: only 3 and 8
    assert recall_at_k(labels[:, :2], gt, 2) == 2 / 4


def test_vector_file_formats_roundtrip(tmp_path):
    """.fvecs / .ivecs / .bvecs / .i8bin readers (the reference demos' inputs,
    common/fvecs_io.cuh, bvecs_io.cuh, spacev_io.cuh): row ranges, padding,
    and errors on ragged or truncated files."""
    from jhq_gpu_b200 import vecio
    rng = np.random.default_rng(5)
    f = rng.standard_normal((37, 12)).astype(np.float32)
    i = rng.integers(0, 1000, (37, 10)).astype(np.int32)
    b = rng.integers(0, 256, (37, 16)).astype(np.uint8)
    s = rng.integers(-128, 128, (37, 100)).astype(np.int8)
    vecio.write_vecs(str(tmp_path / "a.fvecs"), f)
    vecio.write_vecs(str(tmp_path / "a.ivecs"), i)
    vecio.write_vecs(str(tmp_path / "a.bvecs"), b)
    vecio.write_i8bin(str(tmp_path / "a.i8bin"), s)
    assert vecio.vecs_shape(str(tmp_path / "a.fvecs")) == (37, 12)
    assert np.array_equal(vecio.read_vecs(str(tmp_path / "a.fvecs")), f)
    assert np.array_equal(vecio.read_vecs(str(tmp_path / "a.ivecs"), 5, 7), i[5:12])
    assert np.array_equal(vecio.read_vecs(str(tmp_path / "a.bvecs"), 30), b[30:].astype(np.float32))
    r = vecio.read_i8bin(str(tmp_path / "a.i8bin"), 3, 4, pad_to=104)
    assert r.shape == (4, 104) and np.array_equal(r[:, :100], s[3:7]) and not r[:, 100:].any()
    blocks = list(vecio.iter_rows(str(tmp_path / "a.bvecs"), block=10))
    assert [len(x) for x in blocks] == [10, 10, 10, 7]
    raw = open(tmp_path / "a.fvecs", "rb").read()
    open(tmp_path / "bad.fvecs", "wb").write(raw[:-3])               # truncated
    with pytest.raises(ValueError):
        vecio.read_vecs(str(tmp_path / "bad.fvecs"))
    rag = bytearray(raw)
    rag[52:56] = np.int32(11).tobytes()                              # second record's dim
    open(tmp_path / "rag.fvecs", "wb").write(bytes(rag))
    with pytest.raises(ValueError):
        vecio.read_vecs(str(tmp_path / "rag.fvecs"))
    open(tmp_path / "t.i8bin", "wb").write(np.array([37, 100], np.int32).tobytes() + b"\0" * 10)
    with pytest.raises(ValueError):
        vecio.read_i8bin(str(tmp_path / "t.i8bin"))

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

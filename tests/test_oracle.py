"""The oracle (oracle/jhq_oracle.c) pinned against the reference's own CPU code:
golden vectors produced by the reference's cpu/ (tests/golden/make_golden.py),
plus the live reference build oracle/_ref when it is present."""
import os

import numpy as np
import pytest

from oracle import REF_SO


def test_sigma_and_codewords_bit_exact(oracle, golden):
    s = oracle.sigma(golden["sigma_x"])
    assert np.float32(s) == golden["sigma"]                       # cpu/jl_transform.cpp:73-83
    for M, K in ((2, 2), (4, 4), (8, 16), (16, 256)):
        assert np.array_equal(oracle.c1d(s, K), golden[f"c1d_d16_M{M}"])  # codebook.cpp:60-80


def test_encode_reconstruct_bit_exact(oracle, golden):
    s = float(golden["sigma"])
    for M, K in ((2, 2), (4, 4), (8, 16), (16, 256)):
        c1d = oracle.c1d(s, K)
        codes = oracle.encode_primary(golden["enc_y"], M, 8, c1d)
        assert np.array_equal(codes, golden[f"codes_M{M}"])        # codebook.cpp:96-110
        rec = oracle.reconstruct(codes, 16, M, 8, c1d)
        assert np.array_equal(rec, golden[f"recon_M{M}"])          # codebook.cpp:161-171
        # encode(reconstruct(c)) == c  (idempotence of the quantiser)
        assert np.array_equal(oracle.encode_primary(rec, M, 8, c1d), codes)


def test_byte_lut_and_adc_match_reference_within_fp(oracle, golden):
    s = float(golden["sigma"])
    q = golden["enc_q"]
    for M, K in ((2, 2), (4, 4), (8, 16), (16, 256)):
        c1d = oracle.c1d(s, K)
        lut = oracle.byte_lut(q, M, 8, c1d)
        ref = golden[f"flat_lut_M{M}"]
        np.testing.assert_allclose(lut, ref, rtol=1e-5, atol=1e-6)  # codebook.cpp:112-129
        codes = golden[f"codes_M{M}"]
        adc = np.array([oracle.L.oracle_adc(lut, M, np.ascontiguousarray(c)) for c in codes],
                       np.float32)
        np.testing.assert_allclose(adc, golden[f"adc_M{M}"], rtol=1e-4)  # codebook.cpp:147-159
        # byte-LUT sum == factored sum == |q - yhat|^2
        yhat = oracle.reconstruct(codes, 16, M, 8, c1d)
        np.testing.assert_allclose(adc, ((q[None] - yhat) ** 2).sum(1), rtol=1e-4)


def test_kmeans1d_bit_exact(oracle, golden):
    assert np.array_equal(oracle.kmeans1d(golden["km_vals"], 16), golden["km_c16"])
    assert np.array_equal(oracle.kmeans1d(golden["km_vals"][:3], 4), golden["km_c4_small"])


def test_c1d_symmetry(oracle):
    for K in (2, 4, 16, 256):
        c = oracle.c1d(1.3, K)
        assert np.all(np.diff(c) > 0)
        np.testing.assert_allclose(c, -c[::-1], rtol=1e-6, atol=1e-7)


def test_residual_and_corr_identity(oracle):
    """comp = primary + residual + corr = |q - yhat - rhat|^2 + |q|^2 (encode.cu:85)."""
    rng = np.random.default_rng(3)
    d, M, B, Br = 32, 8, 8, 4
    y = rng.standard_normal((64, d)).astype(np.float32)
    c1d = oracle.c1d(1.0, 4)
    codes = oracle.encode_primary(y, M, B, c1d)
    yhat = oracle.reconstruct(codes, d, M, B, c1d)
    res_c1d = oracle.kmeans1d((y - yhat).ravel(), 16)
    rc, corr = oracle.encode_residual(y, codes, M, B, c1d, res_c1d, Br)
    q = rng.standard_normal(d).astype(np.float32)
    lut = oracle.byte_lut(q, M, B, c1d)
    for i in range(64):
        prim = oracle.L.oracle_adc(lut, M, np.ascontiguousarray(codes[i]))
        r = oracle.residual(q, Br, res_c1d, rc[i])
        nib = np.stack([rc[i] & 15, rc[i] >> 4], 1).ravel()[:d]
        rhat = res_c1d[nib]
        want = ((q - yhat[i] - rhat) ** 2).sum() + (q ** 2).sum()
        np.testing.assert_allclose(prim + r + corr[i], want, rtol=1e-4)


def test_oracle_search_equals_bruteforce_on_reconstruction(oracle):
    """Flat search = exact top-ck on primary then exact top-k on composite."""
    rng = np.random.default_rng(5)
    d, M, B, Br, n, nq, k = 16, 4, 8, 4, 500, 7, 5
    y = rng.standard_normal((n, d)).astype(np.float32)
    c1d = oracle.c1d(1.0, 4)
    codes = oracle.encode_primary(y, M, B, c1d)
    yhat = oracle.reconstruct(codes, d, M, B, c1d)
    res_c1d = oracle.kmeans1d((y - yhat).ravel(), 16)
    rc, corr = oracle.encode_residual(y, codes, M, B, c1d, res_c1d, Br)
    q = rng.standard_normal((nq, d)).astype(np.float32)
    cents = np.zeros((1, d), np.float32)
    D, I = oracle.search(q, M=M, B=B, Br=Br, c1d=c1d, res_c1d=res_c1d, codes=codes, res=rc,
                         corr=corr, assign=np.zeros(n, np.int32), cents=cents, k=k, alpha=4.0,
                         nprobe=1)
    ck = oracle.ck(k, 4.0)
    for qi in range(nq):
        lut = oracle.byte_lut(q[qi], M, B, c1d)
        prim = np.array([oracle.L.oracle_adc(lut, M, np.ascontiguousarray(c)) for c in codes])
        order = np.lexsort((np.arange(n), prim))[:ck]
        comp = np.array([(prim[i] + oracle.residual(q[qi], Br, res_c1d, rc[i])) + corr[i]
                         for i in order], np.float32)
        fin = order[np.lexsort((order, comp))][:k]
        assert np.array_equal(I[qi], fin)


@pytest.mark.skipif(not os.path.exists(REF_SO), reason="oracle/_ref not built (needs the reference tree)")
def test_oracle_vs_live_reference_build():
    from oracle import Oracle, RefCPU
    o, r = Oracle(), RefCPU()
    rng = np.random.default_rng(11)
    x = rng.standard_normal((400, 32)).astype(np.float32)
    s = o.sigma(x)
    assert s == r.sigma(x)
    y = r.apply(32, 42, x)
    assert np.array_equal(o.rotate(r.rotation(32, 42), x), y) or \
        np.abs(o.rotate(r.rotation(32, 42), x) - y).max() < 1e-5
    for M in (4, 8, 16, 32):
        K = 1 << (8 // (32 // M))
        c1d = o.c1d(s, K)
        assert np.array_equal(c1d, r.c1d(32, M, 8, s))
        assert np.array_equal(o.encode_primary(y, M, 8, c1d), r.encode(32, M, 8, s, y))


def test_oracle_rerank_is_exact_l2(oracle):
    """oracle_rerank: exact L2 (fp32 lane order) within float rounding of an fp64
    reference, (distance, id) order, -1 candidates skipped, (+inf, -1) padding."""
    rng = np.random.default_rng(3)
    x = rng.standard_normal((500, 68)).astype(np.float32)
    q = rng.standard_normal((7, 68)).astype(np.float32)
    cand = np.stack([rng.permutation(501)[:30] - 1 for _ in range(7)]).astype(np.int32)
    cand[0, :] = -1
    cand[1, 5:] = -1
    D, I = oracle.rerank(q, x, cand, 10)
    assert (I[0] == -1).all() and np.isinf(D[0]).all()
    assert (I[1, 5:] == -1).all()
    for qi in range(2, 7):
        ids = np.unique(cand[qi][cand[qi] >= 0])
        ex = ((x[ids].astype(np.float64) - q[qi]) ** 2).sum(1)
        order = np.lexsort((ids, ex))[:10]
        assert np.allclose(D[qi], ex[order], rtol=1e-5)
        np.testing.assert_allclose(D[qi], ((x[I[qi]].astype(np.float64) - q[qi]) ** 2).sum(1),
                                   rtol=1e-5)
        assert all((D[qi][j], I[qi][j]) <= (D[qi][j + 1], I[qi][j + 1]) for j in range(9))

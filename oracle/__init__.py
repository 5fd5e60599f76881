"""ctypes bindings for the JHQ oracle (test infrastructure only).

`Oracle` wraps oracle/_build/libjhq_oracle.so (the scalar C restatement in
jhq_oracle.c); `RefCPU` wraps oracle/_ref/libjhq_ref.so (the reference's own
cpu/ trainer compiled from its sources by oracle/Makefile). Only tests/,
__graft_entry__.smoke() and bench.py's CPU-baseline legs import this package;
the product (jhq_gpu_b200) never does.
"""
from __future__ import annotations

import ctypes as C
import os
import subprocess

import numpy as np

HERE = os.path.dirname(os.path.abspath(__file__))
ORACLE_SO = os.path.join(HERE, "_build", "libjhq_oracle.so")
REF_SO = os.path.join(HERE, "_ref", "libjhq_ref.so")

_f32p = np.ctypeslib.ndpointer(np.float32, flags="C_CONTIGUOUS")
_u8p = np.ctypeslib.ndpointer(np.uint8, flags="C_CONTIGUOUS")
_i32p = np.ctypeslib.ndpointer(np.int32, flags="C_CONTIGUOUS")
_i64 = C.c_int64


def build(ref: bool = False) -> None:
    """Compile the oracle (and, if asked and the reference tree exists, oracle/_ref)."""
    targets = ["oracle"]
    if ref and os.path.isdir(os.environ.get("JHQ_REFERENCE", "") or "\0"):
        targets.append("ref")
    subprocess.run(["make", "-s", "-C", HERE] + targets, check=True)


def _f32(a):
    return np.ascontiguousarray(a, dtype=np.float32)


class Oracle:
    def __init__(self, path: str = ORACLE_SO):
        if not os.path.exists(path):
            build()
        L = C.CDLL(path)
        L.oracle_sigma.restype = C.c_float
        L.oracle_sigma.argtypes = [_f32p, _i64, C.c_int]
        L.oracle_erfinv.restype = C.c_float
        L.oracle_erfinv.argtypes = [C.c_float]
        L.oracle_c1d.argtypes = [C.c_float, C.c_int, _f32p]
        L.oracle_kmeans1d.argtypes = [_f32p, _i64, C.c_int, C.c_int, _f32p]
        L.oracle_reconstruct.argtypes = [_u8p, _i64, C.c_int, C.c_int, C.c_int, _f32p, _f32p]
        L.oracle_rotate.argtypes = [_f32p, C.c_int, _f32p, _i64, _f32p]
        L.oracle_encode_primary.argtypes = [_f32p, _i64, C.c_int, C.c_int, C.c_int, _f32p, _u8p]
        L.oracle_encode_residual.argtypes = [_f32p, _u8p, _i64, C.c_int, C.c_int, C.c_int,
                                             _f32p, _f32p, C.c_int, _u8p, _f32p]
        L.oracle_encode_residual_ps.argtypes = [_f32p, _u8p, _i64, C.c_int, C.c_int, C.c_int,
                                                _f32p, _f32p, C.c_int, C.c_int, _u8p, _f32p]
        L.oracle_cent_norms.argtypes = [_f32p, C.c_int, C.c_int, _f32p]
        L.oracle_assign.argtypes = [_f32p, _i64, C.c_int, _f32p, _f32p, C.c_int, _i32p]
        L.oracle_train_ivf.argtypes = [_f32p, _i64, C.c_int, C.c_int, C.c_int, _f32p]
        L.oracle_byte_lut.argtypes = [_f32p, C.c_int, C.c_int, C.c_int, _f32p, _f32p]
        L.oracle_adc.restype = C.c_float
        L.oracle_adc.argtypes = [_f32p, C.c_int, _u8p]
        L.oracle_residual.restype = C.c_float
        L.oracle_residual.argtypes = [_f32p, C.c_int, C.c_int, _f32p, _u8p]
        L.oracle_ck.argtypes = [C.c_int, C.c_float]
        L.oracle_search.argtypes = [_f32p, _i64, C.c_int, C.c_int, C.c_int, C.c_int,
                                    _f32p, _f32p, _u8p, _u8p, _f32p, _i32p, _i64,
                                    _f32p, _f32p, C.c_int, C.c_int, C.c_int, C.c_float,
                                    C.c_int, _f32p, _i32p]
        L.oracle_search_ps.argtypes = [_f32p, _i64, C.c_int, C.c_int, C.c_int, C.c_int,
                                       _f32p, _f32p, C.c_int, _u8p, _u8p, _f32p, _i32p, _i64,
                                       _f32p, _f32p, C.c_int, C.c_int, C.c_int, C.c_float,
                                       C.c_int, _f32p, _i32p]
        L.oracle_rerank.argtypes = [_f32p, _i64, C.c_int, _f32p, _i64, _i32p, C.c_int, C.c_int,
                                    _f32p, _i32p]
        self.L = L

    def rerank(self, q, x, cand, k):
        """Exact L2 rerank of candidate ids cand [nq][kr] against x (oracle_rerank)."""
        q, x = _f32(q), _f32(x)
        cand = np.ascontiguousarray(cand, np.int32)
        D = np.zeros((len(q), k), np.float32)
        I = np.zeros((len(q), k), np.int32)
        if self.L.oracle_rerank(q, len(q), q.shape[1], x, len(x), cand, cand.shape[1], k, D, I):
            raise ValueError("oracle_rerank: bad arguments")
        return D, I

    def sigma(self, x):
        x = _f32(x)
        return self.L.oracle_sigma(x, x.shape[0], x.shape[1])

    def c1d(self, sigma, K1D):
        out = np.zeros(K1D, np.float32)
        self.L.oracle_c1d(sigma, K1D, out)
        return out

    def kmeans1d(self, vals, Kr, max_iter=25):
        vals = _f32(vals).ravel()
        out = np.zeros(Kr, np.float32)
        n = self.L.oracle_kmeans1d(vals, vals.size, Kr, max_iter, out)
        return out[:n]

    def reconstruct(self, codes, d, M, B, c1d):
        codes = np.ascontiguousarray(codes, np.uint8)
        out = np.zeros((codes.shape[0], d), np.float32)
        self.L.oracle_reconstruct(codes, codes.shape[0], d, M, B, _f32(c1d), out)
        return out

    def rotate(self, P, x):
        x = _f32(x)
        y = np.zeros_like(x)
        self.L.oracle_rotate(_f32(P), x.shape[1], x, x.shape[0], y)
        return y

    def encode_primary(self, y, M, B, c1d):
        y = _f32(y)
        codes = np.zeros((y.shape[0], M), np.uint8)
        self.L.oracle_encode_primary(y, y.shape[0], y.shape[1], M, B, _f32(c1d), codes)
        return codes

    def encode_residual(self, y, codes, M, B, c1d, res_c1d, Br, per_sub=False):
        """per_sub: res_c1d is [M][Kr], one residual codebook per subspace."""
        y = _f32(y)
        n, d = y.shape
        bpv = (d * Br + 7) // 8
        rc = np.zeros((n, bpv), np.uint8)
        corr = np.zeros(n, np.float32)
        self.L.oracle_encode_residual_ps(y, np.ascontiguousarray(codes, np.uint8), n, d, M, B,
                                         _f32(c1d), _f32(res_c1d).ravel(), Br, int(per_sub), rc,
                                         corr)
        return rc, corr

    def cent_norms(self, cents):
        cents = _f32(cents)
        out = np.zeros(cents.shape[0], np.float32)
        self.L.oracle_cent_norms(cents, cents.shape[0], cents.shape[1], out)
        return out

    def assign(self, y, cents, norms=None):
        y, cents = _f32(y), _f32(cents)
        if norms is None:
            norms = self.cent_norms(cents)
        out = np.zeros(y.shape[0], np.int32)
        self.L.oracle_assign(y, y.shape[0], y.shape[1], cents, _f32(norms), cents.shape[0], out)
        return out

    def train_ivf(self, y, nlist, iters):
        y = _f32(y)
        cents = np.zeros((nlist, y.shape[1]), np.float32)
        self.L.oracle_train_ivf(y, y.shape[0], y.shape[1], nlist, iters, cents)
        return cents

    def byte_lut(self, q_rot, M, B, c1d):
        q = _f32(q_rot).ravel()
        lut = np.zeros((M, 256), np.float32)
        self.L.oracle_byte_lut(q, q.size, M, B, _f32(c1d), lut)
        return lut

    def residual(self, q_rot, Br, res_c1d, rcode):
        q = _f32(q_rot).ravel()
        return self.L.oracle_residual(q, q.size, Br, _f32(res_c1d), np.ascontiguousarray(rcode, np.uint8))

    def ck(self, k, alpha):
        return self.L.oracle_ck(k, alpha)

    def search(self, q_rot, *, M, B, Br, c1d, res_c1d, codes, res, corr, assign,
               cents, k, alpha, nprobe, norms=None, nthreads=0, per_sub=False):
        q = _f32(q_rot)
        nq, d = q.shape
        cents = _f32(cents)
        if norms is None:
            norms = self.cent_norms(cents)
        D = np.zeros((nq, k), np.float32)
        I = np.zeros((nq, k), np.int32)
        rc = self.L.oracle_search_ps(q, nq, d, M, B, Br, _f32(c1d), _f32(res_c1d).ravel(),
                                  int(per_sub), np.ascontiguousarray(codes, np.uint8),
                                  np.ascontiguousarray(res, np.uint8), _f32(corr),
                                  np.ascontiguousarray(assign, np.int32), codes.shape[0],
                                  cents, _f32(norms), cents.shape[0], nprobe, k, alpha,
                                  nthreads, D, I)
        if rc != 0:
            raise ValueError("oracle_search: bad arguments")
        return D, I


class RefCPU:
    """The reference's own cpu/ code (codebook.cpp, jl_transform.cpp) via oracle/_ref."""

    def __init__(self, path: str = REF_SO):
        if not os.path.exists(path):
            raise FileNotFoundError(path)
        L = C.CDLL(path)
        L.ref_rotation.argtypes = [C.c_int, C.c_int, _f32p]
        L.ref_apply.argtypes = [C.c_int, C.c_int, _f32p, C.c_int, _f32p]
        L.ref_sigma.restype = C.c_float
        L.ref_sigma.argtypes = [_f32p, C.c_int, C.c_int]
        L.ref_c1d.argtypes = [C.c_int, C.c_int, C.c_int, C.c_float, _f32p]
        L.ref_encode.argtypes = [C.c_int, C.c_int, C.c_int, C.c_float, _f32p, C.c_int, _u8p]
        L.ref_flat_lut.argtypes = [C.c_int, C.c_int, C.c_int, C.c_float, _f32p, _f32p]
        L.ref_adc.argtypes = [C.c_int, C.c_int, C.c_int, C.c_float, _f32p, _u8p, C.c_int, _f32p]
        L.ref_reconstruct.argtypes = [C.c_int, C.c_int, C.c_int, C.c_float, _u8p, C.c_int, _f32p]
        L.ref_kmeans1d.argtypes = [_f32p, C.c_int, C.c_int, C.c_int, _f32p]
        self.L = L

    def rotation(self, d, seed=42):
        P = np.zeros(d * d, np.float32)
        assert self.L.ref_rotation(d, seed, P) == 0
        return P

    def apply(self, d, seed, x):
        x = _f32(x)
        y = np.zeros_like(x)
        assert self.L.ref_apply(d, seed, x, x.shape[0], y) == 0
        return y

    def sigma(self, x):
        x = _f32(x)
        return self.L.ref_sigma(x, x.shape[0], x.shape[1])

    def c1d(self, d, M, B, sigma):
        out = np.zeros(256, np.float32)
        K = self.L.ref_c1d(d, M, B, sigma, out)
        return out[:K]

    def encode(self, d, M, B, sigma, y):
        y = _f32(y)
        codes = np.zeros((y.shape[0], M), np.uint8)
        assert self.L.ref_encode(d, M, B, sigma, y, y.shape[0], codes) == 0
        return codes

    def flat_lut(self, d, M, B, sigma, q_rot):
        out = np.zeros((M, 256), np.float32)
        assert self.L.ref_flat_lut(d, M, B, sigma, _f32(q_rot).ravel(), out) == 0
        return out

    def adc(self, d, M, B, sigma, q_rot, codes):
        codes = np.ascontiguousarray(codes, np.uint8)
        out = np.zeros(codes.shape[0], np.float32)
        assert self.L.ref_adc(d, M, B, sigma, _f32(q_rot).ravel(), codes, codes.shape[0], out) == 0
        return out

    def reconstruct(self, d, M, B, sigma, codes):
        codes = np.ascontiguousarray(codes, np.uint8)
        out = np.zeros((codes.shape[0], d), np.float32)
        assert self.L.ref_reconstruct(d, M, B, sigma, codes, codes.shape[0], out) == 0
        return out

    def kmeans1d(self, vals, Kr, max_iter=25):
        vals = _f32(vals).ravel()
        out = np.zeros(Kr, np.float32)
        n = self.L.ref_kmeans1d(vals, vals.size, Kr, max_iter, out)
        return out[:n]


class RefGPU:
    """The reference's own CUDA JHQGpuIndex (v14 or v1), built from its sources by
    `make -C oracle ref_gpu`, driven through its public train/add/search API."""

    def __init__(self, version: str = "v14"):
        path = os.path.join(HERE, "_ref", f"libref_{version}.so")
        if not os.path.exists(path):
            raise FileNotFoundError(path)
        L = C.CDLL(path)
        dp = C.POINTER(C.c_double)
        L.ref_gpu_run.argtypes = [_f32p, C.c_int, C.c_int, _f32p, C.c_int, C.c_int, C.c_int,
                                  C.c_int, C.c_int, C.c_float, C.c_int, C.c_int, C.c_int,
                                  C.c_int, C.c_int, _f32p, _i32p, dp, dp, dp]
        self.L = L
        self.version = version

    def run(self, x, q, *, M, B=8, Br=4, alpha=4.0, k=10, nlist=1, nprobe=1, batch=64,
            reps=5, n_train=None):
        x, q = _f32(x), _f32(q)
        n, d = x.shape
        nt = min(n, 100_000) if n_train is None else n_train
        D = np.zeros((len(q), k), np.float32)
        I = np.zeros((len(q), k), np.int32)
        tr, ad, se = C.c_double(), C.c_double(), C.c_double()
        rc = self.L.ref_gpu_run(x, n, nt, q, len(q), d, M, B, Br, alpha, k, nlist, nprobe, batch,
                                reps, D, I, C.byref(tr), C.byref(ad), C.byref(se))
        if rc != 0:
            raise RuntimeError(f"reference {self.version} run failed")
        return D, I, dict(train_ms=tr.value, add_ms=ad.value, search_ms=se.value)

    def sweep(self, x, q, *, M, nlist, nprobes, B=8, Br=4, alpha=4.0, k=10, batch=256, reps=3,
              n_train=None):
        """IVF nprobe sweep on one trained reference index (v14 only)."""
        x, q = _f32(x), _f32(q)
        n, d = x.shape
        nt = min(n, 100_000) if n_train is None else n_train
        nps = np.ascontiguousarray(nprobes, np.int32)
        I = np.zeros((len(nps), len(q), k), np.int32)
        ms = np.zeros(len(nps), np.float64)
        tr, ad = C.c_double(), C.c_double()
        L = self.L
        L.ref_gpu_sweep.argtypes = [_f32p, C.c_int, C.c_int, _f32p, C.c_int, C.c_int, C.c_int,
                                    C.c_int, C.c_int, C.c_float, C.c_int, C.c_int, _i32p, C.c_int,
                                    C.c_int, C.c_int, _i32p, C.POINTER(C.c_double),
                                    C.POINTER(C.c_double),
                                    np.ctypeslib.ndpointer(np.float64, flags="C_CONTIGUOUS")]
        rc = L.ref_gpu_sweep(x, n, nt, q, len(q), d, M, B, Br, alpha, k, nlist, nps, len(nps),
                             batch, reps, I.reshape(-1), C.byref(tr), C.byref(ad), ms)
        if rc != 0:
            raise RuntimeError("reference sweep failed")
        return I, ms, dict(train_ms=tr.value, add_ms=ad.value)

    def pin(self, y, q_rot, *, M, c1d, res_c1d, cents, sigma=1.0, B=8, Br=4, alpha=4.0, k=10,
            nlist=1, nprobe=1, batch=64):
        """Run the reference's own add() encode and search() on the caller's artefacts
        (identity rotation, already-rotated y and q_rot; see ref_gpu_pin). Returns
        (primary codes [n][M], residual codes [n][bpv], corr [n], D [nq][k], I [nq][k]),
        all in id order."""
        y, q = _f32(y), _f32(q_rot)
        n, d = y.shape
        bpv = (d * Br + 7) // 8
        pc = np.zeros((n, M), np.uint8)
        rc = np.zeros((n, bpv), np.uint8)
        co = np.zeros(n, np.float32)
        D = np.zeros((len(q), k), np.float32)
        I = np.zeros((len(q), k), np.int32)
        L = self.L
        L.ref_gpu_pin.argtypes = [_f32p, C.c_int, _f32p, C.c_int, C.c_int, C.c_int, C.c_int,
                                  C.c_int, C.c_float, C.c_int, C.c_int, C.c_int, C.c_int,
                                  _f32p, C.c_int, _f32p, C.c_int, _f32p, C.c_float,
                                  _u8p, _u8p, _f32p, _f32p, _i32p]
        c1d, res_c1d = _f32(c1d), _f32(res_c1d)
        cents = _f32(cents) if nlist > 1 else np.zeros((1, d), np.float32)
        rcode = L.ref_gpu_pin(y, n, q, len(q), d, M, B, Br, alpha, k, nlist, nprobe, batch,
                              c1d, len(c1d), res_c1d, len(res_c1d), cents, sigma,
                              pc, rc, co, D, I)
        if rcode != 0:
            raise RuntimeError(f"reference {self.version} pin run failed ({rcode})")
        return pc, rc, co, D, I

    def pin_sweep(self, y, q_rot, *, M, c1d, res_c1d, cents, alphas, sigma=1.0, B=8, Br=4,
                  k=10, nlist=1, nprobe=1, batch=64, reps=5):
        """Time the reference's search() on the caller's artefacts (identity rotation,
        already-rotated y / q_rot) for each alpha. Returns (ids [len(alphas)][nq][k],
        mean search ms per alpha, add ms)."""
        y, q = _f32(y), _f32(q_rot)
        n, d = y.shape
        a = np.ascontiguousarray(alphas, np.float32)
        I = np.zeros((len(a), len(q), k), np.int32)
        ms = np.zeros(len(a), np.float64)
        ad = C.c_double()
        L = self.L
        L.ref_gpu_pin_sweep.argtypes = [_f32p, C.c_int, _f32p, C.c_int, C.c_int, C.c_int,
                                        C.c_int, C.c_int, C.c_int, C.c_int, C.c_int, C.c_int,
                                        _f32p, C.c_int, _f32p, C.c_int, _f32p, C.c_float,
                                        _f32p, C.c_int, C.c_int, _i32p, C.POINTER(C.c_double),
                                        np.ctypeslib.ndpointer(np.float64, flags="C_CONTIGUOUS")]
        c1d, res_c1d = _f32(c1d), _f32(res_c1d)
        cents = _f32(cents) if nlist > 1 else np.zeros((1, d), np.float32)
        rc = L.ref_gpu_pin_sweep(y, n, q, len(q), d, M, B, Br, k, nlist, nprobe, batch, c1d,
                                 len(c1d), res_c1d, len(res_c1d), cents, sigma, a, len(a), reps,
                                 I.reshape(-1), C.byref(ad), ms)
        if rc != 0:
            raise RuntimeError(f"reference {self.version} pinned sweep failed")
        return I, ms, ad.value


class RefHBlock:
    """The reference's own hblock graph index (v34 / v35 / v36), built from its
    sources by `make -C oracle ref_hblock`, driven like its demo main: train on
    min(n, 200k) rows, add all, warm up at max_ef, time `reps` searches per ef."""

    def __init__(self, version: str = "v34"):
        path = os.path.join(HERE, "_ref", f"libref_hblock_{version}.so")
        if not os.path.exists(path):
            raise FileNotFoundError(path)
        L = C.CDLL(path)
        dp = C.POINTER(C.c_double)
        L.ref_hblock_run.argtypes = [_f32p, C.c_int, _f32p, C.c_int, C.c_int, C.c_int, C.c_int,
                                     C.c_int, _i32p, C.c_int, C.c_int, _i32p, dp, dp,
                                     np.ctypeslib.ndpointer(np.float64, flags="C_CONTIGUOUS")]
        self.L = L
        self.version = version

    def sweep(self, x, q, *, efs=(8, 16, 32, 64, 128, 256), k=10, batch=1024, reps=5):
        """Returns (ids [len(efs)][nq][k], mean search ms per ef, dict(train_ms, add_ms))."""
        x, q = _f32(x), _f32(q)
        e = np.ascontiguousarray(efs, np.int32)
        I = np.zeros((len(e), len(q), k), np.int32)
        ms = np.zeros(len(e), np.float64)
        tr, ad = C.c_double(), C.c_double()
        rc = self.L.ref_hblock_run(x, x.shape[0], q, len(q), x.shape[1], k, int(e.max()), batch,
                                   e, len(e), reps, I.reshape(-1), C.byref(tr), C.byref(ad), ms)
        if rc != 0:
            raise RuntimeError(f"reference hblock {self.version} run failed")
        return I, ms, dict(train_ms=tr.value, add_ms=ad.value)

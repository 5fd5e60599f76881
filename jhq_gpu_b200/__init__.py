"""jhq_gpu_b200 — Python host mirror of the reference's jhq_gpu::JHQGpuIndex
(jhq_v14_streaming_add/jhq_gpu_index.cuh:14-47) over the C-ABI of
include/jhq.h (libjhq_b200.so, built in-tree by jhq_gpu_b200/build.py).

    idx = JHQGpuIndex(d, Params(M=128, B=8, Br=4, alpha=4.0, nlist=1))
    idx.train(x)          # x: (n, d) float32
    idx.add(x)
    D, I = idx.search(q, k=10)

Errors follow the reference's exception classes: JHQ_EINVAL raises
ValueError (std::invalid_argument), JHQ_ESTATE raises RuntimeError
(std::runtime_error); device/IO/timeout failures raise JHQError. The CUDA
library is required: importing works without it, but every call fails
loudly if libjhq_b200.so is missing — there is no CPU fallback.
"""
from __future__ import annotations

import ctypes as C
import dataclasses
import os
from typing import Optional, Tuple

import numpy as np

HERE = os.path.dirname(os.path.abspath(__file__))
LIB_PATH = os.path.join(HERE, "libjhq_b200.so")

JHQ_OK, JHQ_EINVAL, JHQ_ENOMEM, JHQ_ETIMEDOUT, JHQ_EDEVICE, JHQ_ESTATE, JHQ_EIO = range(7)

# Every symbol include/jhq.h declares (checked by tests/test_capi_symbols.py).
EXPORTED = [
    "jhq_params_default", "jhq_index_create", "jhq_index_destroy", "jhq_train", "jhq_add",
    "jhq_search", "jhq_search_device", "jhq_synchronize", "jhq_ntotal", "jhq_dim",
    "jhq_is_trained", "jhq_get_trained", "jhq_set_trained", "jhq_get_codes", "jhq_rotate",
    "jhq_encode", "jhq_save", "jhq_load", "jhq_merge_shards", "jhq_kernel_launches",
    "jhq_last_error", "jhq_version", "jhq_jl_rotation", "jhq_estimate_sigma",
    "jhq_lloyd_max_c1d", "jhq_kmeans_1d", "jhq_set_profiling", "jhq_stage_times",
    "jhq_search_device_noalloc", "jhq_set_nprobe", "jhq_set_rerank", "jhq_get_rerank",
    "jhq_set_alpha", "jhq_list_sizes", "jhq_rotate_queries", "jhq_device_status", "jhq_set_residual_codebooks",
    "jhq_get_residual_codebooks", "jhq_debug_flat_scores", "jhq_set_list_paging", "jhq_paging_waves",
    "jhq_probe_device",
    "jhq_search_device_probes", "jhq_sharded_create", "jhq_sharded_destroy",
    "jhq_sharded_train", "jhq_sharded_add", "jhq_sharded_search", "jhq_sharded_set_nprobe",
    "jhq_sharded_ntotal",
]
STAGES = ["rotate", "coarse+probes", "plan", "scan", "refine"]


class JHQError(RuntimeError):
    def __init__(self, code: int, msg: str):
        super().__init__(f"[JHQ status {code}] {msg}")
        self.code = code


class CParams(C.Structure):
    _fields_ = [("M", C.c_int), ("B", C.c_int), ("Br", C.c_int), ("alpha", C.c_float),
                ("nlist", C.c_int), ("nprobe", C.c_int), ("ivf_iters", C.c_int),
                ("batch_size", C.c_int), ("seed", C.c_int), ("add_batch", C.c_int),
                ("device", C.c_int)]


@dataclasses.dataclass
class Params:
    """JHQGpuIndex::Params (jhq_gpu_index.cuh:16-36), same fields and defaults."""
    M: int = 96
    B: int = 8
    Br: int = 4
    alpha: float = 4.0
    nlist: int = 1024
    nprobe: int = 8
    ivf_iters: int = 8
    batch_size: int = 256
    seed: int = 42
    add_batch: int = 65536
    device: int = -1

    def to_c(self) -> CParams:
        return CParams(*[getattr(self, f.name) for f in dataclasses.fields(self)])


_lib: Optional[C.CDLL] = None


def load_library(path: str = "") -> C.CDLL:
    """Load libjhq_b200.so (raises if it has not been built). The JHQ_LIBRARY
    environment variable selects another build of the same library."""
    global _lib
    if _lib is not None:
        return _lib
    path = path or os.environ.get("JHQ_LIBRARY") or LIB_PATH
    if not os.path.exists(path):
        raise RuntimeError(f"{path} is missing: run `python -m jhq_gpu_b200.build` "
                           "(the CUDA library is required; there is no CPU fallback)")
    L = C.CDLL(path)
    vp, i64, f32p, i32p, u8p = C.c_void_p, C.c_int64, C.POINTER(C.c_float), C.POINTER(C.c_int32), \
        C.POINTER(C.c_uint8)
    L.jhq_params_default.argtypes = [C.POINTER(CParams)]
    L.jhq_index_create.argtypes = [C.c_int, C.POINTER(CParams), C.POINTER(vp)]
    L.jhq_index_destroy.argtypes = [vp]
    L.jhq_train.argtypes = [vp, f32p, i64]
    L.jhq_add.argtypes = [vp, f32p, i64]
    L.jhq_search.argtypes = [vp, f32p, i64, C.c_int, f32p, i32p]
    L.jhq_search_device.argtypes = [vp, vp, i64, C.c_int, vp, vp, vp]
    L.jhq_search_device_noalloc.argtypes = [vp, vp, i64, C.c_int, vp, vp, vp]
    L.jhq_synchronize.argtypes = [vp, C.c_double]
    L.jhq_set_nprobe.argtypes = [vp, C.c_int]
    L.jhq_set_rerank.argtypes = [vp, C.c_int]
    L.jhq_set_alpha.argtypes = [vp, C.c_float]
    L.jhq_rotate_queries.argtypes = [vp, f32p, i64, f32p]
    L.jhq_list_sizes.argtypes = [vp, C.POINTER(C.c_int64)]
    L.jhq_device_status.argtypes = [vp]
    L.jhq_debug_flat_scores.argtypes = [vp, f32p, C.c_int, f32p]
    L.jhq_set_residual_codebooks.argtypes = [vp, C.c_int]
    L.jhq_set_list_paging.argtypes = [vp, i64]
    L.jhq_paging_waves.argtypes = [vp, C.POINTER(C.c_int64)]
    L.jhq_get_residual_codebooks.argtypes = [vp, C.POINTER(C.c_int)]
    L.jhq_get_rerank.argtypes = [vp, C.POINTER(C.c_int)]
    L.jhq_probe_device.argtypes = [vp, vp, i64, vp, vp]
    L.jhq_search_device_probes.argtypes = [vp, vp, vp, i64, C.c_int, vp, vp, vp]
    L.jhq_ntotal.argtypes = [vp, C.POINTER(C.c_int64)]
    L.jhq_dim.argtypes = [vp, C.POINTER(C.c_int)]
    L.jhq_is_trained.argtypes = [vp, C.POINTER(C.c_int)]
    L.jhq_get_trained.argtypes = [vp, f32p, f32p, f32p, f32p, f32p]
    L.jhq_set_trained.argtypes = [vp, f32p, f32p, f32p, f32p, C.c_float]
    L.jhq_get_codes.argtypes = [vp, u8p, u8p, f32p, i32p]
    L.jhq_rotate.argtypes = [vp, f32p, i64, f32p]
    L.jhq_encode.argtypes = [vp, f32p, i64, u8p, u8p, f32p]
    L.jhq_save.argtypes = [vp, C.c_char_p]
    L.jhq_load.argtypes = [C.c_char_p, C.c_int, C.POINTER(vp)]
    L.jhq_merge_shards.argtypes = [vp, vp, C.c_int, i64, C.c_int, vp, vp, vp]
    L.jhq_jl_rotation.argtypes = [C.c_int, C.c_int, f32p]
    L.jhq_estimate_sigma.argtypes = [f32p, i64, C.c_int, f32p]
    L.jhq_lloyd_max_c1d.argtypes = [C.c_float, C.c_int, f32p]
    L.jhq_kmeans_1d.argtypes = [f32p, i64, C.c_int, C.c_int, f32p, C.POINTER(C.c_int)]
    L.jhq_set_profiling.argtypes = [vp, C.c_int]
    L.jhq_stage_times.argtypes = [vp, C.POINTER(C.c_double), C.POINTER(C.c_int64), C.c_int]
    L.jhq_sharded_create.argtypes = [C.c_int, C.POINTER(CParams), C.c_int, i32p, C.POINTER(vp)]
    L.jhq_sharded_destroy.argtypes = [vp]
    L.jhq_sharded_train.argtypes = [vp, f32p, i64]
    L.jhq_sharded_add.argtypes = [vp, f32p, i64]
    L.jhq_sharded_search.argtypes = [vp, f32p, i64, C.c_int, f32p, i32p]
    L.jhq_sharded_set_nprobe.argtypes = [vp, C.c_int]
    L.jhq_sharded_ntotal.argtypes = [vp]
    L.jhq_sharded_ntotal.restype = C.c_int64
    L.jhq_kernel_launches.restype = C.c_int64
    L.jhq_last_error.restype = C.c_char_p
    L.jhq_version.restype = C.c_char_p
    _lib = L
    return L


def _check(rc: int) -> None:
    if rc == JHQ_OK:
        return
    msg = load_library().jhq_last_error().decode(errors="replace")
    if rc == JHQ_EINVAL:
        raise ValueError(msg)
    if rc == JHQ_ESTATE:
        raise RuntimeError(msg)
    raise JHQError(rc, msg)


def _ptr(a: np.ndarray, ct):
    return a.ctypes.data_as(C.POINTER(ct))


def _f32(a) -> np.ndarray:
    return np.ascontiguousarray(a, dtype=np.float32)


def jl_rotation(d: int, seed: int = 42) -> np.ndarray:
    """JLTransform(d, seed) rotation, d*d column-major (host only)."""
    P = np.empty(d * d, np.float32)
    _check(load_library().jhq_jl_rotation(d, seed, _ptr(P, C.c_float)))
    return P


def estimate_sigma(x) -> float:
    x = _f32(x)
    s = C.c_float()
    _check(load_library().jhq_estimate_sigma(_ptr(x, C.c_float), x.shape[0], x.shape[1], C.byref(s)))
    return s.value


def lloyd_max_c1d(sigma: float, K1D: int) -> np.ndarray:
    out = np.empty(K1D, np.float32)
    _check(load_library().jhq_lloyd_max_c1d(sigma, K1D, _ptr(out, C.c_float)))
    return out


def kmeans_1d(vals, Kr: int, max_iter: int = 25) -> np.ndarray:
    v = _f32(vals).ravel()
    out = np.empty(Kr, np.float32)
    n = C.c_int()
    _check(load_library().jhq_kmeans_1d(_ptr(v, C.c_float), v.size, Kr, max_iter,
                                        _ptr(out, C.c_float), C.byref(n)))
    return out[:n.value]


def kernel_launches() -> int:
    return int(load_library().jhq_kernel_launches())


def merge_shards(d_in_dists: int, d_in_ids: int, nshards: int, nq: int, k: int,
                 d_out_dists: int, d_out_ids: int, stream: int = 0) -> None:
    """k-way merge of per-shard device top-k lists (raw device pointers)."""
    _check(load_library().jhq_merge_shards(d_in_dists, d_in_ids, nshards, nq, k,
                                           d_out_dists, d_out_ids, stream))


class JHQGpuIndex:
    """Mirror of jhq_gpu::JHQGpuIndex; one caller at a time (like the reference)."""

    def __init__(self, d: int, params: Optional[Params] = None, *, _handle=None):
        L = load_library()
        self._L = L
        self.params = params or Params()
        if _handle is not None:
            self._h = _handle
        else:
            h = C.c_void_p()
            cp = self.params.to_c()
            _check(L.jhq_index_create(d, C.byref(cp), C.byref(h)))
            self._h = h
        dd = C.c_int()
        _check(L.jhq_dim(self._h, C.byref(dd)))
        self.d = dd.value
        p = self.params
        self.Ds = self.d // p.M
        self.K1D = 1 << (p.B // self.Ds)
        self.Kr = 1 << p.Br
        self.bpv = (self.d * p.Br + 7) // 8

    def __del__(self):
        h = getattr(self, "_h", None)
        if h is not None and h.value:
            try:
                self._L.jhq_index_destroy(h)
            except Exception:
                pass
            self._h = None

    def close(self):
        self.__del__()

    # -- reference API ---------------------------------------------------------
    def train(self, x) -> None:
        x = _f32(x)
        _check(self._L.jhq_train(self._h, _ptr(x, C.c_float), x.shape[0]))

    def add(self, x) -> None:
        x = _f32(x)
        _check(self._L.jhq_add(self._h, _ptr(x, C.c_float), x.shape[0]))

    def search(self, q, k: int) -> Tuple[np.ndarray, np.ndarray]:
        q = _f32(q)
        nq = q.shape[0]
        D = np.empty((nq, k), np.float32)
        I = np.empty((nq, k), np.int32)
        _check(self._L.jhq_search(self._h, _ptr(q, C.c_float), nq, k, _ptr(D, C.c_float),
                                  _ptr(I, C.c_int32)))
        return D, I

    def search_device(self, q_ptr: int, nq: int, k: int, d_ptr: int, i_ptr: int,
                      stream: int = 0) -> None:
        """Device-buffer search (raw CUDA pointers, e.g. torch tensor.data_ptr())."""
        _check(self._L.jhq_search_device(self._h, q_ptr, nq, k, d_ptr, i_ptr, stream))

    def search_device_noalloc(self, q_ptr: int, nq: int, k: int, d_ptr: int, i_ptr: int,
                              stream: int = 0) -> None:
        """Device-buffer search that allocates no device memory: its temporaries sit
        in a fixed 16 MiB array inside the library (for callers that must not
        allocate while serving). Calls that overlap on the GPU race; serialise them."""
        _check(self._L.jhq_search_device_noalloc(self._h, q_ptr, nq, k, d_ptr, i_ptr, stream))

    def probe_device(self, q_ptr: int, nq: int, probes_ptr: int, stream: int = 0) -> None:
        """nprobe list ids per query ([nq][nprobe] int32, device) without searching."""
        _check(self._L.jhq_probe_device(self._h, q_ptr, nq, probes_ptr, stream))

    def search_device_probes(self, q_ptr: int, probes_ptr: int, nq: int, k: int, d_ptr: int,
                             i_ptr: int, stream: int = 0) -> None:
        """Device search with given probe lists (from probe_device, any rank)."""
        _check(self._L.jhq_search_device_probes(self._h, q_ptr, probes_ptr, nq, k, d_ptr, i_ptr,
                                                stream))

    def set_nprobe(self, nprobe: int) -> None:
        """Probe count of later searches (clamped to nlist)."""
        _check(self._L.jhq_set_nprobe(self._h, nprobe))
        self.params.nprobe = min(nprobe, self.params.nlist)

    def set_residual_codebooks(self, per_subspace: bool) -> None:
        """M per-subspace residual codebooks instead of one (before train)."""
        _check(self._L.jhq_set_residual_codebooks(self._h, int(bool(per_subspace))))

    @property
    def residual_per_subspace(self) -> bool:
        v = C.c_int()
        _check(self._L.jhq_get_residual_codebooks(self._h, C.byref(v)))
        return bool(v.value)

    def set_list_paging(self, pool_bytes: int) -> None:
        """Out-of-core lists: codes in mapped host memory, a device page pool of
        pool_bytes staged per search batch (jhq_set_list_paging); before add()."""
        _check(self._L.jhq_set_list_paging(self._h, int(pool_bytes)))

    @property
    def paging_waves(self) -> int:
        v = C.c_int64()
        _check(self._L.jhq_paging_waves(self._h, C.byref(v)))
        return v.value

    def debug_flat_scores(self, q) -> np.ndarray:
        """Approximate ADC scores [nq][ntotal] of the tensor-core flat scan."""
        q = _f32(q)
        out = np.empty((q.shape[0], self.ntotal), np.float32)
        _check(self._L.jhq_debug_flat_scores(self._h, _ptr(q, C.c_float), q.shape[0],
                                             _ptr(out, C.c_float)))
        return out

    def check_device_status(self) -> None:
        """Raises JHQError (JHQ_ETIMEDOUT) if a device wait of a search on the
        caller's stream gave up (jhq_device_status); call after the stream drained."""
        _check(self._L.jhq_device_status(self._h))

    def list_sizes(self) -> np.ndarray:
        out = np.zeros(self.params.nlist, np.int64)
        _check(self._L.jhq_list_sizes(self._h, _ptr(out, C.c_int64)))
        return out

    def set_alpha(self, alpha: float) -> None:
        _check(self._L.jhq_set_alpha(self._h, alpha))
        self.params.alpha = float(alpha)

    def set_rerank(self, R: int) -> None:
        """Exact L2 rerank of the best max(R, k) JHQ candidates over the stored
        vectors (jhq_set_rerank); enable before the first add(). 0 = off."""
        _check(self._L.jhq_set_rerank(self._h, R))

    @property
    def rerank(self) -> int:
        r = C.c_int()
        _check(self._L.jhq_get_rerank(self._h, C.byref(r)))
        return r.value

    def synchronize(self, timeout_s: float = 60.0) -> None:
        _check(self._L.jhq_synchronize(self._h, timeout_s))

    @property
    def ntotal(self) -> int:
        n = C.c_int64()
        _check(self._L.jhq_ntotal(self._h, C.byref(n)))
        return n.value

    @property
    def is_trained(self) -> bool:
        t = C.c_int()
        _check(self._L.jhq_is_trained(self._h, C.byref(t)))
        return bool(t.value)

    def set_profiling(self, on: bool) -> None:
        _check(self._L.jhq_set_profiling(self._h, int(on)))

    def stage_times(self) -> Tuple[dict, int]:
        ms = (C.c_double * 5)()
        nb = C.c_int64()
        _check(self._L.jhq_stage_times(self._h, ms, C.byref(nb), 5))
        return dict(zip(STAGES, list(ms))), nb.value

    # -- artefacts / inspection --------------------------------------------------
    def get_trained(self) -> dict:
        d, p = self.d, self.params
        Pi = np.empty(d * d, np.float32)
        c1d = np.empty(self.K1D, np.float32)
        per_sub = self.residual_per_subspace
        res = np.empty((p.M, self.Kr) if per_sub else self.Kr, np.float32)
        cents = np.empty((p.nlist, d), np.float32)
        sigma = C.c_float()
        _check(self._L.jhq_get_trained(self._h, _ptr(Pi, C.c_float), _ptr(c1d, C.c_float),
                                       _ptr(res, C.c_float), _ptr(cents, C.c_float),
                                       C.byref(sigma)))
        return dict(Pi=Pi, c1d=c1d, res_c1d=res, cents=cents, sigma=sigma.value)

    def set_trained(self, Pi, c1d, res_c1d, cents, sigma: float = 1.0) -> None:
        Pi, c1d, res_c1d, cents = _f32(Pi), _f32(c1d), _f32(res_c1d), _f32(cents)
        nres = self.Kr * (self.params.M if self.residual_per_subspace else 1)
        if Pi.size != self.d * self.d or c1d.size != self.K1D or res_c1d.size != nres or \
                cents.size != self.params.nlist * self.d:
            raise ValueError("set_trained: artefact sizes do not match the index")
        _check(self._L.jhq_set_trained(self._h, _ptr(Pi, C.c_float), _ptr(c1d, C.c_float),
                                       _ptr(res_c1d, C.c_float), _ptr(cents, C.c_float), sigma))

    def get_codes(self):
        n, p = self.ntotal, self.params
        pc = np.empty((n, p.M), np.uint8)
        rc = np.empty((n, self.bpv), np.uint8)
        co = np.empty(n, np.float32)
        asg = np.empty(n, np.int32)
        if n:
            _check(self._L.jhq_get_codes(self._h, _ptr(pc, C.c_uint8), _ptr(rc, C.c_uint8),
                                         _ptr(co, C.c_float), _ptr(asg, C.c_int32)))
        return pc, rc, co, asg

    def rotate(self, x) -> np.ndarray:
        x = _f32(x)
        y = np.empty_like(x)
        _check(self._L.jhq_rotate(self._h, _ptr(x, C.c_float), x.shape[0], _ptr(y, C.c_float)))
        return y

    def rotate_queries(self, x) -> np.ndarray:
        """The rotation search() applies to queries (tensor cores on B200)."""
        x = _f32(x)
        y = np.empty_like(x)
        _check(self._L.jhq_rotate_queries(self._h, _ptr(x, C.c_float), x.shape[0], _ptr(y, C.c_float)))
        return y

    def encode(self, y):
        y = _f32(y)
        n = y.shape[0]
        pc = np.empty((n, self.params.M), np.uint8)
        rc = np.empty((n, self.bpv), np.uint8)
        co = np.empty(n, np.float32)
        _check(self._L.jhq_encode(self._h, _ptr(y, C.c_float), n, _ptr(pc, C.c_uint8),
                                  _ptr(rc, C.c_uint8), _ptr(co, C.c_float)))
        return pc, rc, co

    def save(self, path: str) -> None:
        _check(self._L.jhq_save(self._h, path.encode()))

    @classmethod
    def load(cls, path: str, device: int = -1, params: Optional[Params] = None) -> "JHQGpuIndex":
        L = load_library()
        h = C.c_void_p()
        _check(L.jhq_load(path.encode(), device, C.byref(h)))
        obj = cls.__new__(cls)
        obj.params = params or _read_params(path)
        JHQGpuIndex.__init__(obj, 0, obj.params, _handle=h)
        return obj


def _read_params(path: str) -> Params:
    with open(path, "rb") as f:
        f.read(12)
        hdr = np.frombuffer(f.read(48), np.int32)
        alpha = float(np.frombuffer(f.read(4), np.float32)[0])
    return Params(M=int(hdr[1]), B=int(hdr[2]), Br=int(hdr[3]), alpha=alpha, nlist=int(hdr[4]),
                  nprobe=int(hdr[5]), ivf_iters=int(hdr[6]), batch_size=int(hdr[7]),
                  seed=int(hdr[8]), add_batch=int(hdr[9]))


class JHQShardedIndex:
    """Single-process sharded index (jhq_sharded_*): the JHQGpuIndex call shape
    over shards on `devices` (one GPU each, or repeated ordinals for several
    shards on one GPU). Global id g lives on shard g % nshards."""

    def __init__(self, d: int, params: Optional[Params] = None, devices=(0,)):
        self._L = load_library()
        self.params = params or Params()
        self.devices = [int(x) for x in devices]
        devs = np.asarray(self.devices, np.int32)
        h = C.c_void_p()
        cp = self.params.to_c()
        _check(self._L.jhq_sharded_create(d, C.byref(cp), len(self.devices),
                                          _ptr(devs, C.c_int32), C.byref(h)))
        self._h = h
        self.d = d

    def __del__(self):
        h = getattr(self, "_h", None)
        if h is not None and h.value:
            try:
                self._L.jhq_sharded_destroy(h)
            except Exception:
                pass
            self._h = None

    def close(self):
        self.__del__()

    @property
    def ntotal(self) -> int:
        return int(self._L.jhq_sharded_ntotal(self._h))

    def train(self, x) -> None:
        x = _f32(x)
        _check(self._L.jhq_sharded_train(self._h, _ptr(x, C.c_float), x.shape[0]))

    def add(self, x) -> None:
        x = _f32(x)
        _check(self._L.jhq_sharded_add(self._h, _ptr(x, C.c_float), x.shape[0]))

    def set_nprobe(self, nprobe: int) -> None:
        _check(self._L.jhq_sharded_set_nprobe(self._h, nprobe))

    def search(self, q, k: int) -> Tuple[np.ndarray, np.ndarray]:
        q = _f32(q)
        nq = q.shape[0]
        D = np.empty((nq, k), np.float32)
        I = np.empty((nq, k), np.int32)
        _check(self._L.jhq_sharded_search(self._h, _ptr(q, C.c_float), nq, k, _ptr(D, C.c_float),
                                          _ptr(I, C.c_int32)))
        return D, I

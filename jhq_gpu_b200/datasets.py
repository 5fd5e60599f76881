"""Seeded synthetic stand-ins for the benchmark datasets (no network here).

The reference measures on public embedding sets (Vogue-768, bge-m3, SIFT100M,
SPACEV100M ...); the benchmark configurations replace them with generated
data of the stated shapes and value distributions:

  C0  flat  10,000 + 100     D=128  i.i.d. N(0,1)
  C1  flat  100,000 + 1,000  D=1024 L2-normalised draws from a 1,024-component
            isotropic Gaussian mixture, centres N(0,1), sigma 0.35 before
            normalisation
  C2  IVF   1,000,000 + 10,000, same generator with 4,096 components
  C3  IVF   100M + 10k D=128 uint8: round(clip(x, 0, 255)), 16,384 components,
            centres U(0,120), sigma 18, ~25% of dims zero-heavy (70% mass at 0)
  C4  IVF   100M + 10k D=100 int8 (zero-padded to 104): round(clip(x,-128,127)),
            Student-t(4) mixture of 16,384 components, centres N(0, 20^2), scale 12

Base and query sets are drawn from the same generator with different
sub-seeds derived from the config seed. The 100M-row generators (rows_c3,
rows_c4) seed every 500,000-row block separately, so a rank generates only its
own row range and host memory never holds the whole set.
"""
from __future__ import annotations

from typing import Iterator, Tuple

import numpy as np

CONFIGS = {
    "c0": dict(n=10_000, nq=100, d=128, M=32, nlist=1, nprobe=1, batch=64),
    "c1": dict(n=100_000, nq=1_000, d=1024, M=128, nlist=1, nprobe=1, batch=64),
    "c2": dict(n=1_000_000, nq=10_000, d=1024, M=128, nlist=1024, nprobe=64, batch=256),
    "c3": dict(n=100_000_000, nq=10_000, d=128, M=32, nlist=65_536, nprobe=64, batch=10_000),
    "c4": dict(n=100_000_000, nq=10_000, d=104, M=26, nlist=65_536, nprobe=64, batch=10_000),
}


def _rng(seed: int, sub: int) -> np.random.Generator:
    return np.random.default_rng(np.random.SeedSequence([seed, sub]))


def iid_normal(n: int, d: int, seed: int, sub: int) -> np.ndarray:
    return _rng(seed, sub).standard_normal((n, d), dtype=np.float32)


def normalized_mixture(n: int, d: int, ncomp: int, seed: int, sub: int, sigma: float = 0.35,
                       block: int = 65536) -> np.ndarray:
    """L2-normalised draws from an isotropic Gaussian mixture (C1/C2)."""
    centres = _rng(seed, 1000).standard_normal((ncomp, d), dtype=np.float32)
    rng = _rng(seed, sub)
    out = np.empty((n, d), np.float32)
    for s in range(0, n, block):
        e = min(n, s + block)
        comp = rng.integers(0, ncomp, e - s)
        x = centres[comp] + sigma * rng.standard_normal((e - s, d), dtype=np.float32)
        x /= np.linalg.norm(x, axis=1, keepdims=True)
        out[s:e] = x
    return out


BLOCK = 500_000          # rows per independently seeded block of the 100M-row generators


def _uint8_block(seed: int, sub: int, b: int, rows: int, d: int, centres, zero_dims):
    rng = np.random.default_rng(np.random.SeedSequence([seed, sub, b]))
    comp = rng.integers(0, len(centres), rows)
    x = rng.standard_normal((rows, d), dtype=np.float32)
    x *= 18.0
    x += centres[comp]
    zd = np.flatnonzero(zero_dims)                  # zero-heavy dims: 70% of values set to 0
    sub_x = x[:, zd]
    sub_x[rng.random((rows, len(zd)), dtype=np.float32) < 0.7] = 0.0
    x[:, zd] = sub_x
    np.clip(x, 0, 255, out=x)
    return np.round(x, out=x)


def _int8_block(seed: int, sub: int, b: int, rows: int, d: int, d_pad: int, centres):
    rng = np.random.default_rng(np.random.SeedSequence([seed, sub, b]))
    comp = rng.integers(0, len(centres), rows)
    x = centres[comp] + 12.0 * rng.standard_t(4, (rows, d)).astype(np.float32)
    out = np.zeros((rows, d_pad), np.float32)
    out[:, :d] = np.round(np.clip(x, -128, 127))
    return out


def rows_c3(lo: int, hi: int, seed: int = 0, sub: int = 1, d: int = 128,
            ncomp: int = 16384) -> Iterator[np.ndarray]:
    """C3 rows [lo, hi) (float32 of exact uint8 values), one block-slice at a time;
    block b of BLOCK rows has its own seed, so any row range is generated alone."""
    cr = _rng(seed, 2000)
    centres = cr.uniform(0, 120, (ncomp, d)).astype(np.float32)
    zero_dims = cr.random(d) < 0.25
    for b in range(lo // BLOCK, (hi + BLOCK - 1) // BLOCK):
        blk = _uint8_block(seed, sub, b, BLOCK, d, centres, zero_dims)
        s, e = max(lo, b * BLOCK) - b * BLOCK, min(hi, (b + 1) * BLOCK) - b * BLOCK
        yield blk[s:e]


def rows_c4(lo: int, hi: int, seed: int = 0, sub: int = 1, d: int = 100, d_pad: int = 104,
            ncomp: int = 16384) -> Iterator[np.ndarray]:
    """C4 rows [lo, hi), zero-padded from 100 to 104 dims (float32 of exact integers)."""
    centres = (20.0 * _rng(seed, 3000).standard_normal((ncomp, d))).astype(np.float32)
    for b in range(lo // BLOCK, (hi + BLOCK - 1) // BLOCK):
        blk = _int8_block(seed, sub, b, BLOCK, d, d_pad, centres)
        s, e = max(lo, b * BLOCK) - b * BLOCK, min(hi, (b + 1) * BLOCK) - b * BLOCK
        yield blk[s:e]


def make(config: str, seed: int = 0, n: int | None = None, nq: int | None = None
         ) -> Tuple[np.ndarray, np.ndarray]:
    """(base, queries) for configs that fit in host memory (c0, c1, c2 or reduced sizes)."""
    c = CONFIGS[config]
    n = c["n"] if n is None else n
    nq = c["nq"] if nq is None else nq
    if config == "c0":
        return iid_normal(n, c["d"], seed, 1), iid_normal(nq, c["d"], seed, 2)
    if config in ("c1", "c2"):
        ncomp = 1024 if config == "c1" else 4096
        return (normalized_mixture(n, c["d"], ncomp, seed, 1),
                normalized_mixture(nq, c["d"], ncomp, seed, 2))
    if config == "c3":
        return (np.concatenate(list(rows_c3(0, n, seed, 1))),
                np.concatenate(list(rows_c3(0, nq, seed, 2))))
    if config == "c4":
        return (np.concatenate(list(rows_c4(0, n, seed, 1))),
                np.concatenate(list(rows_c4(0, nq, seed, 2))))
    raise KeyError(config)


def ground_truth_torch(base: np.ndarray, queries: np.ndarray, k: int, device: str = "cuda",
                       block: int = 1 << 16) -> np.ndarray:
    """Exact L2 top-k ids (fp32, TF32 off) by brute force on the GPU."""
    import torch
    prev = torch.backends.cuda.matmul.allow_tf32
    torch.backends.cuda.matmul.allow_tf32 = False
    try:
        q = torch.from_numpy(queries).to(device)
        qn = (q * q).sum(1, keepdim=True)
        best_d = torch.full((q.shape[0], k), float("inf"), device=device)
        best_i = torch.full((q.shape[0], k), -1, dtype=torch.int64, device=device)
        for s in range(0, base.shape[0], block):
            b = torch.from_numpy(base[s:s + block]).to(device)
            dist = qn - 2.0 * q @ b.T + (b * b).sum(1)[None, :]
            dd = torch.cat([best_d, dist], 1)
            ii = torch.cat([best_i, torch.arange(s, s + b.shape[0], device=device)
                            .expand(q.shape[0], -1)], 1)
            best_d, pos = dd.topk(k, dim=1, largest=False)
            best_i = ii.gather(1, pos)
        return best_i.cpu().numpy().astype(np.int32)
    finally:
        torch.backends.cuda.matmul.allow_tf32 = prev


def ground_truth_numpy(base: np.ndarray, queries: np.ndarray, k: int) -> np.ndarray:
    bn = (base.astype(np.float64) ** 2).sum(1)
    out = np.empty((len(queries), k), np.int32)
    for i, q in enumerate(queries.astype(np.float64)):
        dist = bn - 2.0 * base @ q
        out[i] = np.argsort(dist, kind="stable")[:k]
    return out


def recall_at_k(labels: np.ndarray, gt: np.ndarray, k: int) -> float:
    """Hits of returned ids among the first gt columns / (nq k) — the reference's
    recall_at_k (examples/demo_jhq_v14_streaming_add.cu:15-27)."""
    hits = 0
    for row, g in zip(labels[:, :k], gt):
        gs = set(int(v) for v in g)
        hits += sum(1 for v in row if int(v) in gs)
    return hits / float(labels.shape[0] * k)


def _torch_gen(device, seed: int, sub: int, b: int):
    import torch
    g = torch.Generator(device=device)
    g.manual_seed((seed * 1_000_003 + sub) * 1_000_003 + b)
    return g


def rows_torch(config: str, lo: int, hi: int, device, seed: int = 0, sub: int = 1):
    """C3 / C4 rows [lo, hi) generated on a CUDA device (float32 tensor of exact
    integer values), for the 100M-row sharded runs. Every BLOCK-row block has
    its own generator seed, so a rank can make exactly its own row range and
    the rows do not depend on the number of ranks. Same distributions as
    rows_c3 / rows_c4 (which use numpy and are used for small sets)."""
    import torch
    if config == "c3":
        d, ncomp = 128, 16384
        g0 = _torch_gen(device, seed, 2000, 0)
        centres = torch.rand((ncomp, d), generator=g0, device=device) * 120.0
        zero_dims = torch.rand(d, generator=g0, device=device) < 0.25
    else:
        d, d_pad, ncomp = 100, 104, 16384
        g0 = _torch_gen(device, seed, 3000, 0)
        centres = 20.0 * torch.randn((ncomp, d), generator=g0, device=device)
    out = []
    for b in range(lo // BLOCK, (hi + BLOCK - 1) // BLOCK):
        g = _torch_gen(device, seed, sub, b)
        comp = torch.randint(0, ncomp, (BLOCK,), generator=g, device=device)
        if config == "c3":
            x = centres[comp] + 18.0 * torch.randn((BLOCK, d), generator=g, device=device)
            zmask = (torch.rand((BLOCK, d), generator=g, device=device) < 0.7) & zero_dims[None, :]
            x = torch.where(zmask, torch.zeros_like(x), x)
            x = torch.round(torch.clamp(x, 0, 255))
        else:
            z = torch.randn((BLOCK, d), generator=g, device=device)
            chi = torch.randn((BLOCK, d, 4), generator=g, device=device).pow(2).sum(-1) / 4.0
            t = z / torch.sqrt(chi)                         # Student-t, 4 degrees of freedom
            x = torch.zeros((BLOCK, d_pad), device=device)
            x[:, :d] = torch.round(torch.clamp(centres[comp] + 12.0 * t, -128, 127))
        s, e = max(lo, b * BLOCK) - b * BLOCK, min(hi, (b + 1) * BLOCK) - b * BLOCK
        out.append(x[s:e])
    return torch.cat(out) if out else torch.zeros((0, 128 if config == "c3" else 104),
                                                   device=device)

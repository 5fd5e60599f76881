"""Generate tests/golden/ref_cpu_golden.npz from the REFERENCE's own CPU code.

Runs the reference's cpu/ trainer (cpu/jl_transform.cpp, cpu/codebook.cpp),
compiled from the reference tree by oracle/Makefile into oracle/_ref, on small
seeded inputs and stores its outputs. These are the known answers that pin the
oracle (oracle/jhq_oracle.c) and the product's host training; the GPU box does
not need the reference tree because the vectors are committed.

    make -C oracle ref && python tests/golden/make_golden.py
"""
import os
import sys

import numpy as np

ROOT = os.path.dirname(os.path.dirname(os.path.dirname(os.path.abspath(__file__))))
sys.path.insert(0, ROOT)
from oracle import RefCPU  # noqa: E402


def main():
    r = RefCPU()
    rng = np.random.default_rng(20261201)
    out = {}
    # JLTransform(d, seed=42) rotation Pi (column-major), cpu/jl_transform.cpp:21-56
    for d in (16, 104):
        out[f"pi_d{d}"] = r.rotation(d, 42)
    # estimate_sigma + LloydMaxCodebook c1d, cpu/jl_transform.cpp:73-83, codebook.cpp:60-80
    x = rng.standard_normal((300, 16)).astype(np.float32) * 1.7
    out["sigma_x"] = x
    out["sigma"] = np.float32(r.sigma(x))
    for (d, M) in ((16, 2), (16, 4), (16, 8), (16, 16)):     # K1D = 256, 16, 4, 2 at B=8
        out[f"c1d_d{d}_M{M}"] = r.c1d(d, M, 8, out["sigma"])
    # encode / flat LUT / ADC / reconstruct, cpu/codebook.cpp:96-171
    y = (rng.standard_normal((200, 16)) * out["sigma"]).astype(np.float32)
    out["enc_y"] = y
    q = (rng.standard_normal(16) * out["sigma"]).astype(np.float32)
    out["enc_q"] = q
    for M in (2, 4, 8, 16):
        codes = r.encode(16, M, 8, out["sigma"], y)
        out[f"codes_M{M}"] = codes
        out[f"flat_lut_M{M}"] = r.flat_lut(16, M, 8, out["sigma"], q)
        out[f"adc_M{M}"] = r.adc(16, M, 8, out["sigma"], q, codes)
        out[f"recon_M{M}"] = r.reconstruct(16, M, 8, out["sigma"], codes)
    # train_1d_kmeans, cpu/codebook.cpp:8-58 (residual codebook, Kr = 16)
    vals = (rng.standard_normal(5000) * 0.3).astype(np.float32)
    out["km_vals"] = vals
    out["km_c16"] = r.kmeans1d(vals, 16)
    out["km_c4_small"] = r.kmeans1d(vals[:3], 4)    # n < Kr edge case
    path = os.path.join(os.path.dirname(os.path.abspath(__file__)), "ref_cpu_golden.npz")
    np.savez_compressed(path, **out)
    print("wrote", path, os.path.getsize(path), "bytes")


if __name__ == "__main__":
    main()

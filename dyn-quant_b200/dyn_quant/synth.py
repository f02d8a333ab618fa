"""Seeded synthetic weights and activations for the benchmark shapes.

The reference's benchmarks use Llama-2 7B/70B and Mixtral-8x7B GEMV shapes
(benchmarks/bench_latency.cu:100-107 of dyn-quant) with random data; no
dataset is involved.  These generators fix the draw order so that every
implementation (the kernels, the CPU oracle, the reference build) sees the
same inputs:

  W = default_rng(seed).standard_normal((d_out, d_in), float32) / sqrt(d_in)  -> f16
  x = default_rng(seed).standard_normal(d_in)          (or Student-t(3))
      idx = choice(d_in, round(frac*d_in), replace=False)
      x[idx] *= uniform(lo, hi, n) * choice([-1, 1], n)                        -> f16
"""
from __future__ import annotations

import numpy as np

# Benchmark shapes (d_out, d_in) and their outlier fractions.
SHAPES = {
    "llama2_7b_q": (4096, 4096, 0.02),
    "llama2_7b_gate": (11008, 4096, 0.01),
    "llama2_7b_up": (11008, 4096, 0.01),
    "llama2_7b_down": (4096, 11008, 0.01),
    "llama2_70b_q": (8192, 8192, 0.03),
    "llama2_70b_gate": (28672, 8192, 0.03),
    "llama2_70b_up": (28672, 8192, 0.03),
    "llama2_70b_down": (8192, 28672, 0.03),
    "mixtral_w1": (14336, 4096, 0.02),
    "mixtral_w3": (14336, 4096, 0.02),
    "mixtral_w2": (4096, 14336, 0.02),
}


def weights(d_out: int, d_in: int, seed: int = 0) -> np.ndarray:
    """FP16 weights N(0, 1/d_in) (std 1/sqrt(d_in)), row-major [d_out, d_in]."""
    rng = np.random.default_rng(seed)
    w = rng.standard_normal((d_out, d_in), dtype=np.float32)
    w /= np.float32(np.sqrt(d_in))
    return w.astype(np.float16)


def activation(d_in: int, frac: float, seed: int = 1, lo: float = 10.0, hi: float = 100.0,
               dist: str = "normal") -> np.ndarray:
    """FP16 activation vector with round(frac*d_in) outlier channels scaled by U[lo, hi] x (+-1)."""
    rng = np.random.default_rng(seed)
    if dist == "normal":
        x = rng.standard_normal(d_in)
    elif dist == "t3":
        x = rng.standard_t(3, d_in)
    else:
        raise ValueError(f"unknown dist {dist!r}")
    n = int(round(frac * d_in))
    if n:
        idx = rng.choice(d_in, n, replace=False)
        f = rng.uniform(lo, hi, n)
        s = rng.choice(np.array([-1.0, 1.0]), n)
        x[idx] *= f * s
    return x.astype(np.float16)


def activations(m: int, d_in: int, frac: float, seed: int = 1, **kw) -> np.ndarray:
    """[m, d_in] FP16 activations, token t drawn with seed + t."""
    return np.stack([activation(d_in, frac, seed + t, **kw) for t in range(m)])

"""Seeded synthetic datasets with the shapes of the benchmark configs.

The reference measures on BIGANN/Deep/GIST/OpenAI files that are not
available here; these generators stand in for them (same dimensions and value
ranges).  All return float16 numpy arrays [n, dim].

* ``gaussian``   -- i.i.d. N(0, 1) (config 1).
* ``sift_like``  -- Gaussian mixture of integer-valued points: centres uniform
  integers in [0, 128], per-dimension sigma 12, rounded and clipped to
  [0, 255] (configs 2 and 5).  Every value is exact in fp16 and every squared
  L2 distance is an exact integer below 2^24, so distances have many ties.
* ``relu_sphere`` -- mixture of 256 N(0, 1) centres, sigma 0.3, ReLU-clamped
  and L2-normalised (config 4, inner product).
"""
from __future__ import annotations

import numpy as np


def gaussian(n: int, dim: int, seed: int) -> np.ndarray:
    rng = np.random.default_rng(seed)
    return rng.standard_normal((n, dim), dtype=np.float32).astype(np.float16)


def sift_like(n: int, dim: int, seed: int, n_centers: int = 1024, sigma: float = 12.0,
              chunk: int = 1 << 20, center_seed: int | None = None) -> np.ndarray:
    """Queries of a base set use the base seed as ``center_seed`` (same mixture)."""
    crng = np.random.default_rng(seed if center_seed is None else center_seed)
    centers = crng.integers(0, 129, size=(n_centers, dim)).astype(np.float32)
    rng = np.random.default_rng(seed) if center_seed is not None else crng
    out = np.empty((n, dim), dtype=np.float16)
    for s in range(0, n, chunk):
        m = min(chunk, n - s)
        c = rng.integers(0, n_centers, size=m)
        x = centers[c] + rng.standard_normal((m, dim), dtype=np.float32) * np.float32(sigma)
        out[s:s + m] = np.clip(np.rint(x), 0, 255).astype(np.float16)
    return out


def relu_sphere(n: int, dim: int, seed: int, n_centers: int = 256, sigma: float = 0.3,
                chunk: int = 1 << 18, center_seed: int | None = None) -> np.ndarray:
    crng = np.random.default_rng(seed if center_seed is None else center_seed)
    centers = crng.standard_normal((n_centers, dim), dtype=np.float32)
    rng = np.random.default_rng(seed) if center_seed is not None else crng
    out = np.empty((n, dim), dtype=np.float16)
    for s in range(0, n, chunk):
        m = min(chunk, n - s)
        c = rng.integers(0, n_centers, size=m)
        x = centers[c] + rng.standard_normal((m, dim), dtype=np.float32) * np.float32(sigma)
        x = np.maximum(x, 0.0)
        nrm = np.linalg.norm(x, axis=1, keepdims=True)
        nrm[nrm == 0] = 1.0
        out[s:s + m] = (x / nrm).astype(np.float16)
    return out


def config_data(config: int, which: str = "base", n: int | None = None):
    """Base or query rows of a numbered benchmark config (1, 2, 4)."""
    if config == 1:
        return gaussian(n or (100_000 if which == "base" else 1000), 128, 0 if which == "base" else 1)
    if config == 2:
        if which == "base":
            return sift_like(n or 1_000_000, 128, 2)
        return sift_like(n or 10_000, 128, 3, center_seed=2)
    if config == 4:
        if which == "base":
            return relu_sphere(n or 1_000_000, 960, 6)
        return relu_sphere(n or 1000, 960, 7, center_seed=6)
    raise ValueError(f"no generator for config {config}")

"""Seeded synthetic embeddings for the IVF workloads (numpy ``default_rng``).

There is no public dataset on this path: every workload is a seeded stand-in
with the shapes, sizes and value distributions of the index it models.

* ``unit_gaussian``: entries i.i.d. N(0, 1), each row then L2-normalised.
* ``gaussian_mixture``: component means N(0, I_D) normalised to the unit sphere;
  each point is ``mean[c] + sigma * g / sqrt(D)`` with g ~ N(0, I_D) (so the
  noise has norm ~sigma, comparable to the unit mean), then renormalised.
  Component sizes are uniform, or Zipf(s)-skewed when ``zipf`` is given.
* ``shifted_means``: the means moved by N(0, offset^2 / D) per coordinate and
  renormalised, for an insert stream that drifts away from the trained centroids.
"""
from __future__ import annotations

import numpy as np


def _normalize(x: np.ndarray) -> np.ndarray:
    n = np.linalg.norm(x, axis=1, keepdims=True)
    n[n == 0] = 1.0
    x /= n
    return x


def unit_gaussian(n: int, d: int, rng: np.random.Generator) -> np.ndarray:
    """n rows of i.i.d. N(0,1) entries, L2-normalised (float32, C order)."""
    x = rng.standard_normal((n, d), dtype=np.float32)
    return _normalize(x)


def mixture_means(ncomp: int, d: int, rng: np.random.Generator) -> np.ndarray:
    return _normalize(rng.standard_normal((ncomp, d), dtype=np.float32))


def component_weights(ncomp: int, zipf: float | None) -> np.ndarray:
    if not zipf:
        return np.full(ncomp, 1.0 / ncomp)
    w = 1.0 / np.arange(1, ncomp + 1, dtype=np.float64) ** zipf
    return w / w.sum()


def gaussian_mixture(n: int, means: np.ndarray, sigma: float, rng: np.random.Generator,
                     zipf: float | None = None, chunk: int = 1 << 18):
    """n unit-norm rows drawn from the mixture; returns (X float32[n, d], comp int32[n])."""
    ncomp, d = means.shape
    comp = rng.choice(ncomp, size=n, p=component_weights(ncomp, zipf)).astype(np.int32)
    x = np.empty((n, d), np.float32)
    scale = np.float32(sigma / np.sqrt(d))
    for b in range(0, n, chunk):
        e = min(n, b + chunk)
        g = rng.standard_normal((e - b, d), dtype=np.float32)
        g *= scale
        g += means[comp[b:e]]
        x[b:e] = _normalize(g)
    return x, comp


def shifted_means(means: np.ndarray, offset: float, rng: np.random.Generator) -> np.ndarray:
    d = means.shape[1]
    m = means + rng.standard_normal(means.shape, dtype=np.float32) * np.float32(offset / np.sqrt(d))
    return _normalize(m.astype(np.float32))

"""Seeded synthetic inputs for the benchmark configurations (host-sized ones).

Test infrastructure (see ``oracle/__init__.py``).  The reference publishes no
dataset for this path; these generators stand in with the shapes and value
distributions of the benchmark configurations:

* single linear: ``W ~ N(0, 0.02^2)`` 1024x1024, ``X ~ N(0, 1)`` 2048x1024
  with 8 random input channels scaled x20, ``H = X^T X / tokens``;
* pivoted QR: ``A = G diag(s)``, ``G ~ N(0, 1)``, ``s_k = 10^(-6k/n)`` in a
  shuffled column order, optionally with 256 columns replaced by random
  linear combinations of the others (rank-deficient variant).
"""

from __future__ import annotations

import numpy as np


def single_linear(seed: int = 0, m: int = 1024, n: int = 1024, tokens: int = 2048,
                  n_outliers: int = 8):
    rng = np.random.Generator(np.random.PCG64(seed))
    w = (rng.standard_normal((m, n)) * 0.02).astype(np.float32)
    x = rng.standard_normal((tokens, n)).astype(np.float32)
    cols = rng.choice(n, size=n_outliers, replace=False)
    x[:, cols] *= np.float32(20.0)
    return w, x


def qr_matrix(seed: int = 1, m: int = 4096, n: int = 4096, rank_deficient: bool = False,
              n_dependent: int = 256):
    rng = np.random.Generator(np.random.PCG64(seed))
    g = rng.standard_normal((m, n)).astype(np.float32)
    s = (10.0 ** (-6.0 * np.arange(n) / n)).astype(np.float32)
    s = s[rng.permutation(n)]
    a = (g * s[None, :]).astype(np.float32)
    if rank_deficient:
        dep = rng.choice(n, size=min(n_dependent, n // 2), replace=False)
        indep = np.setdiff1d(np.arange(n), dep)
        coef = rng.standard_normal((indep.shape[0], dep.shape[0])).astype(np.float32)
        coef /= np.sqrt(np.float32(indep.shape[0]))
        a[:, dep] = (a[:, indep] @ coef).astype(np.float32)
    return a

"""process_hessian's eigh branch (gptq_ref.py:95-133) on the device.

Every step runs on the library's kernels: the Jacobi eigensolver
(``gq_syevj``), the unpivoted and the pivoted Householder QR (``gq_qrcp``).
Reference semantics against vectors produced by the reference's own code:
permutations equal, |R| equal to float32 eigensolver precision (eigenvector
and QR row signs are implementation choices and cancel in GPTQ, which divides
each row's error by its own diagonal).  Intended semantics: R^T R equals the
permuted inverse Hessian."""

import os

import numpy as np
import pytest

pytestmark = pytest.mark.gpu

from jax_gptq_b200.config import QuantConfig
from jax_gptq_b200.gptq_ref import process_hessian

GOLDEN = os.path.join(os.path.dirname(__file__), "golden", "eigh_golden.npz")
MODES = ("none", "diag_h", "pivot_sqrt_h", "pivot_sqrt_hinv_smallest")


@pytest.mark.parametrize("name", ["full", "deficient"])
@pytest.mark.parametrize("mode", MODES)
def test_reference_semantics_match_golden(name, mode):
    g = np.load(GOLDEN)
    h = g[f"eigh_{name}_h"]
    r, p = process_hessian(h, QuantConfig(solver_mode="eigh", ordering_mode=mode), panel_size=8)
    gr, gp = g[f"eigh_{name}_{mode}_r"], g[f"eigh_{name}_{mode}_perm"]
    assert np.array_equal(p, gp)
    assert r.shape == gr.shape
    rank = g[f"eigh_{name}_pivot_sqrt_hinv_smallest_r"].shape[0]
    if rank < h.shape[0] and mode != "pivot_sqrt_hinv_smallest":
        # the clamped gather repeats the last kept eigen-column: R after the
        # first repeat is any valid completion, only R^T R = E^T lam^-1 E
        # (E selects columns clip(perm, rank - 1)) is defined
        lam = np.linalg.eigvalsh(h.astype(np.float64))[::-1][:rank]
        c = np.clip(gp, 0, rank - 1)
        gram = np.where(c[:, None] == c[None, :], 1.0 / lam[c][:, None], 0.0)
        rr = r.astype(np.float64)
        err = np.abs(rr.T @ rr - gram).max() / np.abs(gram).max()
        assert err < 1e-3, err
        return
    tol = 2e-3 * float(np.abs(gr).max())
    assert np.allclose(np.abs(r), np.abs(gr), atol=tol), float(np.abs(np.abs(r) - np.abs(gr)).max())


@pytest.mark.parametrize("mode", MODES)
def test_intended_semantics_factor_the_permuted_inverse(mode):
    g = np.load(GOLDEN)
    h = g["eigh_full_h"].astype(np.float64)
    cfg = QuantConfig(solver_mode="eigh", ordering_mode=mode, semantics="intended")
    r, p = process_hessian(g["eigh_full_h"], cfg, panel_size=8)
    r = r.astype(np.float64)
    hinv = np.linalg.inv(h)[p][:, p]
    assert np.allclose(np.tril(r, -1), 0.0, atol=1e-6 * np.abs(r).max())
    err = np.abs(r.T @ r - hinv).max() / np.abs(hinv).max()
    assert err < 1e-4, err


def test_eigh_rejects_unknown_ordering():
    with pytest.raises(ValueError):
        process_hessian(np.eye(8, dtype=np.float32),
                        QuantConfig(solver_mode="eigh", ordering_mode="bogus"))


@pytest.mark.parametrize("n", [64, 257, 512])
def test_jacobi_eigensolver_matches_float64(n):
    """gq_syevj (parallel cyclic Jacobi) against numpy's float64 eigh:
    eigenvalues within 1e-5 of the largest, A V = V diag(w) within 1e-5,
    ascending order, and V^T V = I within 3e-5: each column of V takes
    about n float32 rotations per sweep, and their rounding adds up (1.05e-5
    measured at n = 512)."""
    import torch
    from jax_gptq_b200.gptq_ref import eigh
    rng = np.random.default_rng(n)
    x = rng.standard_normal((2 * n, n)) * rng.lognormal(0, 1, n)
    a = (x.T @ x / (2 * n)).astype(np.float32)
    w, v = eigh(torch.from_numpy(a).cuda())
    w, v = w.cpu().numpy().astype(np.float64), v.cpu().numpy().astype(np.float64)
    a64 = a.astype(np.float64)
    ref = np.linalg.eigvalsh(a64)
    top = np.abs(ref).max()
    assert np.all(np.diff(w) >= 0)
    assert np.abs(w - ref).max() <= 1e-5 * top, np.abs(w - ref).max() / top
    assert np.abs(a64 @ v - v * w[None, :]).max() <= 1e-5 * top
    assert np.abs(v.T @ v - np.eye(n)).max() <= 3e-5


def test_unpivoted_householder_qr_matches_float64():
    """The reduced R of the library's Householder QR without pivoting (the
    eigh branch's QR): upper triangular, R^T R = A^T A within 1e-5 and |R|
    equal to numpy's float64 R up to row signs."""
    import importlib
    import torch
    BQ = importlib.import_module("jax_gptq_b200.pallas.blocked_pivoted_qr")
    rng = np.random.default_rng(9)
    for (m, n) in [(300, 200), (128, 192), (256, 256)]:
        a = rng.standard_normal((m, n)).astype(np.float32)
        r = BQ.householder_qr_r(torch.from_numpy(a).cuda()).cpu().numpy().astype(np.float64)
        assert r.shape == (min(m, n), n)
        assert np.array_equal(np.tril(r, -1), np.zeros_like(r))
        a64 = a.astype(np.float64)
        gram = a64.T @ a64
        assert np.abs(r.T @ r - gram).max() <= 1e-5 * np.abs(gram).max()
        r64 = np.linalg.qr(a64, mode="r")
        assert np.allclose(np.abs(r), np.abs(r64), atol=1e-4 * np.abs(r64).max())

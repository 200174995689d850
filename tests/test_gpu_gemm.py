"""GPU checks of the float32-accurate GEMMs (tcgen05 3xTF32 and CUDA-core).

Tolerance: relative Frobenius error <= 2e-6 against a float64 product for the
3xTF32 tensor-core kernel (about 2^-21 per product), <= 1e-6 for the CUDA-core
kernel.
"""

import ctypes

import numpy as np
import pytest
import torch

pytestmark = pytest.mark.gpu

from jax_gptq_b200 import _arrays as A
from jax_gptq_b200 import _lib


def _status():
    v = ctypes.c_int(-1)
    _lib.call("gq_device_status", ctypes.byref(v), 1, A.stream())
    return v.value


@pytest.mark.parametrize("M,N,K,tb,alpha,beta", [
    (128, 128, 32, 1, 1.0, 0.0), (256, 384, 128, 1, -1.0, 1.0), (300, 200, 76, 1, 0.5, 2.0),
    (1000, 520, 640, 1, 1.0, 0.0), (129, 1024, 36, 1, -1.0, 1.0), (4096, 256, 128, 1, -1.0, 1.0),
    (512, 512, 4096, 1, 1.0, 0.0), (96, 256, 128, 1, -1.0, 1.0), (1, 384, 64, 1, 1.0, 0.0),
    (33, 130, 96, 1, 2.0, -1.0)])
def test_tf32x3_matches_float64(M, N, K, tb, alpha, beta):
    rng = np.random.default_rng(M + N + K)
    a = rng.standard_normal((M, K)).astype(np.float32)
    b = rng.standard_normal((N, K) if tb else (K, N)).astype(np.float32)
    c = rng.standard_normal((M, N)).astype(np.float32)
    ref = alpha * (a.astype(np.float64) @ (b.T if tb else b).astype(np.float64)) + beta * c
    at, bt, ct = (torch.from_numpy(x).cuda() for x in (a, b, c))
    _lib.call("gq_gemm_f32_tc", tb, M, N, K, alpha, A.ptr(at), K, A.ptr(bt), bt.shape[1], beta,
              A.ptr(ct), N, 0, A.stream())
    assert _status() == 0
    got = ct.cpu().numpy()
    rel = np.linalg.norm(got - ref) / np.linalg.norm(ref)
    assert rel <= 2e-6, rel


def test_tf32x3_lower_tiles_only():
    M = N = 384
    K = 64
    rng = np.random.default_rng(3)
    p = rng.standard_normal((M, K)).astype(np.float32)
    c = np.zeros((M, N), np.float32)
    pt, ct = torch.from_numpy(p).cuda(), torch.from_numpy(c).cuda()
    _lib.call("gq_gemm_f32_tc", 1, M, N, K, 1.0, A.ptr(pt), K, A.ptr(pt), K, 0.0, A.ptr(ct), N, 1,
              A.stream())
    got = ct.cpu().numpy()
    ref = p.astype(np.float64) @ p.T
    low = np.tril(np.ones((M, N), bool))
    assert np.allclose(got[low], ref[low], rtol=1e-5, atol=1e-4)
    # tiles strictly above the diagonal are untouched
    assert np.all(got[:128, 256:] == 0.0)


def test_nn_layout_is_rejected_by_the_tensor_core_entry():
    a = torch.zeros((128, 64), device="cuda")
    with pytest.raises(ValueError, match="gq_gemm_f32_tc"):
        _lib.call("gq_gemm_f32_tc", 0, 128, 128, 64, 1.0, A.ptr(a), 64, A.ptr(a), 128, 0.0,
                  A.ptr(a), 128, 0, A.stream())


def test_dispatcher_uses_exact_zero_for_zero_operand():
    """alpha * A @ 0 + C == C bit for bit (the U = I sweep relies on it)."""
    rng = np.random.default_rng(4)
    a = rng.standard_normal((512, 128)).astype(np.float32)
    b = np.zeros((640, 128), np.float32)
    c = rng.standard_normal((512, 640)).astype(np.float32)
    at, bt, ct = (torch.from_numpy(x).cuda() for x in (a, b, c))
    for tb, ldb in ((1, 128), (0, 640)):
        _lib.call("gq_sgemm", 0, tb, 512, 640, 128, -1.0, A.ptr(at), 128, A.ptr(bt), ldb, 1.0,
                  A.ptr(ct), 640, 0, A.stream())
        assert np.array_equal(ct.cpu().numpy(), c)


def test_simt_matches_float64():
    rng = np.random.default_rng(5)
    for (M, N, K, ta, tb) in [(130, 70, 33, 1, 0), (257, 129, 65, 0, 1)]:
        a = rng.standard_normal((K, M) if ta else (M, K)).astype(np.float32)
        b = rng.standard_normal((N, K) if tb else (K, N)).astype(np.float32)
        ref = (a.T if ta else a).astype(np.float64) @ (b.T if tb else b)
        c = torch.zeros((M, N), device="cuda")
        at, bt = torch.from_numpy(a).cuda(), torch.from_numpy(b).cuda()
        _lib.call("gq_sgemm_simt", ta, tb, M, N, K, 1.0, A.ptr(at), at.shape[1], A.ptr(bt),
                  bt.shape[1], 0.0, A.ptr(c), N, 0, A.stream())
        rel = np.linalg.norm(c.cpu().numpy() - ref) / np.linalg.norm(ref)
        assert rel <= 1e-6, rel

"""Failure detection on the GPU without a fault.

Every device-side wait in the tensor-core kernels is bounded.  These tests
shorten the bound to 50 ms (``gq_set_wait_limit_ns``), run a kernel whose
wait nothing satisfies through the same bounded-wait code as the statistics
kernels and the fp32 GEMM (``gq_test_expire_wait``), and check that the wait
gives up, the host reads GQ_ETIMEOUT (``DeviceTimeout``), and the context
stays usable.  Nothing traps, faults or hangs: the kernel returns after the
bound.
"""

import time

import numpy as np
import pytest
import torch

pytestmark = pytest.mark.gpu

from jax_gptq_b200 import _arrays as A
from jax_gptq_b200 import _lib
from jax_gptq_b200 import stats


@pytest.fixture
def short_wait_limit():
    _lib.check_device()  # start from a clean status word
    _lib.call("gq_set_wait_limit_ns", 50_000_000)
    try:
        yield 0.05
    finally:
        _lib.call("gq_set_wait_limit_ns", 2_000_000_000)


@pytest.mark.parametrize("unit", [0, 1])
def test_expired_wait_returns_timeout_status(short_wait_limit, unit):
    obs = torch.full((1,), -1, dtype=torch.int32, device="cuda")
    t0 = time.perf_counter()
    _lib.call("gq_test_expire_wait", unit, A.ptr(obs), A.stream())
    with pytest.raises(_lib.DeviceTimeout, match="bounded device-side wait expired"):
        _lib.check_device()
    elapsed = time.perf_counter() - t0
    assert obs.item() == 1
    assert short_wait_limit <= elapsed < 1.5, elapsed
    _lib.check_device()  # the word was cleared by the check


def test_context_usable_after_expired_waits(short_wait_limit):
    obs = torch.zeros((1,), dtype=torch.int32, device="cuda")
    _lib.call("gq_test_expire_wait", 0, A.ptr(obs), A.stream())
    _lib.call("gq_test_expire_wait", 1, A.ptr(obs), A.stream())
    with pytest.raises(_lib.DeviceTimeout):
        _lib.check_device()
    _lib.call("gq_set_wait_limit_ns", 2_000_000_000)
    gen = torch.Generator(device="cuda").manual_seed(3)
    x = torch.randn((2048, 384), generator=gen, device="cuda").to(torch.bfloat16)
    h = torch.empty((384, 384), dtype=torch.float32, device="cuda")
    stats.syrk_into(h, x, accumulate=False)
    xd = x.double()
    ref = xd.T @ xd
    assert (torch.linalg.norm(h.double() - ref) / torch.linalg.norm(ref)).item() < 1e-5
    a = torch.randn((256, 128), generator=gen, device="cuda")
    b = torch.randn((256, 128), generator=gen, device="cuda")
    c = torch.zeros((256, 256), device="cuda")
    _lib.call("gq_gemm_f32_tc", 1, 256, 256, 128, 1.0, A.ptr(a), 128, A.ptr(b), 128, 0.0,
              A.ptr(c), 256, 0, A.stream())
    ref2 = a.double() @ b.double().T
    assert (torch.linalg.norm(c.double() - ref2) / torch.linalg.norm(ref2)).item() < 2e-6
    _lib.check_device()


def test_wait_limit_range_is_checked():
    with pytest.raises(ValueError, match="outside"):
        _lib.call("gq_set_wait_limit_ns", 10)
    with pytest.raises(ValueError, match="outside"):
        _lib.call("gq_set_wait_limit_ns", 10 ** 12)

"""The allocation-free GPTQ sweep, checked against the workspace version.

``gq_gptq_sweep_static`` exists for callers that cannot allocate device
memory themselves -- typically a host framework that keeps nearly all GPU
memory in its own pool, where a library-side cudaMalloc would fail.  It takes
its scratch from one static device buffer instead of a caller workspace.
These tests call it through the C ABI twice in a row (different shapes, so
the second call starts from the first call's leftovers) and require the
same codes, scales, zeros, group indices and dequantized weights as
``gq_gptq_sweep`` with a caller-provided workspace (bit-exact: both run the
same kernels on the same inputs).  The file is named to be collected last.
"""

import numpy as np
import pytest
import torch

pytestmark = pytest.mark.gpu

from jax_gptq_b200 import _arrays as A
from jax_gptq_b200 import _lib
from jax_gptq_b200.config import QuantConfig
from jax_gptq_b200.gptq_ref import factor_hessian

STATIC_BYTES = 32 * 1024 * 1024


def _problem(m, n, seed):
    rng = np.random.default_rng(seed)
    w = torch.from_numpy((rng.standard_normal((m, n)) * 0.02).astype(np.float32)).cuda()
    x = (rng.standard_normal((4 * n, n)) * rng.lognormal(0, 1, n)).astype(np.float32)
    h = x.T @ x
    f = factor_hessian(h, QuantConfig(ordering_mode="diag_h", semantics="intended"))
    return w, f.u, f.perm


def _outputs(m, n, g):
    return {
        "dequant": torch.empty((m, n), dtype=torch.float32, device="cuda"),
        "codes": torch.empty((m, n), dtype=torch.uint8, device="cuda"),
        "scales": torch.empty((m, n // g), dtype=torch.float32, device="cuda"),
        "zeros": torch.empty((m, n // g), dtype=torch.float32, device="cuda"),
        "g_idx": torch.empty((n,), dtype=torch.int32, device="cuda"),
    }


def _sweep(static, w, u, perm, bits, g):
    m, n = w.shape
    o = _outputs(m, n, g)
    common = (A.ptr(w), m, n, n, None, A.ptr(u), n, A.ptr(perm), bits, g, 0, 128, None, None, 0,
              A.ptr(o["dequant"]), A.ptr(o["codes"]), A.ptr(o["scales"]), A.ptr(o["zeros"]),
              A.ptr(o["g_idx"]))
    if static:
        _lib.call("gq_gptq_sweep_static", *common, A.stream())
    else:
        ws = A.workspace(_lib.lib().gq_gptq_sweep_workspace_size(m, n))
        _lib.call("gq_gptq_sweep", *common, A.ptr(ws), ws.numel(), A.stream())
    torch.cuda.synchronize()
    return {k: v.cpu().numpy() for k, v in o.items()}


def test_static_sweep_matches_workspace_sweep_on_two_calls():
    for (m, n, bits, g, seed) in [(512, 1024, 4, 128, 1), (200, 768, 3, 64, 2)]:
        w, u, perm = _problem(m, n, seed)
        ref = _sweep(False, w, u, perm, bits, g)
        got = _sweep(True, w, u, perm, bits, g)
        for key in ref:
            assert np.array_equal(got[key], ref[key]), (m, n, key)


def test_static_sweep_rejects_sizes_beyond_its_buffer():
    m, n = 4096, 4096
    assert _lib.lib().gq_gptq_sweep_workspace_size(m, n) > STATIC_BYTES
    w = torch.zeros((1, 1), device="cuda")
    with pytest.raises(ValueError, match="static buffer"):
        _lib.call("gq_gptq_sweep_static", A.ptr(w), m, n, n, None, A.ptr(w), n, None, 4, 128, 0,
                  128, None, None, 0, None, None, None, None, None, A.stream())

"""Kernel-backend selection -- compatibility shim for ``src/jax_gptq/pallas/backend.py:1-49``.

The reference dispatches between Pallas GPU/TPU kernels and a dense JAX
path through ``JAX_GPTQ_USE_PALLAS`` and ``JAX_GPTQ_KERNEL_BACKEND``.  This
package has exactly one backend -- the sm_100a CUDA library -- so the
variables are read and validated (same error text) but select nothing.
"""

from __future__ import annotations

import os

VALID_KERNEL_BACKENDS = {"auto", "gpu", "tpu", "reference"}


def pallas_enabled() -> bool:
    return os.environ.get("JAX_GPTQ_USE_PALLAS", "0") == "1"


def requested_kernel_backend() -> str:
    backend = os.environ.get("JAX_GPTQ_KERNEL_BACKEND", "auto").lower()
    if backend not in VALID_KERNEL_BACKENDS:
        raise ValueError(
            "JAX_GPTQ_KERNEL_BACKEND must be one of "
            f"{sorted(VALID_KERNEL_BACKENDS)}, got {backend!r}")
    return backend


def runtime_backend() -> str:
    return "cuda-sm100a"


def selected_kernel_backend() -> str:
    requested_kernel_backend()  # validate like the reference
    return "cuda-sm100a"


def describe_backend_selection() -> dict[str, object]:
    return {
        "runtime_backend": runtime_backend(),
        "pallas_enabled": pallas_enabled(),
        "requested_kernel_backend": requested_kernel_backend(),
        "selected_kernel_backend": selected_kernel_backend(),
    }

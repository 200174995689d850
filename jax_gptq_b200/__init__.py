"""B200-native (sm_100a) implementation of the jax_gptq quantization hot path.

Drop-in for ``src/jax_gptq/__init__.py``: the same public names with the
same argument meaning and ``ValueError`` contracts.  The arithmetic runs in
``libgq.so`` (hand-written CUDA for sm_100a, C ABI in ``include/gq.h``);
there is no CPU fallback.
"""

import os

# A layer set runs one stream per input group plus the factor's side streams;
# with the driver's default of 8 hardware work queues, streams that share a
# queue wait on one another's pending dependencies.  Raise it to the maximum
# unless the host process chose a value (read when the CUDA context is
# created, so it has no effect once CUDA is initialised).
os.environ.setdefault("CUDA_DEVICE_MAX_CONNECTIONS", "32")

from .config import QuantConfig  # noqa: E402
from .gptq_ref import gptq_forward_step, process_hessian  # noqa: E402
from .noop_quant import run_noop_quantization  # noqa: E402
from .quant import quantize_dequantize  # noqa: E402
from .qronos_ref import qronos_single_layer_update_ref  # noqa: E402
from .stats import h_g_from_activations  # noqa: E402

__all__ = [
    "QuantConfig",
    "quantize_dequantize",
    "h_g_from_activations",
    "gptq_forward_step",
    "qronos_single_layer_update_ref",
    "run_noop_quantization",
    "process_hessian",
]

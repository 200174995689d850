"""B200-native (sm_100a) implementation of the jax_gptq quantization hot path.

Drop-in for ``src/jax_gptq/__init__.py``: the same public names with the
same argument meaning and ``ValueError`` contracts.  The arithmetic runs in
``libgq.so`` (hand-written CUDA for sm_100a, C ABI in ``include/gq.h``);
there is no CPU fallback.
"""

from .config import QuantConfig
from .gptq_ref import gptq_forward_step, process_hessian
from .noop_quant import run_noop_quantization
from .quant import quantize_dequantize
from .qronos_ref import qronos_single_layer_update_ref
from .stats import h_g_from_activations

__all__ = [
    "QuantConfig",
    "quantize_dequantize",
    "h_g_from_activations",
    "gptq_forward_step",
    "qronos_single_layer_update_ref",
    "run_noop_quantization",
    "process_hessian",
]

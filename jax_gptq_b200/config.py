"""Quantization config -- mirrors ``src/jax_gptq/config.py:1-25``.

Same fields, defaults and literal modes as the reference's frozen
``QuantConfig``, plus one field:

``semantics`` -- ``"reference"`` (default) reproduces what the reference
actually returns: ``process_hessian`` yields the identity factor (its
Cholesky branch always falls back, gptq_ref.py:85-92), ``gptq_forward_step``
and ``qronos_single_layer_update_ref`` are round-to-nearest.  ``"intended"``
runs the algorithms the reference describes: a working damped Cholesky,
the real GPTQ column sweep and the Qronos update.
"""

from __future__ import annotations

from dataclasses import dataclass
from typing import Literal

SolverMode = Literal["chol", "eigh"]
OrderingMode = Literal["none", "diag_h", "pivot_sqrt_h", "pivot_sqrt_hinv_smallest"]
TruncationMode = Literal["abs", "percent", "mean_top32", "energy"]
Semantics = Literal["reference", "intended"]


@dataclass(frozen=True)
class QuantConfig:
    w_bits: int = 4
    group_size: int = 128
    sym: bool = False
    damp_percent: float = 0.01
    rank_eps: float = 1e-5
    truncation_mode: TruncationMode = "abs"
    truncation_value: float = 1e-5
    solver_mode: SolverMode = "chol"
    ordering_mode: OrderingMode = "none"
    semantics: Semantics = "reference"

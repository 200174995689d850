"""CPU oracle for the jax_gptq quantization hot path -- TEST INFRASTRUCTURE ONLY.

This package is a numpy/scipy restatement of the reference's algorithms
(davidtweedle/jax_gptq, ``src/jax_gptq``), used as the checker for the CUDA
library and as the timed CPU baseline.  Only ``tests/``,
``__graft_entry__.smoke()`` and ``bench.py`` (its CPU baseline and
``--impl reference`` legs) may import it; the product package
``jax_gptq_b200`` never does.

Pinning (how far each restatement is trusted):

* ``oracle.quant``, ``oracle.stats``, ``oracle.gptq`` (reference semantics),
  ``oracle.qronos`` (reference semantics) and ``oracle.qr`` (compiled-path
  semantics) are pinned against golden vectors in ``tests/golden/`` that
  ``tests/golden/make_golden.py`` produced by running the reference's own,
  unmodified source files under a numpy-backed ``jax`` stand-in (JAX itself
  is not installable offline).  The QR restatement is additionally pinned by
  the known-answer cases of the reference's ``tests/test_blocked_pivoted_qr.py``.
  Those vectors carry numpy's fp32 rounding, not XLA's: control flow, op
  order, pivots and integer codes are pinned; fp32 values agree to rounding.
* ``oracle.gptq`` / ``oracle.qronos`` "intended" semantics (a working damped
  Cholesky, the real GPTQ column sweep, the Qronos first-step correction)
  have no counterpart in the reference, whose GPTQ/Qronos are placeholders
  (``gptq_ref.py:142-155``, ``qronos_ref.py:14-25``).  They follow the
  published algorithms and are checked only by properties (they reduce to
  the reference exactly when the inverse-Hessian factor is the identity).
  Parity for that mode is unpinned by the reference.
"""

"""A numpy-backed stand-in for the few ``jax`` entry points jax_gptq touches.

Test infrastructure only (see ``jax/numpy/__init__.py``).  ``jit`` and
``register_dataclass`` are identities, ``lax.cond`` / ``lax.fori_loop`` run
eagerly, and ``jax.experimental`` is deliberately absent so the reference's
optional Pallas imports take their ``ImportError`` branch.
"""

from __future__ import annotations

import numpy as _np

from . import numpy  # noqa: F401
from . import lax  # noqa: F401
from . import tree_util  # noqa: F401

ShapeDtypeStruct = None


def jit(fun=None, **_kwargs):
    if fun is None:
        return lambda f: f
    return fun


def device_get(x):
    return _np.asarray(x)


def default_backend():
    return "cpu"


def devices():
    return ["cpu:0"]

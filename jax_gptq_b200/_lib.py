"""ctypes binding of ``libgq.so`` (the C ABI declared in ``include/gq.h``).

The library must have been built in-tree (``python -m jax_gptq_b200.csrc.build``
or ``__graft_entry__.build()``).  There is no fallback: if it is missing, or
the process has no CUDA device, the calls raise.
"""

from __future__ import annotations

import ctypes
import os
from ctypes import c_double, c_float, c_int, c_int64, c_void_p

_HERE = os.path.dirname(os.path.abspath(__file__))
LIB_PATH = os.path.join(_HERE, "libgq.so")

GQ_OK = 0
GQ_EINVAL = 1
GQ_ENOTPD = 2
GQ_ETIMEOUT = 3
GQ_ECUDA = 4
GQ_EUNSUPPORTED = 5
GQ_ENCCL = 6

_P = c_void_p
# name -> (restype, argtypes)
SIGNATURES = {
    "gq_version": (c_int, []),
    "gq_last_error": (ctypes.c_char_p, []),
    "gq_launch_count": (ctypes.c_longlong, []),
    "gq_set_cta_budget": (c_int, [c_int]),
    "gq_set_sweep_row_groups": (c_int, [c_int]),
    "gq_set_pair_kernels": (c_int, [c_int]),
    "gq_packed_words": (c_int64, [c_int64, c_int]),
    "gq_pack_codes": (c_int, [_P, c_int64, c_int64, c_int64, c_int, _P, c_int64, _P]),
    "gq_unpack_dequant": (c_int, [_P, c_int64, c_int64, c_int64, c_int, c_int, _P, _P, c_int64,
                                  _P, _P, _P, _P]),
    "gq_nccl_unique_id": (c_int, [_P, c_int64]),
    "gq_handle_create": (c_int, [c_int, _P, ctypes.POINTER(_P)]),
    "gq_handle_create_nccl": (c_int, [c_int, _P, c_int, c_int, ctypes.POINTER(_P)]),
    "gq_handle_destroy": (c_int, [_P]),
    "gq_handle_ranks": (c_int, [_P, ctypes.POINTER(c_int), ctypes.POINTER(c_int)]),
    "gq_allreduce_sum_f32": (c_int, [_P, _P, c_int64, _P]),
    "gq_allreduce_sym_f32": (c_int, [_P, _P, c_int64, c_int64, _P, _P]),
    "gq_sym_packed_size": (c_int64, [c_int64]),
    "gq_sym_pack_upper": (c_int, [_P, c_int64, c_int64, _P, _P]),
    "gq_sym_unpack_upper": (c_int, [_P, c_int64, _P, c_int64, _P]),
    "gq_comm_check": (c_int, [_P, c_int]),
    "gq_handle_abort": (c_int, [_P]),
    "gq_rtn": (c_int, [_P, c_int64, c_int64, c_int64, _P, c_int, c_int, c_int, _P, _P, _P, _P, _P]),
    "gq_sgemm": (c_int, [c_int, c_int, c_int64, c_int64, c_int64, c_float, _P, c_int64, _P, c_int64,
                         c_float, _P, c_int64, c_int, _P]),
    "gq_sgemm_simt": (c_int, [c_int, c_int, c_int64, c_int64, c_int64, c_float, _P, c_int64, _P,
                              c_int64, c_float, _P, c_int64, c_int, _P]),
    "gq_gemm_f32_tc": (c_int, [c_int, c_int64, c_int64, c_int64, c_float, _P, c_int64, _P, c_int64,
                               c_float, _P, c_int64, c_int, _P]),
    "gq_syrk_bf16": (c_int, [_P, c_int64, c_int64, c_int64, _P, c_int64, c_int, _P]),
    "gq_gemm_tn_bf16": (c_int, [_P, c_int64, _P, c_int64, c_int64, c_int64, c_int64, _P, c_int64,
                                c_int, _P]),
    "gq_syrk_f32": (c_int, [_P, c_int64, c_int64, c_int64, _P, c_int64, c_int, _P]),
    "gq_gemm_tn_f32": (c_int, [_P, c_int64, _P, c_int64, c_int64, c_int64, c_int64, _P, c_int64,
                               c_int, _P]),
    "gq_symmetrize_upper": (c_int, [_P, c_int64, c_int64, _P]),
    "gq_act_order_perm": (c_int, [_P, c_int64, c_int64, c_int, _P, _P]),
    "gq_hessian_factor_workspace_size": (c_int64, [c_int64]),
    "gq_factor_from_x_workspace_size": (c_int64, [c_int64, c_int64]),
    "gq_factor_from_x_attempt": (c_int, [_P, c_int64, c_int64, c_int64, c_int, c_double, c_int,
                                         _P, c_int64, _P, _P, c_int64, _P, _P, _P]),
    "gq_hessian_factor": (c_int, [_P, c_int64, c_int64, _P, c_double, _P, c_int64, _P, _P, c_int64,
                                  ctypes.POINTER(c_int), _P]),
    "gq_hessian_factor_attempt": (c_int, [_P, c_int64, c_int64, _P, c_double, c_int, _P, c_int64,
                                          _P, _P, c_int64, _P, _P]),
    "gq_hessian_prepare": (c_int, [_P, c_int64, c_int64, _P, c_double, c_int, _P, _P, _P, _P]),
    "gq_inv_chol_workspace_size": (c_int64, [c_int64]),
    "gq_inv_chol": (c_int, [_P, c_int64, c_int64, _P, c_int64, _P, _P]),
    "gq_reverse_lower": (c_int, [_P, c_int64, c_int64, _P, c_int64, _P]),
    "gq_sgemm_tri": (c_int, [c_int, c_int, c_int64, c_int64, c_int64, c_float, _P, c_int64, _P,
                             c_int64, c_float, _P, c_int64, c_int, _P]),
    "gq_gptq_sweep_workspace_size": (c_int64, [c_int64, c_int64]),
    "gq_gptq_sweep": (c_int, [_P, c_int64, c_int64, c_int64, _P, _P, c_int64, _P, c_int, c_int, c_int,
                              c_int, _P, _P, c_int, _P, _P, _P, _P, _P, _P, c_int64, _P]),
    "gq_device_status": (c_int, [ctypes.POINTER(c_int), c_int, _P]),
    "gq_check_device": (c_int, [_P]),
    "gq_set_wait_limit_ns": (c_int, [ctypes.c_uint64]),
    "gq_test_expire_wait": (c_int, [c_int, _P, _P]),
    "gq_gptq_sweep_static": (c_int, [_P, c_int64, c_int64, c_int64, _P, _P, c_int64, _P, c_int,
                                     c_int, c_int, c_int, _P, _P, c_int, _P, _P, _P, _P, _P, _P]),
    "gq_qrcp_workspace_size": (c_int64, [c_int64, c_int64, c_int]),
    "gq_qrcp": (c_int, [_P, c_int64, c_int64, c_int64, c_int, c_int, c_int, _P, _P, c_int64, _P, _P,
                        ctypes.POINTER(c_int), _P, c_int64, _P]),
    "gq_qr_factor_panel": (c_int, [_P, c_int64, c_int64, c_int64, _P, _P, c_int64, c_int, c_int, c_int,
                                   _P, _P, _P, ctypes.POINTER(c_int), _P, c_int64, _P]),
    "gq_qr_apply_panel": (c_int, [_P, c_int64, c_int64, c_int64, _P, c_int64, _P, c_int64, c_int, _P,
                                  _P]),
    "gq_syevj_workspace_size": (c_int64, [c_int64]),
    "gq_syevj": (c_int, [_P, c_int64, c_int64, _P, _P, c_int64, c_int, ctypes.POINTER(c_int), _P,
                         c_int64, _P]),
    "gq_masked_nll_workspace_size": (c_int64, [c_int64, c_int64]),
    "gq_masked_nll": (c_int, [_P, c_int, c_int64, c_int64, c_int64, _P, _P, _P, _P, c_int64, _P]),
    "gq_qronos_workspace_size": (c_int64, [c_int64, c_int64]),
    "gq_qronos": (c_int, [_P, _P, c_int64, c_int64, _P, _P, _P, _P, c_int, c_int, c_int, c_int, _P,
                          _P, _P, _P, _P, _P, c_int64, _P]),
}


class GQError(RuntimeError):
    def __init__(self, status: int, message: str):
        super().__init__(f"libgq status {status}: {message}")
        self.status = status


class DeviceTimeout(GQError):
    """GQ_ETIMEOUT: a kernel's bounded device-side wait expired; the kernel
    returned early (no trap), so its outputs are incomplete."""


_lib = None


def lib():
    """Load libgq.so once and attach the declared signatures."""
    global _lib
    if _lib is None:
        if not os.path.exists(LIB_PATH):
            raise RuntimeError(
                f"{LIB_PATH} is missing: build it with `python -m jax_gptq_b200.csrc.build`")
        handle = ctypes.CDLL(LIB_PATH)
        for name, (res, args) in SIGNATURES.items():
            fn = getattr(handle, name, None)
            if fn is None:
                continue
            fn.restype = res
            fn.argtypes = args
        _lib = handle
    return _lib


def exported_symbols() -> list[str]:
    handle = lib()
    return [n for n in SIGNATURES if getattr(handle, n, None) is not None]


def call(name: str, *args):
    """Call ``name``; raise ``GQError`` (``ValueError`` for GQ_EINVAL) on failure."""
    fn = getattr(lib(), name)
    status = fn(*args)
    if status != GQ_OK:
        msg = lib().gq_last_error().decode(errors="replace")
        if status == GQ_EINVAL:
            raise ValueError(msg)
        if status == GQ_ETIMEOUT:
            raise DeviceTimeout(status, msg)
        raise GQError(status, msg)
    return status


def check_device(stream=None) -> None:
    """Raise :class:`DeviceTimeout` if a bounded device-side wait expired
    since the last check (``gq_check_device``; synchronizes ``stream``, by
    default torch's current stream)."""
    if stream is None:
        import torch
        stream = torch.cuda.current_stream().cuda_stream
    call("gq_check_device", stream)

"""CPU-side checks of the C ABI: the library loads, exports every symbol that
``include/gq.h`` declares, and rejects bad arguments before launching
anything (no GPU needed for either)."""

import ctypes
import os
import re

import pytest

from jax_gptq_b200 import _lib

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))


def _declared_symbols():
    names = set()
    for fn in os.listdir(os.path.join(ROOT, "include")):
        if fn.endswith(".h"):
            text = open(os.path.join(ROOT, "include", fn)).read()
            names |= set(re.findall(r"\b(gq_[a-z0-9_]+)\s*\(", text))
    return names


def test_library_exports_every_declared_symbol():
    handle = _lib.lib()
    declared = _declared_symbols()
    assert "gq_rtn" in declared and "gq_gptq_sweep" in declared
    missing = [n for n in sorted(declared) if getattr(handle, n, None) is None]
    assert not missing, missing


def test_every_declared_symbol_has_a_ctypes_signature():
    declared = _declared_symbols()
    assert declared <= set(_lib.SIGNATURES), sorted(declared - set(_lib.SIGNATURES))


def test_version_and_error_string():
    assert _lib.lib().gq_version() >= 100


def test_invalid_group_size_is_rejected_without_launch():
    lib = _lib.lib()
    st = lib.gq_rtn(None, 4, 130, 130, None, 4, 128, 0, None, None, None, None, None)
    assert st == _lib.GQ_EINVAL
    assert b"group_size" in lib.gq_last_error()
    with pytest.raises(ValueError, match="group_size"):
        _lib.call("gq_rtn", None, 4, 130, 130, None, 4, 128, 0, None, None, None, None, None)


def test_sweep_rejects_unsupported_block_and_group():
    lib = _lib.lib()
    st = lib.gq_gptq_sweep(None, 4, 256, 256, None, None, 256, None, 4, 128, 0, 64, None, None, 0,
                           None, None, None, None, None, None, 0, None)
    assert st == _lib.GQ_EINVAL
    st = lib.gq_gptq_sweep(None, 4, 192, 192, None, None, 192, None, 4, 96, 0, 128, None, None, 0,
                           None, None, None, None, None, None, 0, None)
    assert st == _lib.GQ_EINVAL


def test_workspace_sizes_are_positive():
    lib = _lib.lib()
    assert lib.gq_gptq_sweep_workspace_size(4096, 11008) >= 4096 * 11008 * 5
    assert lib.gq_hessian_factor_workspace_size(4096) >= 4096 * 4096 * 4
    assert lib.gq_qronos_workspace_size(64, 256) > lib.gq_gptq_sweep_workspace_size(64, 256)


def test_hessian_factor_rejects_small_workspace():
    lib = _lib.lib()
    att = ctypes.c_int(0)
    st = lib.gq_hessian_factor(ctypes.c_void_p(16), 64, 64, None, 0.01, ctypes.c_void_p(16), 64,
                               None, ctypes.c_void_p(16), 8, ctypes.byref(att), None)
    assert st == _lib.GQ_EINVAL


def test_comm_handle_argument_errors_without_a_gpu():
    lib = _lib.lib()
    h = ctypes.c_void_p()
    assert lib.gq_handle_create(0, None, ctypes.byref(h)) == _lib.GQ_OK and h.value
    n, r = ctypes.c_int(-1), ctypes.c_int(-1)
    assert lib.gq_handle_ranks(h, ctypes.byref(n), ctypes.byref(r)) == _lib.GQ_OK
    assert (n.value, r.value) == (1, 0)
    # a handle without a communicator cannot reduce
    assert lib.gq_allreduce_sum_f32(h, ctypes.c_void_p(16), 4, None) == _lib.GQ_EINVAL
    assert b"no communicator" in lib.gq_last_error()
    assert lib.gq_handle_destroy(h) == _lib.GQ_OK
    assert lib.gq_handle_create(0, None, None) == _lib.GQ_EINVAL
    assert lib.gq_handle_create(-1, None, ctypes.byref(h)) == _lib.GQ_EINVAL
    assert lib.gq_allreduce_sum_f32(None, None, 0, None) == _lib.GQ_EINVAL
    small = ctypes.create_string_buffer(16)
    assert lib.gq_nccl_unique_id(small, 16) == _lib.GQ_EINVAL
    assert lib.gq_handle_create_nccl(0, small, 2, 2, ctypes.byref(h)) == _lib.GQ_EINVAL


def test_pair_kernel_switch_validates_its_argument():
    lib = _lib.lib()
    assert lib.gq_set_pair_kernels(0) == 0
    assert lib.gq_set_pair_kernels(1) == 0
    assert lib.gq_set_pair_kernels(2) != 0


def test_packed_symmetric_size_and_argument_checks():
    """gq_sym_packed_size against the layout restated here (128-row blocks,
    row r from column 128 (r // 128) on), and the pack / unpack / packed
    all-reduce entries reject bad arguments before launching anything."""
    lib = _lib.lib()
    for d in (0, 1, 127, 128, 129, 1000, 4096, 11008, 28672):
        expect = sum(d - 128 * (r // 128) for r in range(d))
        assert lib.gq_sym_packed_size(d) == expect, d
    assert lib.gq_sym_packed_size(28672) * 4 < 0.51 * 4 * 28672 ** 2
    p = ctypes.c_void_p(256)
    assert lib.gq_sym_pack_upper(p, -1, 4, p, None) == _lib.GQ_EINVAL
    assert lib.gq_sym_pack_upper(None, 4, 4, p, None) == _lib.GQ_EINVAL
    assert lib.gq_sym_pack_upper(p, 4, 3, p, None) == _lib.GQ_EINVAL
    assert lib.gq_sym_unpack_upper(p, 4, None, 4, None) == _lib.GQ_EINVAL
    assert lib.gq_sym_unpack_upper(p, 4, p, 3, None) == _lib.GQ_EINVAL
    assert lib.gq_sym_pack_upper(None, 0, 0, None, None) == 0
    assert lib.gq_allreduce_sym_f32(None, p, 4, 4, p, None) == _lib.GQ_EINVAL


def test_sweep_row_group_switch_validates_its_argument():
    lib = _lib.lib()
    for r in (-1, 1, 2, 4, 0):
        assert lib.gq_set_sweep_row_groups(r) == 0
    for r in (3, 5, -2, 8):
        assert lib.gq_set_sweep_row_groups(r) == _lib.GQ_EINVAL
    assert lib.gq_set_sweep_row_groups(0) == 0


def test_factor_from_activations_validates_before_launching():
    lib = _lib.lib()
    p = ctypes.c_void_p(256)
    need = lib.gq_factor_from_x_workspace_size(1024, 512)
    assert need >= 512 * 512 * 4 + 1024 * 512 * 2
    args = dict(x=p, tokens=1024, d=512, ldx=512, ordering=1, damp=0.01, reserve=12, u=p, ldu=512,
                perm=p, ws=p, ws_bytes=need, status=p)

    def call(**kw):
        a = dict(args, **kw)
        return lib.gq_factor_from_x_attempt(a["x"], a["tokens"], a["d"], a["ldx"], a["ordering"],
                                            a["damp"], a["reserve"], a["u"], a["ldu"], a["perm"],
                                            a["ws"], a["ws_bytes"], a["status"], None, None)

    assert call(d=516, ldx=516, ldu=516) == _lib.GQ_EINVAL       # d not a multiple of 8
    assert b"multiples of 8" in lib.gq_last_error()
    assert call(ordering=2) == _lib.GQ_EINVAL
    assert call(ws_bytes=need - 1) == _lib.GQ_EINVAL
    assert call(ws=ctypes.c_void_p(272)) == _lib.GQ_EINVAL        # not 256-byte aligned
    assert call(x=ctypes.c_void_p(264)) == _lib.GQ_EINVAL         # x not 16-byte aligned
    assert call(damp=-1.0) == _lib.GQ_EINVAL
    assert call(reserve=-1) == _lib.GQ_EINVAL
    assert call(d=40000, ldx=40000, ldu=40000,
                ws_bytes=lib.gq_factor_from_x_workspace_size(1024, 40000)) == _lib.GQ_EINVAL
    assert b"too large" in lib.gq_last_error()


def test_wait_limit_and_failure_entries_reject_bad_arguments():
    with pytest.raises(ValueError, match="outside"):
        _lib.call("gq_set_wait_limit_ns", 10)
    with pytest.raises(ValueError, match="outside"):
        _lib.call("gq_set_wait_limit_ns", 10 ** 12)
    with pytest.raises(ValueError, match="unit"):
        _lib.call("gq_test_expire_wait", 2, ctypes.c_void_p(16), None)
    with pytest.raises(ValueError, match="NULL"):
        _lib.call("gq_comm_check", None, 1)
    with pytest.raises(ValueError, match="NULL"):
        _lib.call("gq_handle_abort", None)


def test_sweep_rejects_shapes_whose_workspace_would_overflow():
    with pytest.raises(ValueError, match="too large"):
        _lib.call("gq_gptq_sweep_static", None, 1 << 60, 4096, 4096, None, None, 4096, None, 4,
                  128, 0, 128, None, None, 0, None, None, None, None, None, None)
    with pytest.raises(ValueError, match="row buffer"):
        _lib.call("gq_gptq_sweep_static", None, 4, 1 << 20, 1 << 20, None, None, 1 << 20, None, 4,
                  128, 0, 128, None, None, 0, None, None, None, None, None, None)


def test_eigensolver_and_qr_modes_reject_bad_arguments():
    with pytest.raises(ValueError, match="max_sweeps"):
        _lib.call("gq_syevj", ctypes.c_void_p(16), 8, 8, ctypes.c_void_p(16), ctypes.c_void_p(16),
                  8, 0, None, ctypes.c_void_p(256), 1 << 20, None)
    with pytest.raises(ValueError, match="staged row"):
        _lib.call("gq_syevj", ctypes.c_void_p(16), 60000, 60000, ctypes.c_void_p(16),
                  ctypes.c_void_p(16), 60000, 10, None, ctypes.c_void_p(256), 1 << 40, None)
    with pytest.raises(ValueError, match="pivot_mode"):
        _lib.call("gq_qrcp", ctypes.c_void_p(16), 8, 8, 8, 8, 3, 1, ctypes.c_void_p(16), None, 8,
                  None, None, None, ctypes.c_void_p(256), 1 << 20, None)

"""Generate the golden vectors in ``tests/golden/*.npz`` from the reference itself.

Run in a container that has the reference checked out (read-only is fine),
naming its ``src`` directory on the command line or in ``JAX_GPTQ_REFERENCE_SRC``:

    python tests/golden/make_golden.py --reference-src <checkout>/src

JAX is not installable offline, so the reference's own, unmodified modules
(``quant.py``, ``stats.py``, ``gptq_ref.py``, ``qronos_ref.py``,
``pallas/blocked_pivoted_qr.py``) are imported with
``tests/golden/jaxshim`` -- a numpy-backed stand-in for the ``jax`` API subset
they use -- first on ``sys.path``.  The outputs therefore carry the
reference's control flow and op order with numpy's float32 rounding.  The
GPU box never runs this script; the tests only read the ``.npz`` files.
"""

from __future__ import annotations

import argparse
import os
import sys

import numpy as np

HERE = os.path.dirname(os.path.abspath(__file__))


def _import_reference(src: str):
    sys.dont_write_bytecode = True
    sys.path.insert(0, src)
    sys.path.insert(0, os.path.join(HERE, "jaxshim"))
    import jax.numpy as jnp  # the shim
    import jax_gptq
    import importlib
    gptq_ref = importlib.import_module("jax_gptq.gptq_ref")
    bpq = importlib.import_module("jax_gptq.pallas.blocked_pivoted_qr")
    return jnp, jax_gptq, gptq_ref, bpq


def _np(x):
    return np.array(x)


def make_rtn_cases(jnp, ref):
    cases = {}
    rng = np.random.Generator(np.random.PCG64(100))
    shapes = [
        ("asym4_g128", (16, 256), dict(w_bits=4, group_size=128, sym=False)),
        ("sym4_g128", (16, 256), dict(w_bits=4, group_size=128, sym=True)),
        ("asym3_g128", (8, 384), dict(w_bits=3, group_size=128, sym=False)),
        ("asym8_g64", (8, 128), dict(w_bits=8, group_size=64, sym=False)),
        ("asym4_g32", (4, 96), dict(w_bits=4, group_size=32, sym=False)),
        ("sym2_g16", (4, 64), dict(w_bits=2, group_size=16, sym=True)),
    ]
    for name, shape, kw in shapes:
        w = (rng.standard_normal(shape) * 0.02).astype(np.float32)
        # a constant group (scale floor), an all-positive and an all-negative group
        w[0, :kw["group_size"]] = 0.0
        w[1, :kw["group_size"]] = np.abs(w[1, :kw["group_size"]]) + 0.01
        w[2, :kw["group_size"]] = -np.abs(w[2, :kw["group_size"]]) - 0.01
        cfg = ref.QuantConfig(**kw)
        out = _np(ref.quantize_dequantize(jnp.asarray(w), cfg))
        cases[f"rtn_{name}_w"] = w
        cases[f"rtn_{name}_out"] = out
        cases[f"rtn_{name}_cfg"] = np.array([kw["w_bits"], kw["group_size"], int(kw["sym"])])
    # the reference's smoke shapes (scripts/smoke.py:9-16)
    cfg = ref.QuantConfig(w_bits=4, group_size=4, sym=False, rank_eps=1e-5)
    w = np.arange(0.0, 32.0, dtype=np.float32).reshape(4, 8)
    xq = np.arange(0.0, 80.0, dtype=np.float32).reshape(10, 8)
    xf = xq + np.float32(0.01)
    h, g = ref.h_g_from_activations(jnp.asarray(xq), jnp.asarray(xf))
    perm = np.arange(8, dtype=np.int32)
    out = ref.gptq_forward_step(jnp.asarray(w), h_inv_sqrt=h, perm=jnp.asarray(perm), cfg=cfg)
    cases.update(smoke_w=w, smoke_xq=xq, smoke_xf=xf, smoke_h=_np(h), smoke_g=_np(g),
                 smoke_out=_np(out))
    return cases


def make_gptq_cases(jnp, ref, gptq_ref):
    cases = {}
    rng = np.random.Generator(np.random.PCG64(101))
    for name, (m, n, tokens, ordering, kw) in {
        "none": (32, 256, 64, "none", dict(w_bits=4, group_size=128, sym=False)),
        "diag": (32, 256, 64, "diag_h", dict(w_bits=4, group_size=128, sym=False)),
        "diag_sym3": (16, 192, 48, "diag_h", dict(w_bits=3, group_size=64, sym=True)),
    }.items():
        w = (rng.standard_normal((m, n)) * 0.02).astype(np.float32)
        x = (rng.standard_normal((tokens, n)) * rng.lognormal(0, 1, n)).astype(np.float32)
        # ties in diag(H): duplicate two channels to pin the stable-sort tie rule
        x[:, 7] = x[:, 3]
        cfg = ref.QuantConfig(ordering_mode=ordering, **kw)
        h, g = ref.h_g_from_activations(jnp.asarray(x))
        h_inv_sqrt, perm = gptq_ref.process_hessian(h, cfg)
        out = ref.gptq_forward_step(jnp.asarray(w), h_inv_sqrt, perm, cfg)
        xf = (x + rng.standard_normal(x.shape).astype(np.float32) * np.float32(0.05)).astype(np.float32)
        h2, g2 = ref.h_g_from_activations(jnp.asarray(x), jnp.asarray(xf))
        qr_out = ref.qronos_single_layer_update_ref(jnp.asarray(w), jnp.asarray(w), h2, g2, cfg)
        hinv = _np(h_inv_sqrt)
        cases.update({
            f"gptq_{name}_w": w, f"gptq_{name}_x": x, f"gptq_{name}_xf": xf,
            f"gptq_{name}_hinv_is_eye": np.array(bool(np.array_equal(hinv, np.eye(n)))),
            f"gptq_{name}_perm": _np(perm),
            f"gptq_{name}_out": _np(out), f"gptq_{name}_qronos": _np(qr_out),
            f"gptq_{name}_cfg": np.array([kw["w_bits"], kw["group_size"], int(kw["sym"]),
                                          int(ordering == "diag_h")]),
        })
        if name == "none":
            cases.update({f"gptq_{name}_h": _np(h), f"gptq_{name}_g": _np(g),
                          f"gptq_{name}_g2": _np(g2)})
    return cases


def make_qr_cases(jnp, bpq):
    cases = {}
    rng = np.random.Generator(np.random.PCG64(102))
    example = np.array([[3.0, 1.0, 0.0, 2.0], [4.0, 0.0, 2.0, 1.0],
                        [0.0, 5.0, 1.0, 0.0], [0.0, 0.0, 6.0, 1.0]], np.float32)
    specs = [
        ("ex_p2_largest", example, 2, "largest"),
        ("ex_p2_smallest", example, 2, "smallest"),
        ("ex_p4_largest", example, 4, "largest"),
        ("zero3_p2_smallest", np.zeros((3, 3), np.float32), 2, "smallest"),
    ]
    for name, (m, n, panel, mode) in {
        "r48x40_p8_largest": (48, 40, 8, "largest"),
        "r40x48_p16_largest": (40, 48, 16, "largest"),
        "r64_p1_largest": (64, 64, 1, "largest"),
        "r64_p64_largest": (64, 64, 64, "largest"),
        "r64_p16_smallest": (64, 64, 16, "smallest"),
        "r96_p32_largest": (96, 96, 32, "largest"),
    }.items():
        g = rng.standard_normal((m, n)).astype(np.float32)
        s = (10.0 ** (-3.0 * np.arange(n) / n)).astype(np.float32)[rng.permutation(n)]
        specs.append((name, (g * s).astype(np.float32), panel, mode))
    for name, a, panel, mode in specs:
        work, perm = bpq.blocked_pivoted_qr(jnp.asarray(a), panel_size=panel, pivot_mode=mode)
        cases[f"qr_{name}_a"] = a
        cases[f"qr_{name}_work"] = _np(work)
        cases[f"qr_{name}_perm"] = _np(perm)
        cases[f"qr_{name}_cfg"] = np.array([panel, int(mode == "smallest")])
    # exact QRCP: the reference's eager panel path (JAX_GPTQ_QR_TIMING=1) at
    # panel_size=1, where every reflector comes from the pivot column
    import contextlib
    import io
    for name, (m, n, mode) in {"r64": (64, 64, "largest"), "r80x48": (80, 48, "largest"),
                               "r48x64": (48, 64, "largest"),
                               "r64_smallest": (64, 64, "smallest")}.items():
        g = rng.standard_normal((m, n)).astype(np.float32)
        s = (10.0 ** (-3.0 * np.arange(n) / n)).astype(np.float32)[rng.permutation(n)]
        a = (g * s).astype(np.float32)
        os.environ["JAX_GPTQ_QR_TIMING"] = "1"
        try:
            with contextlib.redirect_stdout(io.StringIO()):
                work, perm = bpq.blocked_pivoted_qr(jnp.asarray(a), panel_size=1, pivot_mode=mode)
        finally:
            os.environ.pop("JAX_GPTQ_QR_TIMING", None)
        cases[f"exact_{name}_a"] = a
        cases[f"exact_{name}_work"] = _np(work)
        cases[f"exact_{name}_perm"] = _np(perm)
        cases[f"exact_{name}_cfg"] = np.array([1, int(mode == "smallest")])
    # one panel of the compiled path with its compact-WY state
    a = specs[4][1]
    norms = np.sum(np.square(a), axis=0).astype(np.float32)
    res = bpq.factor_panel_pallas(jnp.asarray(a), jnp.arange(a.shape[1], dtype=jnp.int32),
                                  jnp.asarray(norms), 8, 8, "largest")
    cases.update(panel_a=a, panel_norms_in=norms, panel_a_out=_np(res.a),
                 panel_perm_out=_np(res.perm), panel_norms_out=_np(res.norms),
                 panel_y=_np(res.panel.y), panel_tau=_np(res.panel.tau),
                 panel_t=_np(res.panel.t), panel_end=np.array(int(res.panel.panel_end)))
    return cases


def make_eigh_cases(jnp, ref, gptq_ref):
    """process_hessian with solver_mode="eigh" (gptq_ref.py:95-133), all four
    ordering modes, for a full-rank H and a rank-deficient one (fewer tokens
    than features, so the default truncation drops eigenvalues and the
    none/diag_h gathers run past the kept columns)."""
    cases = {}
    rng = np.random.Generator(np.random.PCG64(102))
    for name, (n, tokens) in {"full": (48, 400), "deficient": (48, 40)}.items():
        x = (rng.standard_normal((tokens, n)) * rng.uniform(0.5, 2.0, n)).astype(np.float32)
        h = (x.T.astype(np.float64) @ x / tokens).astype(np.float32)
        cases[f"eigh_{name}_h"] = h
        for mode in ("none", "diag_h", "pivot_sqrt_h", "pivot_sqrt_hinv_smallest"):
            cfg = ref.QuantConfig(solver_mode="eigh", ordering_mode=mode)
            r, perm = gptq_ref.process_hessian(jnp.asarray(h), cfg, panel_size=8)
            cases[f"eigh_{name}_{mode}_r"] = _np(r)
            cases[f"eigh_{name}_{mode}_perm"] = _np(perm)
    return cases


def main() -> None:
    ap = argparse.ArgumentParser()
    ap.add_argument("--reference-src", default=os.environ.get("JAX_GPTQ_REFERENCE_SRC"),
                    help="the reference checkout's src directory (or set JAX_GPTQ_REFERENCE_SRC)")
    ap.add_argument("--out", default=HERE)
    args = ap.parse_args()
    if not args.reference_src:
        ap.error("--reference-src (or JAX_GPTQ_REFERENCE_SRC) is required")
    jnp, ref, gptq_ref, bpq = _import_reference(args.reference_src)
    np.savez_compressed(os.path.join(args.out, "rtn_golden.npz"), **make_rtn_cases(jnp, ref))
    np.savez_compressed(os.path.join(args.out, "gptq_golden.npz"),
                        **make_gptq_cases(jnp, ref, gptq_ref))
    np.savez_compressed(os.path.join(args.out, "qr_golden.npz"), **make_qr_cases(jnp, bpq))
    np.savez_compressed(os.path.join(args.out, "eigh_golden.npz"),
                        **make_eigh_cases(jnp, ref, gptq_ref))
    print("wrote golden vectors to", args.out)


if __name__ == "__main__":
    main()

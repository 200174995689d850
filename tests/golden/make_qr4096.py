"""Generate ``tests/golden/qr4096_fixture.npz``: the 4096 x 4096 pivoted-QR
benchmark matrices factored by the oracle on the CPU.

    python tests/golden/make_qr4096.py [--n 4096] [--out tests/golden/qr4096_fixture.npz]

The matrices come from ``oracle.inputs.qr_matrix`` (seed 1): ``A = G diag(s)``
with ``s_k = 10^(-6k/n)`` in a shuffled column order, and the rank-deficient
variant with 256 columns replaced by random combinations of the others.
Four factorizations are stored, each as its column permutation (int16) and
``|diag R|`` (float32), about 24 KB per case:

* ``intended_largest`` -- exact Householder QR with column pivoting
  (``oracle.qr.exact_pivoted_qr``; the reference's eager path at panel 1);
* ``reference_largest`` -- the reference's compiled blocked path at panel 64
  (``oracle.qr.blocked_pivoted_qr``, with its stale mid-panel pivots);
* ``intended_rankdef_smallest`` -- exact QRCP of the rank-deficient matrix
  with ``pivot_mode="smallest"``;
* ``intended_rankdef_largest`` -- the same with ``pivot_mode="largest"``
  (rank-revealing: the 256 dependent columns come last, at noise level).

The GPU test regenerates the matrices from the same seed (host numpy, so the
bytes are identical) and compares its pivots and diagonal with these.  The
whole run takes about a quarter of an hour on 16 cores.
"""

from __future__ import annotations

import argparse
import os
import sys
import time

import numpy as np

HERE = os.path.dirname(os.path.abspath(__file__))
ROOT = os.path.dirname(os.path.dirname(HERE))
sys.path.insert(0, ROOT)

from oracle import inputs  # noqa: E402
from oracle import qr as oqr  # noqa: E402


def main() -> None:
    ap = argparse.ArgumentParser()
    ap.add_argument("--n", type=int, default=4096)
    ap.add_argument("--panel", type=int, default=64)
    ap.add_argument("--out", default=os.path.join(HERE, "qr4096_fixture.npz"))
    args = ap.parse_args()
    n = args.n
    a = inputs.qr_matrix(1, n, n)
    a_def = inputs.qr_matrix(1, n, n, rank_deficient=True)
    out = {"n": np.int32(n), "panel": np.int32(args.panel)}
    cases = [("intended_largest", lambda: oqr.exact_pivoted_qr(a, "largest")),
             ("reference_largest", lambda: oqr.blocked_pivoted_qr(a, args.panel, "largest")),
             ("intended_rankdef_smallest", lambda: oqr.exact_pivoted_qr(a_def, "smallest")),
             ("intended_rankdef_largest", lambda: oqr.exact_pivoted_qr(a_def, "largest"))]
    for name, run in cases:
        t0 = time.time()
        work, perm = run()
        out[name + "_perm"] = np.asarray(perm, np.int16)
        out[name + "_absdiag"] = np.abs(np.diag(work)).astype(np.float32)
        print(f"{name}: {time.time() - t0:.1f} s", flush=True)
    np.savez_compressed(args.out, **out)
    print("wrote", args.out)


if __name__ == "__main__":
    main()

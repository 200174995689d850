"""Tie-aware comparison of integer codes, shared by the parity tests.

The GPU sweep and the oracle's sweep run the same column recurrence but add
the lazy-update terms in different orders (batched tensor-core GEMMs against
numpy BLAS), so their float32 values differ by reassociation.  A code may
then round the other way only where the unrounded value ``w / scale + zero``
sits next to a half step: a rounding tie.  Rows are independent, so in each
row that differs at all, the FIRST differing code must be such a tie; later
codes of that row follow from the flipped error feedback and are counted,
not checked.

``TIE_TOL`` is the largest distance from the half step (in units of one
quantization step) that is accepted as a tie: 1e-5, about ten float32 ulps
of a 4-bit code value (ulp(8) = 9.5e-7).  Measured on B200, the first
differing codes of the sweep and Qronos tests sat 0 to 6.2e-6 from the half
step.
"""

from __future__ import annotations

import json
import os

import numpy as np

TIE_TOL = 1e-5


def code_diffs(got_perm: np.ndarray, ref_perm: np.ndarray, ref_pre_perm: np.ndarray) -> dict:
    """Compare codes in permuted (sweep) column order.

    ``got_perm``/``ref_perm``: [rows, n] codes as floats (q, not q - qmin);
    ``ref_pre_perm``: the oracle's unrounded values.  Returns the number of
    rows that differ (``tie_rows``), of codes that differ, and the distance of
    each such row's first differing value from its half step."""
    diff = np.asarray(got_perm) != np.asarray(ref_perm)
    bad_rows = np.flatnonzero(diff.any(axis=1))
    if bad_rows.size == 0:
        return {"rows": int(diff.shape[0]), "tie_rows": 0, "codes_differing": 0,
                "max_tie_dist": 0.0, "dist": np.zeros(0)}
    first = diff[bad_rows].argmax(axis=1)
    pre = np.asarray(ref_pre_perm)[bad_rows, first].astype(np.float64)
    dist = np.abs(pre - np.floor(pre) - 0.5)
    return {"rows": int(diff.shape[0]), "tie_rows": int(bad_rows.size),
            "codes_differing": int(diff.sum()), "max_tie_dist": float(dist.max()), "dist": dist}


def report(name: str, **fields) -> None:
    """Append one JSON line of measured parity figures to the file named by
    ``GQ_PARITY_REPORT`` (nothing when unset)."""
    path = os.environ.get("GQ_PARITY_REPORT")
    if not path:
        return
    rec = {"test": name}
    for k, v in fields.items():
        if isinstance(v, np.ndarray):
            continue
        rec[k] = v.item() if hasattr(v, "item") else v
    d = os.path.dirname(path)
    if d:
        os.makedirs(d, exist_ok=True)
    with open(path, "a") as f:
        f.write(json.dumps(rec) + "\n")

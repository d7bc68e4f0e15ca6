"""Selection comparison with the near-tie excuse — test infrastructure only.

Two Quest selections of one (layer, request) are compared as ordered
position lists.  The recent window / dense layout must match exactly.  The
selected pages may differ only where the two choices are near-tied: at every
slot the float64 page scores of the two pages must agree within ``rel_tol``
(1e-5 relative).  Such excused cases are counted by the callers.
"""

from __future__ import annotations

from dataclasses import dataclass

import numpy as np


def score_pages_f64(bounds: np.ndarray, qbar: np.ndarray) -> np.ndarray:
    """Quest page scores in float64: ``bounds [pages, kv, d, 2]``, ``qbar [kv, d]``."""
    b = np.asarray(bounds, dtype=np.float64)
    q = np.asarray(qbar, dtype=np.float64)[None]
    chosen = np.where(q >= 0, b[..., 1], b[..., 0])
    with np.errstate(over="ignore", invalid="ignore"):
        return (q * chosen).sum(axis=(1, 2))


@dataclass
class SelectionMismatch:
    exact: bool
    excused: bool
    detail: str = ""


def _rel_close(a: float, b: float, rel_tol: float) -> bool:
    if a == b:
        return True
    if not (np.isfinite(a) and np.isfinite(b)):
        return False
    return abs(a - b) <= rel_tol * max(abs(a), abs(b), 1e-30)


def compare_selection(
    ours: np.ndarray,
    ref: np.ndarray,
    *,
    seq_len: int,
    top_k: int,
    page_size: int,
    scores_f64: np.ndarray | None,
    rel_tol: float = 1e-5,
) -> SelectionMismatch:
    """Compare two ``[top_k]`` position rows of one (layer, request)."""
    ours = np.asarray(ours, dtype=np.int64)
    ref = np.asarray(ref, dtype=np.int64)
    n = min(seq_len, top_k)
    if np.array_equal(ours[:n], ref[:n]):
        return SelectionMismatch(True, False)
    if seq_len <= top_k:
        return SelectionMismatch(False, False, "dense layout differs")
    P = page_size
    sel = top_k // P - 1
    if not np.array_equal(ours[sel * P :], ref[sel * P :]):
        return SelectionMismatch(False, False, "recent window differs")
    pa = ours[: sel * P].reshape(sel, P)
    pb = ref[: sel * P].reshape(sel, P)
    for blk in (pa, pb):
        if not np.array_equal(blk - blk[:, :1], np.broadcast_to(np.arange(P), blk.shape)):
            return SelectionMismatch(False, False, "selected block is not a page expansion")
    pages_a, pages_b = pa[:, 0] // P, pb[:, 0] // P
    if scores_f64 is None:
        return SelectionMismatch(False, False, "pages differ and no scores to classify")
    for j in range(sel):
        sa, sb = float(scores_f64[pages_a[j]]), float(scores_f64[pages_b[j]])
        if not _rel_close(sa, sb, rel_tol):
            return SelectionMismatch(
                False, False,
                f"slot {j}: page {pages_a[j]} (score {sa!r}) vs page {pages_b[j]} (score {sb!r})",
            )
    return SelectionMismatch(False, True, "near-tie reorder")

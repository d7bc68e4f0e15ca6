"""Record-by-record comparison of two lifecycle runs (test infrastructure)."""

from __future__ import annotations

import json
from dataclasses import dataclass, field
from pathlib import Path

import numpy as np

from oracle.parity import compare_selection
from tests.harness import DecodeRecord, records_to_arrays

GOLDEN_DIR = Path(__file__).resolve().parent / "golden"

#: attention tolerances (absolute): bf16 outputs, fp32 outputs
ATOL_BF16 = 2e-2
ATOL_F32 = 1e-5


def bf16_ulp(x: np.ndarray) -> np.ndarray:
    """Spacing of bf16 values at |x| (8 significant bits)."""
    ax = np.maximum(np.abs(np.asarray(x, dtype=np.float64)), 2.0 ** -126)
    return 2.0 ** (np.floor(np.log2(ax)) - 7)


def bf16_output_tolerance(ref: np.ndarray) -> np.ndarray:
    """Per-element tolerance between two bf16-rounded attention outputs.

    2e-2 absolute; where one bf16 step of the value is larger (|ref| >= 4) the
    two independently rounded results may sit one step apart, so one ulp.
    """
    return np.maximum(ATOL_BF16, bf16_ulp(ref))


def load_golden(name: str) -> tuple[dict[str, np.ndarray], dict]:
    with np.load(GOLDEN_DIR / name, allow_pickle=False) as z:
        arrays = {k: z[k] for k in z.files if k != "meta"}
        meta = json.loads(str(z["meta"]))
    return arrays, meta


@dataclass
class ParityReport:
    records: int = 0
    exact: int = 0
    excused: int = 0
    out_checked: int = 0
    max_out_err: float = 0.0
    buffer_checked: int = 0
    failures: list[str] = field(default_factory=list)

    def ok(self) -> bool:
        return not self.failures

    def summary(self) -> str:
        return (f"records={self.records} exact={self.exact} excused_near_ties={self.excused} "
                f"out_checked={self.out_checked} max_out_err={self.max_out_err:.3g} "
                f"buffer_checked={self.buffer_checked} failures={len(self.failures)}")


def compare_runs(
    ours: dict[str, np.ndarray],
    ref: dict[str, np.ndarray],
    oracle_records: list[DecodeRecord],
    *,
    top_k: int,
    page_size: int,
    bf16: bool,
    check_buffers: bool,
    max_fail: int = 10,
) -> ParityReport:
    """``ours`` / ``ref`` are :func:`records_to_arrays` outputs of the same scenario."""
    rep = ParityReport()
    atol = ATOL_BF16 if bf16 else ATOL_F32
    n = len(ref["step"])
    if len(ours["step"]) != n:
        rep.failures.append(f"record count {len(ours['step'])} != {n}")
        return rep
    for key in ("step", "layer", "req", "slot", "seq_len", "n"):
        if not np.array_equal(ours[key], ref[key]):
            rep.failures.append(f"schedule field {key} differs")
            return rep
    diverged: set[tuple[int, int]] = set()
    rep.records = n
    for i in range(n):
        sl, cnt = int(ref["seq_len"][i]), int(ref["n"][i])
        req_layer = (int(ref["req"][i]), int(ref["layer"][i]))
        s64 = oracle_records[i].scores64 if oracle_records is not None else None
        m = compare_selection(ours["positions"][i, :cnt], ref["positions"][i, :cnt], seq_len=sl,
                              top_k=top_k, page_size=page_size, scores_f64=s64)
        if m.exact:
            rep.exact += 1
            diff = np.abs(ours["out"][i] - ref["out"][i])
            err = float(np.max(diff))
            rep.max_out_err = max(rep.max_out_err, err)
            rep.out_checked += 1
            tol = bf16_output_tolerance(ref["out"][i]) if bf16 else atol
            if not bool(np.all(diff <= tol)):
                rep.failures.append(f"record {i} {req_layer} L={sl}: out err {err:.3g} beyond tolerance")
        elif m.excused:
            rep.excused += 1
            diverged.add(req_layer)
        else:
            rep.failures.append(f"record {i} {req_layer} L={sl}: selection differs: {m.detail}")
        if check_buffers and req_layer not in diverged and "buffer_tokens" in ref:
            rep.buffer_checked += 1
            if not np.array_equal(ours["buffer_tokens"][i], ref["buffer_tokens"][i]):
                rep.failures.append(f"record {i} {req_layer} L={sl}: buffer_tokens differ")
            if not np.array_equal(ours["lru_slots"][i], ref["lru_slots"][i]):
                rep.failures.append(f"record {i} {req_layer} L={sl}: lru_slots differ")
        if len(rep.failures) >= max_fail:
            break
    return rep


def oracle_run(sc, mode):
    from oracle.driver import OracleLifecycleDriver

    drv = OracleLifecycleDriver(sc, mode)
    recs = drv.run()
    return recs, records_to_arrays(recs, sc.top_k), drv.stats()

"""The numpy oracle reproduces the reference's committed golden outputs (CPU).

Pins the oracle before it is trusted as the checker of the CUDA path: for every
fixture written by ``tests/golden/make_golden.py`` from the reference
backends, the oracle replays the same seeded scenario and must make the same
selections (bit-exact positions, near-ties excused and counted), produce the
same attention outputs within tolerance, reach the same HiSparse hot-buffer
state bit for bit and count the same hits / misses.
"""

from __future__ import annotations

import pytest

from tests.golden.scenarios import GOLDEN, fixture_name
from tests.parity_helpers import compare_runs, load_golden, oracle_run


@pytest.mark.parametrize(("sc", "mode", "prefill"), GOLDEN, ids=lambda x: getattr(x, "name", x))
def test_oracle_matches_reference_golden(sc, mode, prefill):
    ref, meta = load_golden(fixture_name(sc, mode))
    recs, ours, stats = oracle_run(sc, mode)
    rep = compare_runs(ours, ref, recs, top_k=sc.top_k, page_size=sc.page_size, bf16=sc.bf16,
                       check_buffers=True)
    assert rep.ok(), rep.summary() + "\n" + "\n".join(rep.failures)
    assert rep.exact >= 0.95 * rep.records, rep.summary()
    if mode == "quest_hisparse" and rep.excused == 0:
        assert stats == meta["stats"]


def test_oracle_config0_selects_planted_pages():
    """Config 0 plants four high-scoring pages; the reference picked them all."""
    from tests.golden.scenarios import CONFIG0

    ref, _ = load_golden(fixture_name(CONFIG0, "quest"))
    recs, ours, _ = oracle_run(CONFIG0, "quest")
    assert ours["positions"][0].tolist() == ref["positions"][0].tolist()

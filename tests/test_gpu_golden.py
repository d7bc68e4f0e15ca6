"""The CUDA backends reproduce the reference's golden outputs (GPU).

Each committed scenario is replayed through ``B200QuestOnlyBackend`` /
``B200QuestHiSparseBackend`` via the public ``AttentionBackend`` interface,
exactly as ``Engine.generate`` drives it.  Selections must equal the
reference's position lists (near-ties excused and counted), attention
outputs must be within 2e-2 (bf16) / 1e-5 (fp32), HiSparse hot-buffer state
(``buffer_tokens``, ``lru_slots``) must match bit for bit, and the swap-in
hit/miss counts must agree.

The Mode 2 fixtures are replayed a second time with no ``QuestTrace``
attached: the backend then makes the single fused selection + attention call
per layer that the benchmark times (a trace makes it split the call in two),
and the positions are read back from its position buffer.
"""

from __future__ import annotations

import pytest

from tests.harness import LifecycleDriver, b200_api, records_to_arrays
from tests.golden.scenarios import GOLDEN, fixture_name
from tests.parity_helpers import compare_runs, load_golden, oracle_run

pytestmark = pytest.mark.gpu


@pytest.mark.parametrize(("sc", "mode", "prefill"), GOLDEN, ids=lambda x: getattr(x, "name", x))
def test_b200_backend_matches_reference_golden(sc, mode, prefill, cuda_device):
    ref, meta = load_golden(fixture_name(sc, mode))
    drv = LifecycleDriver(sc, mode, b200_api(), cuda_device, prefill=prefill)
    recs = drv.run()
    drv.backend.synchronize()
    ours = records_to_arrays(recs, sc.top_k)
    orecs, _, _ = oracle_run(sc, mode)
    rep = compare_runs(ours, ref, orecs, top_k=sc.top_k, page_size=sc.page_size, bf16=sc.bf16,
                       check_buffers=True)
    print(f"{sc.name}/{mode}: {rep.summary()}")
    assert rep.ok(), rep.summary() + "\n" + "\n".join(rep.failures)
    assert rep.exact >= 0.95 * rep.records, rep.summary()
    if mode == "quest_hisparse" and rep.excused == 0:
        assert drv.stats() == meta["stats"]


FUSED = [g for g in GOLDEN if g[1] == "quest"]


@pytest.mark.parametrize(("sc", "mode", "prefill"), FUSED, ids=lambda x: getattr(x, "name", x))
def test_fused_call_matches_reference_golden(sc, mode, prefill, cuda_device):
    ref, _ = load_golden(fixture_name(sc, mode))
    drv = LifecycleDriver(sc, mode, b200_api(), cuda_device, prefill=prefill, trace=False)
    assert drv.backend.fused and drv.backend.quest.trace is None and drv.backend.kernel_events is None
    recs = drv.run()
    drv.backend.synchronize()
    ours = records_to_arrays(recs, sc.top_k)
    orecs, _, _ = oracle_run(sc, mode)
    rep = compare_runs(ours, ref, orecs, top_k=sc.top_k, page_size=sc.page_size, bf16=sc.bf16,
                       check_buffers=False)
    print(f"{sc.name}/{mode} (fused call): {rep.summary()}")
    assert rep.ok(), rep.summary() + "\n" + "\n".join(rep.failures)
    assert rep.exact >= 0.95 * rep.records, rep.summary()

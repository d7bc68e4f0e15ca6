"""Generate the golden fixtures from the reference implementation itself.

Run in a container where the reference source is available (it is pure
Python + torch, CPU only)::

    python tests/golden/make_golden.py /path/to/QwenQuest/src

For every entry of ``scenarios.GOLDEN`` it drives the reference's
``QuestOnlyBackend`` / ``QuestHiSparseBackend`` (``src/qwenquest/attention``)
through :class:`qwenquest_b200.harness.LifecycleDriver` on CPU with the
reference's own pools, ``ForwardBatch`` and ``QuestTrace``, and writes per
(step, layer, request): the selected positions in attention order, the
attention output, and for HiSparse the hot-buffer state (``buffer_tokens``,
``lru_slots``) plus the swap-in statistics.  Only outputs are stored; the
inputs are regenerated from the scenario seeds.
"""

from __future__ import annotations

import json
import sys
import time
from pathlib import Path

import numpy as np
import torch

HERE = Path(__file__).resolve().parent
REPO = HERE.parents[1]
sys.path.insert(0, str(REPO))

from qwenquest_b200.harness import LifecycleAPI, LifecycleDriver, records_to_arrays  # noqa: E402
from tests.golden.scenarios import GOLDEN, fixture_name  # noqa: E402


def reference_api(src: str) -> LifecycleAPI:
    sys.path.insert(0, src)
    from qwenquest.attention import QuestHiSparseBackend, QuestOnlyBackend
    from qwenquest.batch import ForwardBatch, ForwardMode
    from qwenquest.memory import MHATokenToKVPool, ReqToTokenPool, TokenToKVPoolAllocator
    from qwenquest.quest import QuestTrace

    return LifecycleAPI(
        ForwardBatch, ForwardMode, ReqToTokenPool, MHATokenToKVPool, TokenToKVPoolAllocator,
        QuestOnlyBackend, QuestHiSparseBackend, QuestTrace,
    )


def main(argv: list[str]) -> None:
    src = argv[1] if len(argv) > 1 else "/root/reference/src"
    api = reference_api(src)
    torch.set_num_threads(max(1, torch.get_num_threads()))
    only = set(argv[2:])
    for sc, mode, prefill in GOLDEN:
        if only and sc.name not in only:
            continue
        t0 = time.time()
        drv = LifecycleDriver(sc, mode, api, "cpu", prefill=prefill)
        recs = drv.run()
        arrays = records_to_arrays(recs, sc.top_k)
        meta = {
            "scenario": sc.name,
            "mode": mode,
            "prefill": prefill,
            "torch": torch.__version__,
            "stats": drv.stats(),
            "records": len(recs),
        }
        path = HERE / fixture_name(sc, mode)
        np.savez_compressed(path, meta=np.array(json.dumps(meta)), **arrays)
        print(f"{path.name}: {len(recs)} records, {path.stat().st_size / 1e3:.0f} kB, "
              f"{time.time() - t0:.1f}s, stats={meta['stats']}")


if __name__ == "__main__":
    main(sys.argv)

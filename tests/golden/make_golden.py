"""Generate the golden fixtures from the reference implementation itself.

Run where the reference package ``qwenquest`` is importable (it is pure
Python + torch, CPU only; ``tests._reference`` finds an install under
``baseline/_ref`` or the directory ``QWENQUEST_REF`` names)::

    python tests/golden/make_golden.py [scenario names...]

For every entry of ``scenarios.GOLDEN`` it drives the reference's
``QuestOnlyBackend`` / ``QuestHiSparseBackend`` (``src/qwenquest/attention``)
through :class:`tests.harness.LifecycleDriver` on CPU with the
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

from tests.golden.scenarios import GOLDEN, fixture_name  # noqa: E402
from tests.harness import LifecycleDriver, records_to_arrays, reference_api  # noqa: E402


def main(argv: list[str]) -> None:
    api = reference_api()
    torch.set_num_threads(max(1, torch.get_num_threads()))
    only = set(argv[1:])
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

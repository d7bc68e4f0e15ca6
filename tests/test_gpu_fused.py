"""Selection and attention in one call (qq_quest_decode_attention) against the two calls (GPU).

``B200QuestOnlyBackend`` makes the fused call when nothing traces the
selection; with a ``QuestTrace`` it makes ``qq_quest_retrieve_topk`` and
``qq_sparse_decode_attention`` in turn.  The fused call runs the same two
kernels (the attention kernel only starts earlier and reads each request's
rows behind that request's ready word), so every decode output must be
bit-identical to the two-call run of the same scenario: ragged lengths,
dense fallbacks, requests that finish and admit new ones mid-run, and
enough requests that the selection splits requests into parts and the
attention splits segments across warps and blocks, and a batch of more
requests than the GPU has SMs (dense and sparse mixed).
"""

from __future__ import annotations

import numpy as np
import pytest

from tests.harness import LifecycleDriver, b200_api
from tests.workloads import Scenario
from tests.test_gpu_configs import CONFIG2_SAMPLE

pytestmark = pytest.mark.gpu

_rng = np.random.default_rng(11)
WIDE = Scenario(
    name="fused_wide", layers=2, q_heads=32, kv_heads=4, head_dim=128, bf16=True,
    top_k=2048, page_size=64, device_buffer_size=4096,
    prompt_lens=tuple(int(x) for x in _rng.integers(1200, 9000, size=28)),
    new_tokens=tuple(int(x) for x in _rng.integers(2, 6, size=28)),
    max_running=20, max_context_len=9216, seed=4, planted_pages=1, q_decode_only=True,
)


_rng2 = np.random.default_rng(12)
MANY = Scenario(
    name="fused_many", layers=1, q_heads=32, kv_heads=4, head_dim=128, bf16=True,
    top_k=2048, page_size=64, device_buffer_size=4096,
    prompt_lens=tuple(int(x) for x in _rng2.integers(300, 3000, size=160)),
    new_tokens=tuple(int(x) for x in _rng2.integers(2, 4, size=160)),
    max_running=160, max_context_len=3072, seed=6, planted_pages=1, q_decode_only=True,
)


@pytest.mark.parametrize("sc", [CONFIG2_SAMPLE, WIDE, MANY], ids=["config2", "wide", "many"])
def test_fused_call_equals_two_calls(sc, cuda_device):
    two = LifecycleDriver(sc, "quest", b200_api(), cuda_device, prefill="direct", trace=True)
    rec_two = two.run()
    two.backend.synchronize()
    one = LifecycleDriver(sc, "quest", b200_api(), cuda_device, prefill="direct", trace=False)
    rec_one = one.run()
    one.backend.synchronize()
    assert len(rec_one) == len(rec_two) > 0
    for a, b in zip(rec_two, rec_one, strict=True):
        assert (a.step, a.layer, a.req) == (b.step, b.layer, b.req)
        assert np.array_equal(a.out, b.out), (a.step, a.layer, a.req)

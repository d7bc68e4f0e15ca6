"""Scenarios whose reference outputs are committed as golden fixtures.

``make_golden.py`` (beside this file) runs each scenario through the
reference's own backends on CPU and stores what they decided; the tests
regenerate the same seeded inputs with
:func:`tests.workloads.scenario_tensors`.
"""

from __future__ import annotations

from tests.workloads import Scenario

# The budget the reference's engine tests use (tests/test_engine.py:13), the
# tiny model geometry (8 q heads / 2 KV heads / head_dim 16, fp32) and its
# prompt lengths (tests/conftest.py:16-19).
TINY_F32 = Scenario(
    name="tiny_f32", layers=3, q_heads=8, kv_heads=2, head_dim=16, bf16=False,
    top_k=32, page_size=8, device_buffer_size=48, prompt_lens=(90, 107, 64),
    new_tokens=(30, 30, 30), max_running=2, max_context_len=256, seed=11,
)
TINY_F32_AVOID = Scenario(
    name="tiny_f32_avoid", layers=3, q_heads=8, kv_heads=2, head_dim=16, bf16=False,
    top_k=32, page_size=8, device_buffer_size=48, prompt_lens=(90, 107, 64),
    new_tokens=(30, 30, 30), max_running=2, max_context_len=256, seed=12,
    avoid_recent_overlap=True,
)
# bf16 budget of tests/test_bf16.py:15 with its prompt lengths (70, 45)
TINY_BF16 = Scenario(
    name="tiny_bf16", layers=2, q_heads=8, kv_heads=2, head_dim=16, bf16=True,
    top_k=32, page_size=8, device_buffer_size=40, prompt_lens=(70, 45),
    new_tokens=(20, 20), max_running=2, max_context_len=128, seed=13,
)
# one slot reused by four requests in turn (tests/test_engine.py:89-95)
SLOT_REUSE = Scenario(
    name="slot_reuse", layers=2, q_heads=8, kv_heads=2, head_dim=16, bf16=False,
    top_k=32, page_size=8, device_buffer_size=48, prompt_lens=(90, 107, 64, 90),
    new_tokens=(12, 12, 12, 12), max_running=1, max_context_len=256, seed=14,
)
# Qwen3-30B-A3B geometry (32/4 heads, head_dim 128, bf16, top_k 2048, page 64):
# one long request crossing page boundaries, one dense-fallback request.
GEOM_BF16 = Scenario(
    name="geom_bf16", layers=2, q_heads=32, kv_heads=4, head_dim=128, bf16=True,
    top_k=2048, page_size=64, device_buffer_size=2560, prompt_lens=(4150, 1500, 2300),
    new_tokens=(40, 40, 40), max_running=3, max_context_len=4352, seed=15, planted_pages=4,
)
# Benchmark config 0: bs 1, 8192-token prefix, one layer, four planted pages,
# one decode step (seq_len 8193).
CONFIG0 = Scenario(
    name="config0", layers=1, q_heads=32, kv_heads=4, head_dim=128, bf16=True,
    top_k=2048, page_size=64, device_buffer_size=4096, prompt_lens=(8192,),
    new_tokens=(2,), max_running=1, max_context_len=8256, seed=0, planted_pages=4,
)

#: (scenario, mode, prefill) triples with committed fixtures
GOLDEN = [
    (TINY_F32, "quest", "forward"),
    (TINY_F32, "quest_hisparse", "forward"),
    (TINY_F32_AVOID, "quest", "forward"),
    (TINY_F32_AVOID, "quest_hisparse", "forward"),
    (TINY_BF16, "quest", "forward"),
    (TINY_BF16, "quest_hisparse", "forward"),
    (SLOT_REUSE, "quest", "forward"),
    (SLOT_REUSE, "quest_hisparse", "forward"),
    (GEOM_BF16, "quest", "direct"),
    (GEOM_BF16, "quest_hisparse", "direct"),
    (CONFIG0, "quest", "direct"),
]


def fixture_name(sc: Scenario, mode: str) -> str:
    return f"{sc.name}__{mode}.npz"

"""Host-side logic (CPU): the backends' ``--hisparse-config`` handling, the workload generator.

The backends parse their ``sparse_config`` with the reference's own
``parse_hisparse_config`` (``src/qwenquest/config.py:298-359``) and apply the
reference backends' Quest check (``attention/quest_only.py:52-54``); these
tests pin that they accept and reject exactly what the reference does.
"""

from __future__ import annotations

import numpy as np
import pytest
from qwenquest.config import SparseConfig, parse_hisparse_config

from qwenquest_b200.backends import _parse_quest_config
from tests.workloads import Scenario, scenario_tensors


@pytest.mark.parametrize("raw", [{"algorithm": "quest"}, '{"algorithm":"quest","top_k":256,"quest_page_size":16}',
                                 {"algorithm": "quest", "avoid_recent_overlap": True, "device_buffer_size": 8192}])
def test_quest_configs_parse_as_the_reference_does(raw):
    cfg = _parse_quest_config(raw)
    assert isinstance(cfg, SparseConfig)
    assert cfg == parse_hisparse_config(raw)
    assert cfg.avoid_recent_overlap == bool(isinstance(raw, dict) and raw.get("avoid_recent_overlap"))


def test_parsed_objects_pass_through():
    cfg = SparseConfig(top_k=64, quest_page_size=16, algorithm="quest")
    assert _parse_quest_config(cfg) is cfg


@pytest.mark.parametrize("bad", [
    None,
    {"top_k": 64},
    {"top_k": 100, "algorithm": "quest"},
    {"top_k": 64, "device_buffer_size": 32, "algorithm": "quest"},
    {"swap_in_block_size": 0, "algorithm": "quest"},
    {"algorithm": "quest", "quest_page_size": 0},
    "{not json",
])
def test_non_quest_or_invalid_configs_raise_value_error(bad):
    with pytest.raises(ValueError):
        _parse_quest_config(bad)


def test_scenario_tensors_are_seeded_and_bf16_exact():
    sc = Scenario(name="t", layers=2, q_heads=8, kv_heads=2, head_dim=16, bf16=True, top_k=32, page_size=8,
                  device_buffer_size=48, prompt_lens=(40,), new_tokens=(5,), max_running=1, max_context_len=64)
    a, b = scenario_tensors(sc, 0), scenario_tensors(sc, 0)
    for key in ("q", "k", "v"):
        assert np.array_equal(a[key], b[key])
        low = a[key].view(np.uint32) & 0xFFFF
        assert not low.any()
    assert a["k"].shape == (2, 45, 2, 16) and a["q"].shape == (2, 45, 8, 16)

"""Host-side logic (CPU): ``--hisparse-config`` parsing, the workload generator, the lifecycle driver."""

from __future__ import annotations

import sys
from pathlib import Path

import numpy as np
import pytest

from qwenquest_b200.config import SparseConfig, avoid_recent_overlap, parse_hisparse_config
from qwenquest_b200.workloads import Scenario, scenario_tensors

REF_SRC = Path("/root/reference/src")


def test_defaults_follow_upstream():
    cfg = parse_hisparse_config({"algorithm": "quest"})
    assert (cfg.top_k, cfg.device_buffer_size, cfg.quest_page_size) == (2048, 4096, 64)
    assert (cfg.host_to_device_ratio, cfg.swap_in_block_size) == (2, 960)
    assert not avoid_recent_overlap(cfg)


def test_unknown_keys_go_to_the_extra_config():
    cfg = parse_hisparse_config('{"algorithm": "quest", "top_k": 32, "quest_page_size": 8, '
                                '"avoid_recent_overlap": true, "foo": 1}')
    assert cfg.sparse_extra_config == {"avoid_recent_overlap": True, "foo": 1}
    assert avoid_recent_overlap(cfg) and cfg.avoid_recent_overlap


@pytest.mark.parametrize("bad", [
    {"top_k": 100, "algorithm": "quest"},
    {"top_k": 64, "device_buffer_size": 32},
    {"swap_in_block_size": 0},
    {"swap_in_block_size": 2000},
    {"swap_in_block_size": True},
    {"algorithm": "quest", "quest_page_size": 0},
    "{not json",
])
def test_invalid_configs_raise_value_error(bad):
    with pytest.raises(ValueError):
        parse_hisparse_config(bad)


def test_parsed_objects_pass_through():
    cfg = SparseConfig(top_k=64, quest_page_size=16, algorithm="quest")
    assert parse_hisparse_config(cfg) is cfg


@pytest.mark.skipif(not REF_SRC.exists(), reason="reference source not present")
@pytest.mark.parametrize("raw", [None, {"algorithm": "quest"}, '{"algorithm":"quest","top_k":256,"quest_page_size":16}',
                                 {"algorithm": "quest", "avoid_recent_overlap": True, "device_buffer_size": 8192}])
def test_parsing_matches_the_reference(raw):
    sys.path.insert(0, str(REF_SRC))
    from qwenquest.config import parse_hisparse_config as ref_parse

    a, b = parse_hisparse_config(raw), ref_parse(raw)
    for name in ("top_k", "device_buffer_size", "host_to_device_ratio", "swap_in_block_size", "algorithm",
                 "quest_page_size", "sparse_extra_config", "avoid_recent_overlap"):
        assert getattr(a, name) == getattr(b, name), name


def test_scenario_tensors_are_seeded_and_bf16_exact():
    sc = Scenario(name="t", layers=2, q_heads=8, kv_heads=2, head_dim=16, bf16=True, top_k=32, page_size=8,
                  device_buffer_size=48, prompt_lens=(40,), new_tokens=(5,), max_running=1, max_context_len=64)
    a, b = scenario_tensors(sc, 0), scenario_tensors(sc, 0)
    for key in ("q", "k", "v"):
        assert np.array_equal(a[key], b[key])
        low = a[key].view(np.uint32) & 0xFFFF
        assert not low.any()
    assert a["k"].shape == (2, 45, 2, 16) and a["q"].shape == (2, 45, 8, 16)

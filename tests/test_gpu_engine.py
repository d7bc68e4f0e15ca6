"""The drop-in seam: the reference ``Engine.generate`` with the B200 backends injected (GPU).

``B200Engine`` overrides the reference's ``Engine._make_backend``
(``src/qwenquest/engine.py:115-135``), which is the whole integration; everything else
is the reference's own code: its tiny Qwen3-MoE (``tiny_config(num_hidden_layers=3)``,
``init_random_weights(seed=0, std=0.05)``, as its ``tests/conftest.py``),
its engine, scheduler, pools and model, on ``cuda:0``.  The checks follow the
reference's ``tests/test_engine.py``:

* generated tokens equal the reference's own Quest backend's (Mode 2) run by
  the same engine on the same GPU, logits within 1e-4 (fp32 model, the
  attention summed in a different order);
* Mode 3 (host tier + LRU hot buffer) equals Mode 2 bit for bit
  (``test_engine.py:59-69``), and the hot buffer really swapped;
* every sparse decode output equals ``decode_attention`` over the traced
  positions (``test_engine.py:98-124``, 1e-6 on fp32);
* reused request slots give the same results (``test_engine.py:86-96``).
"""

from __future__ import annotations

import json

import pytest
import torch
from qwenquest import Engine, EngineConfig, Qwen3MoeForCausalLM, QuestTrace, init_random_weights, tiny_config
from qwenquest.attention.ops import decode_attention
from qwenquest.config import parse_hisparse_config

from qwenquest_b200 import B200QuestHiSparseBackend, B200QuestOnlyBackend

pytestmark = pytest.mark.gpu

SMALL_QUEST = {"top_k": 32, "quest_page_size": 8, "device_buffer_size": 48}


class B200Engine(Engine):
    """The reference engine with the B200 backends behind its attention seam."""

    def _make_backend(self):
        cfg = self.config
        if cfg.attention_mode not in ("quest", "quest_hisparse"):
            return super()._make_backend()
        raw = cfg.hisparse_config
        d = dict(json.loads(raw)) if isinstance(raw, str) else dict(raw or {})
        d.setdefault("algorithm", "quest")
        sparse = parse_hisparse_config(d)
        if cfg.attention_mode == "quest":
            return B200QuestOnlyBackend(self.req_to_token_pool, self.token_to_kv_pool, sparse)
        return B200QuestHiSparseBackend(
            self.req_to_token_pool, self.token_to_kv_pool, sparse,
            host_pool_size=cfg.max_running_requests * self.max_context_len, host_device=cfg.host_device,
        )


@pytest.fixture(scope="module")
def model(cuda_device):
    torch.manual_seed(0)
    m = Qwen3MoeForCausalLM(tiny_config(num_hidden_layers=3))
    return init_random_weights(m, seed=0, std=0.05).to(cuda_device)


@pytest.fixture(scope="module")
def prompts():
    gen = torch.Generator().manual_seed(1234)
    return [torch.randint(0, 256, (n,), generator=gen).tolist() for n in (90, 107, 64)]


def _run(engine_cls, model, prompts, mode, cfg=SMALL_QUEST, max_running=2, max_new_tokens=30):
    engine = engine_cls(model, EngineConfig(attention_mode=mode, hisparse_config=cfg,
                                            max_running_requests=max_running, max_context_len=256))
    outs = engine.generate(prompts, return_logits=True, stop_token_ids=[], max_new_tokens=max_new_tokens)
    return engine, outs


def _logits(out):
    return torch.stack(out.logits)


def test_generate_matches_the_reference_backend(model, prompts):
    ref_engine, ref = _run(Engine, model, prompts, "quest")
    engine, ours = _run(B200Engine, model, prompts, "quest")
    assert isinstance(engine.attn_backend, B200QuestOnlyBackend)
    assert not isinstance(ref_engine.attn_backend, B200QuestOnlyBackend)
    for a, b in zip(ref, ours, strict=True):
        assert a.output_ids == b.output_ids
        torch.testing.assert_close(_logits(b), _logits(a), atol=1e-4, rtol=0)


@pytest.mark.parametrize("avoid_recent_overlap", [False, True])
def test_hisparse_equals_quest_bit_for_bit(model, prompts, avoid_recent_overlap):
    cfg = {**SMALL_QUEST, "avoid_recent_overlap": avoid_recent_overlap}
    _, quest = _run(B200Engine, model, prompts, "quest", cfg)
    engine, hisparse = _run(B200Engine, model, prompts, "quest_hisparse", cfg)
    assert isinstance(engine.attn_backend, B200QuestHiSparseBackend)
    for a, b in zip(quest, hisparse, strict=True):
        assert a.output_ids == b.output_ids
        assert torch.equal(_logits(a), _logits(b))
    stats = engine.attn_backend.coord.stats
    assert stats.misses > 0 and stats.hits > 0  # the hot buffer really had to swap
    assert engine.allocator.available_size() == engine.token_to_kv_pool.size


def test_attention_reads_exactly_the_traced_positions(model, prompts):
    engine = B200Engine(model, EngineConfig(attention_mode="quest", hisparse_config=SMALL_QUEST,
                                            max_context_len=256))
    quest = engine.quest
    quest.trace = QuestTrace()
    backend = engine.attn_backend
    original = backend.forward_decode
    checked: list[bool] = []

    def spy(q, k, v, layer, batch):
        out = original(q, k, v, layer, batch)
        rec = quest.trace.records[-1]
        assert rec.layer_id == layer.layer_id and not rec.dense
        req = int(batch.req_pool_indices[0])
        slots = engine.req_to_token_pool.req_to_token[req, rec.positions.to(q.device)].long()
        k_buf, v_buf = engine.token_to_kv_pool.get_kv_buffer(layer.layer_id)
        expected = decode_attention(q[0], k_buf[slots], v_buf[slots], layer.scaling)
        checked.append(torch.allclose(out[0], expected, atol=1e-6))
        return out

    backend.forward_decode = spy
    engine.generate([prompts[1]], max_new_tokens=3, stop_token_ids=[])
    assert len(checked) == 2 * model.config.num_hidden_layers and all(checked)


@pytest.mark.parametrize("mode", ["quest", "quest_hisparse"])
def test_request_slots_are_reused_cleanly(model, prompts, mode):
    _, sequential = _run(B200Engine, model, prompts * 2, mode, max_running=1)
    for first, second in zip(sequential[:3], sequential[3:], strict=True):
        assert first.output_ids == second.output_ids
        assert torch.equal(_logits(first), _logits(second))

"""Qwen3-MoE expert block on the tensor cores (``qq_moe_experts``) against the reference (GPU).

``B200SparseMoeBlock`` wraps a reference ``Qwen3MoeSparseMoeBlock`` and shares its
weights; its routing is the reference's own torch code, so both route every
token to the same experts.  Compared with the reference block run on the same
GPU in bf16 and with the numpy oracle (``oracle/moe.py``).  Tolerance: two
bf16 steps of the output's scale (max |ref|): every tensor the reference
makes is rounded to bf16, and the GEMMs sum their products in a different
order than cuBLAS, so a rounding can land one step apart, and a step in an
intermediate moves the output by at most about one step of its scale.
"""

from __future__ import annotations

import numpy as np
import pytest
import torch

from oracle.moe import sparse_moe_block
from qwenquest_b200.moe import B200SparseMoeBlock, install_moe, moe_plan

pytestmark = pytest.mark.gpu


def _block(hidden, inter, experts, top_k, seed, std=0.02):
    from qwenquest.config import Qwen3MoeConfig
    from qwenquest.model.qwen3_moe import Qwen3MoeSparseMoeBlock

    cfg = Qwen3MoeConfig(hidden_size=hidden, moe_intermediate_size=inter, num_experts=experts,
                         num_experts_per_tok=top_k, norm_topk_prob=True)
    dev = torch.device("cuda", 0)
    with torch.device(dev):
        blk = Qwen3MoeSparseMoeBlock(cfg).to(torch.bfloat16)
    g = torch.Generator(device=dev).manual_seed(seed)
    with torch.no_grad():
        for p in blk.parameters():
            p.copy_(torch.randn(p.shape, generator=g, device=dev) * std)
    return blk


def _tol(ref: torch.Tensor) -> float:
    return 2 * 2.0 ** -8 * float(ref.abs().max())


@pytest.mark.parametrize("tokens", [1, 5, 300])
def test_small_geometry_matches_reference_and_oracle(tokens):
    blk = _block(256, 128, 16, 4, seed=tokens)
    x = torch.randn(tokens, 256, generator=torch.Generator().manual_seed(7)).to(torch.bfloat16).cuda()
    ours = B200SparseMoeBlock(blk)
    with torch.no_grad():
        out = ours(x)
        ref = blk(x)
    ours.check_errors()
    assert float((out.float() - ref.float()).abs().max()) <= _tol(ref)
    f = lambda t: t.detach().float().cpu().numpy()  # noqa: E731
    ora = sparse_moe_block(f(x), f(blk.gate.weight), np.stack([f(m.gate_proj.weight) for m in blk.experts]),
                           np.stack([f(m.up_proj.weight) for m in blk.experts]),
                           np.stack([f(m.down_proj.weight) for m in blk.experts]), 4, True, bf16=True)
    assert float(np.abs(f(out) - ora).max()) <= _tol(ref)


@pytest.mark.parametrize("tokens", [8, 1000])
def test_qwen3_30b_geometry_matches_reference(tokens):
    """hidden 2048, 128 experts of 768, top 8: config 4's decode batch (8 tokens) and a prefill chunk."""
    blk = _block(2048, 768, 128, 8, seed=3)
    x = torch.randn(tokens, 2048, generator=torch.Generator().manual_seed(tokens)).to(torch.bfloat16).cuda()
    ours = B200SparseMoeBlock(blk)
    with torch.no_grad():
        out = ours(x)
        ref = blk(x)
    ours.check_errors()
    err = float((out.float() - ref.float()).abs().max())
    assert err <= _tol(ref), (err, float(ref.abs().max()))
    # most elements are bit-identical to the reference
    assert float((out == ref).float().mean()) > 0.9


def test_plan_groups_pairs_by_expert_tokens_ascending():
    experts = torch.tensor([[3, 1], [1, 0], [3, 2], [0, 1]], device="cuda")
    weights = torch.rand(4, 2, device="cuda").to(torch.bfloat16)
    pt, pw, off, tp = moe_plan(experts, weights, 4)
    assert off.tolist() == [0, 2, 5, 6, 8]
    assert pt.tolist() == [1, 3, 0, 1, 3, 2, 0, 2]  # expert 0: tokens 1, 3; expert 1: 0, 1, 3; ...
    for t in range(4):
        for s in range(2):
            p = int(tp[t, s])
            assert int(pt[p]) == t and bool(pw[p] == weights[t, s])


def test_install_replaces_every_moe_block():
    from qwenquest import Qwen3MoeForCausalLM, tiny_config

    model = Qwen3MoeForCausalLM(tiny_config(num_hidden_layers=3, hidden_size=256, moe_intermediate_size=128,
                                            num_attention_heads=8, num_key_value_heads=2, head_dim=32))
    assert install_moe(model) == 3
    assert all(isinstance(layer.mlp, B200SparseMoeBlock) for layer in model.model.layers)


def test_forward_makes_no_host_sync():
    """Routing, plan and experts are all queued without waiting for the GPU (graph-friendly)."""
    blk = _block(256, 128, 16, 4, seed=9)
    x = torch.randn(64, 256, generator=torch.Generator().manual_seed(1)).to(torch.bfloat16).cuda()
    ours = B200SparseMoeBlock(blk)
    with torch.no_grad():
        ours(x)  # first call: pointer tables
        torch.cuda.synchronize()
        torch.cuda.set_sync_debug_mode("error")
        try:
            out = ours(x)
        finally:
            torch.cuda.set_sync_debug_mode(0)
        ref = blk(x)
    assert float((out.float() - ref.float()).abs().max()) <= _tol(ref)


@pytest.mark.parametrize("tokens", [1, 8, 200, 256])
def test_device_plan_equals_torch_plan(tokens):
    from qwenquest_b200.moe import device_moe_plan

    g = torch.Generator(device="cuda").manual_seed(tokens)
    logits = torch.randn(tokens, 128, generator=g, device="cuda")
    weights, experts = torch.topk(torch.softmax(logits, -1), 8, dim=-1)
    weights = weights.to(torch.bfloat16)
    got = device_moe_plan(experts, weights, 128)
    want = moe_plan(experts, weights, 128)
    for a, b in zip(got, want, strict=True):
        assert torch.equal(a.view(-1).to(b.dtype), b.view(-1)), (a, b)

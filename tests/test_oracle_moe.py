"""The oracle's MoE block pinned to the reference's own ``Qwen3MoeSparseMoeBlock`` (CPU).

``oracle.moe.sparse_moe_block`` restates ``model/qwen3_moe.py:121-147``; both
run on the same seeded weights and tokens on the CPU: in float32 they agree
within 1e-5, in bf16 (the reference rounds each tensor it makes) within two
bf16 steps of the output's scale, since the two sum their products in
different orders before each rounding.
"""

from __future__ import annotations

import numpy as np
import pytest
import torch

from oracle.moe import sparse_moe_block


def _block(hidden, inter, experts, top_k, dtype, seed):
    from qwenquest.config import Qwen3MoeConfig
    from qwenquest.model.qwen3_moe import Qwen3MoeSparseMoeBlock

    cfg = Qwen3MoeConfig(hidden_size=hidden, moe_intermediate_size=inter, num_experts=experts,
                         num_experts_per_tok=top_k, norm_topk_prob=True)
    torch.manual_seed(seed)
    blk = Qwen3MoeSparseMoeBlock(cfg)
    with torch.no_grad():
        for p in blk.parameters():
            p.normal_(0.0, 0.05)
    return blk.to(dtype)


def weights_of(blk):
    ex = blk.experts
    f = lambda t: t.detach().float().numpy()  # noqa: E731
    return (f(blk.gate.weight), np.stack([f(m.gate_proj.weight) for m in ex]),
            np.stack([f(m.up_proj.weight) for m in ex]), np.stack([f(m.down_proj.weight) for m in ex]))


@pytest.mark.parametrize("dtype", [torch.float32, torch.bfloat16])
def test_oracle_matches_reference_moe_block(dtype):
    blk = _block(64, 32, 8, 2, dtype, seed=1)
    x = torch.randn(13, 64, generator=torch.Generator().manual_seed(2)).to(dtype)
    with torch.no_grad():
        ref = blk(x).float().numpy()
    gw, wg, wu, wd = weights_of(blk)
    ora = sparse_moe_block(x.float().numpy(), gw, wg, wu, wd, 2, True, bf16=dtype == torch.bfloat16)
    if dtype == torch.float32:
        assert float(np.abs(ora - ref).max()) <= 1e-5
    else:
        scale = float(np.abs(ref).max())
        assert float(np.abs(ora - ref).max()) <= 2 * 2.0 ** -8 * scale

"""Host-side behaviour of the MoE drop-in (CPU): ``install_moe`` keeps the model's parameter
names, is idempotent, and a block the kernels cannot take runs the reference's own forward."""

from __future__ import annotations

import torch

from qwenquest_b200.moe import B200SparseMoeBlock, install_moe, moe_plan


def test_install_keeps_state_dict_and_falls_back_off_gpu():
    from qwenquest import Qwen3MoeForCausalLM, tiny_config

    torch.manual_seed(0)
    model = Qwen3MoeForCausalLM(tiny_config(num_hidden_layers=2))
    keys = list(model.state_dict().keys())
    x = torch.randn(5, model.config.hidden_size)
    ref = model.model.layers[0].mlp(x)
    assert install_moe(model) == 2
    assert install_moe(model) == 0  # already installed
    assert list(model.state_dict().keys()) == keys
    assert all(isinstance(layer.mlp, B200SparseMoeBlock) for layer in model.model.layers)
    assert torch.equal(model.model.layers[0].mlp(x), ref)  # CPU tensors: the reference's forward


def test_plan_offsets_and_pair_order_on_cpu():
    experts = torch.tensor([[5, 2], [2, 7], [0, 5]])
    weights = torch.arange(6, dtype=torch.float32).view(3, 2).to(torch.bfloat16)
    pt, pw, off, tp = moe_plan(experts, weights, 8)
    assert off.tolist() == [0, 1, 1, 3, 3, 3, 5, 5, 6]
    assert pt.tolist() == [2, 0, 1, 0, 2, 1]  # expert 0: token 2; 2: tokens 0, 1; 5: 0, 2; 7: 1
    for t in range(3):
        for s in range(2):
            assert int(pt[tp[t, s]]) == t and float(pw[tp[t, s]]) == float(weights[t, s])

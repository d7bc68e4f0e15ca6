"""Drop-in for the reference's ``Qwen3MoeSparseMoeBlock`` (``model/qwen3_moe.py:121-147``).

:class:`B200SparseMoeBlock` is a subclass of the reference block that takes
over a block's own ``gate`` and ``experts`` modules (nothing is copied, and
the parameter names of the model's ``state_dict`` stay the same).  ``forward`` computes the routing with the reference's
own torch operations (``qwen3_moe.py:133-138``: gate logits, fp32 softmax,
top-k, renormalisation, cast to the logits' dtype), groups the (token, slot)
pairs by expert, tokens ascending within an expert (the order ``torch.where``
gives the reference's loop: one ``qq_moe_route_plan`` launch for small
batches, a stable torch sort for large ones), and runs the expert loop
(``qwen3_moe.py:139-147``) as one ``qq_moe_experts`` call: two grouped GEMMs
on the tcgen05 tensor cores and a combine, no host synchronisation.
Geometries the kernels do not take (not bf16, hidden not a multiple of 256,
intermediate not a multiple of 128, more than 16 experts per token) run the
reference's own ``forward``.

:func:`install_moe` swaps every MoE block of a reference
``Qwen3MoeForCausalLM`` for the drop-in.
"""

from __future__ import annotations

import torch
import torch.nn.functional as F
from torch import nn

from qwenquest_b200 import _lib
from qwenquest_b200._lib import check
from qwenquest_b200.quest import stream_of

__all__ = ["B200SparseMoeBlock", "device_moe_plan", "install_moe", "moe_plan"]


def moe_plan(experts: torch.Tensor, weights: torch.Tensor, num_experts: int):
    """The (token, slot) pairs of a routing grouped by expert: ``pair_token`` (int32),
    ``pair_weight`` (the routing weights' dtype), ``offsets`` (int64 ``[E + 1]``) and
    ``token_pairs`` (int32 ``[T, k]``: the pair of each token's slot), all on the device."""
    tokens, k = experts.shape
    flat = experts.reshape(-1)
    order = torch.argsort(flat, stable=True)  # by expert; within one, by token then slot
    pair_token = torch.div(order, k, rounding_mode="floor").to(torch.int32)
    pair_weight = weights.reshape(-1)[order].contiguous()
    # expert e's pairs start at the first sorted id >= e (no host synchronisation, unlike bincount)
    bounds = torch.arange(num_experts + 1, dtype=flat.dtype, device=experts.device)
    offsets = torch.searchsorted(flat[order].contiguous(), bounds).to(torch.int64)
    token_pairs = torch.empty(tokens * k, dtype=torch.int32, device=experts.device)
    token_pairs[order] = torch.arange(tokens * k, dtype=torch.int32, device=experts.device)
    return pair_token, pair_weight, offsets, token_pairs.view(tokens, k)


def _reference_block_class():
    from qwenquest.model.qwen3_moe import Qwen3MoeSparseMoeBlock

    return Qwen3MoeSparseMoeBlock


#: routings of at most this many (token, slot) pairs are grouped by one qq_moe_route_plan launch
ROUTE_PLAN_MAX_PAIRS = 2048


def device_moe_plan(experts: torch.Tensor, weights: torch.Tensor, num_experts: int, err_ptr=None):
    """:func:`moe_plan` in one ``qq_moe_route_plan`` launch (CUDA tensors, at most
    ``ROUTE_PLAN_MAX_PAIRS`` pairs); the same arrays, bit for bit."""
    tokens, k = experts.shape
    dev = experts.device
    experts = experts.to(torch.int64).contiguous()
    weights = weights.to(torch.bfloat16).contiguous()
    pairs = tokens * k
    pair_token = torch.empty(pairs, dtype=torch.int32, device=dev)
    pair_weight = torch.empty(pairs, dtype=torch.bfloat16, device=dev)
    offsets = torch.empty(num_experts + 1, dtype=torch.int64, device=dev)
    token_pairs = torch.empty((tokens, k), dtype=torch.int32, device=dev)
    rc = _lib.load().qq_moe_route_plan(experts.data_ptr(), weights.data_ptr(), tokens, k, num_experts,
                                       pair_token.data_ptr(), pair_weight.data_ptr(), offsets.data_ptr(),
                                       token_pairs.data_ptr(), err_ptr, stream_of(dev))
    check(rc, "moe route plan")
    return pair_token, pair_weight, offsets, token_pairs


class B200SparseMoeBlock(_reference_block_class()):
    """The reference block's computation with its expert loop on the B200 kernels."""

    def __init__(self, block: nn.Module):
        nn.Module.__init__(self)  # the block's modules are adopted, not rebuilt
        self.top_k = block.top_k
        self.norm_topk_prob = block.norm_topk_prob
        self.gate = block.gate
        self.experts = block.experts
        self._tables = None
        self._key = None
        self._err = torch.zeros(1, dtype=torch.int32).pin_memory() if torch.cuda.is_available() else None
        self._err_dev = None

    # ------------------------------------------------------------ weights

    def _weights(self):
        ex = self.experts
        return ([m.gate_proj.weight for m in ex], [m.up_proj.weight for m in ex], [m.down_proj.weight for m in ex])

    def _state(self, device):
        """Per-device pointer tables and the geometry check, built once (rebuilt if the
        weights moved: their first and last pointers are compared on every call)."""
        ex = self.experts
        key = (device, ex[0].gate_proj.weight.data_ptr(), ex[-1].down_proj.weight.data_ptr())
        if self._key != key:
            gate, up, down = self._weights()
            inter, hidden = gate[0].shape
            ok = (hidden % 256 == 0 and inter % 128 == 0 and self.top_k <= 16 and len(gate) <= 1024
                  and all(w.dtype == torch.bfloat16 and w.is_contiguous() and w.device == device
                          for ws in (gate, up, down) for w in ws))

            def table(ws):
                return torch.tensor([w.data_ptr() for w in ws], dtype=torch.int64, device=device)

            self._tables = (table(gate), table(up), table(down), ok, hidden, inter, len(gate)) if ok else (
                None, None, None, False, hidden, inter, len(gate))
            self._key = key
        return self._tables

    def supported(self, x: torch.Tensor) -> bool:
        if not (x.is_cuda and x.dim() == 2 and x.dtype == torch.bfloat16):
            return False
        state = self._state(x.device)
        return state[3] and x.shape[1] == state[4]

    # ------------------------------------------------------------ forward

    def forward(self, x: torch.Tensor) -> torch.Tensor:
        if not self.supported(x):
            return super().forward(x)
        # routing: the reference's own operations (qwen3_moe.py:133-138)
        router_logits = self.gate(x)
        probs = F.softmax(router_logits, dim=-1, dtype=torch.float32)
        weights, experts = torch.topk(probs, self.top_k, dim=-1)
        if self.norm_topk_prob:
            weights = weights / weights.sum(dim=-1, keepdim=True)
        weights = weights.to(router_logits.dtype)
        return self.experts_forward(x, experts, weights)

    def experts_forward(self, x: torch.Tensor, experts: torch.Tensor, weights: torch.Tensor) -> torch.Tensor:
        """The expert loop (``qwen3_moe.py:139-147``) for a given routing."""
        lib = _lib.load()
        dev = x.device
        x = x.contiguous()
        tg, tu, td, _, hidden, inter, num_experts = self._state(dev)
        tokens = x.shape[0]
        weights = weights.to(torch.bfloat16)
        if self._err_dev is None:
            from qwenquest_b200.hisparse import host_device_pointer

            self._err_dev = host_device_pointer(self._err)
        if tokens * self.top_k <= ROUTE_PLAN_MAX_PAIRS:
            pair_token, pair_weight, offsets, token_pairs = device_moe_plan(experts, weights, num_experts,
                                                                             self._err_dev)
        else:
            pair_token, pair_weight, offsets, token_pairs = moe_plan(experts, weights, num_experts)
        pairs = pair_token.numel()
        h = torch.empty((pairs, inter), dtype=torch.bfloat16, device=dev)
        y = torch.empty((pairs, hidden), dtype=torch.bfloat16, device=dev)
        out = torch.empty_like(x)
        plan = _lib.QQMoePlan(pair_token.data_ptr(), offsets.data_ptr(), pair_weight.data_ptr(),
                              token_pairs.data_ptr(), tokens, pairs, self.top_k, num_experts)
        rc = lib.qq_moe_experts(plan, x.data_ptr(), x.stride(0), hidden, inter, tg.data_ptr(), tu.data_ptr(),
                                td.data_ptr(), h.data_ptr(), y.data_ptr(), out.data_ptr(), out.stride(0),
                                self._err_dev, stream_of(dev))
        check(rc, "moe experts")
        return out

    def check_errors(self) -> None:
        """Raise for device errors of earlier calls (synchronises the current stream)."""
        torch.cuda.current_stream().synchronize()
        bits = int(self._err[0])
        self._err.zero_()
        _lib.raise_device_error(bits, "(moe)")


def install_moe(model: nn.Module) -> int:
    """Replace every ``Qwen3MoeSparseMoeBlock`` of a reference ``Qwen3MoeForCausalLM`` by
    :class:`B200SparseMoeBlock` (parameters shared); returns how many were replaced."""
    from qwenquest.model.qwen3_moe import Qwen3MoeSparseMoeBlock

    n = 0
    for layer in model.model.layers:
        if isinstance(layer.mlp, Qwen3MoeSparseMoeBlock) and not isinstance(layer.mlp, B200SparseMoeBlock):
            layer.mlp = B200SparseMoeBlock(layer.mlp)
            n += 1
    return n

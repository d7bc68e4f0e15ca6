"""A decode step captured in a CUDA graph and replayed equals the eager steps (GPU).

Two backends built from the same seed (benchmark config 1 geometry, small:
8 requests, 4096-token prefixes, 3 layers) decode the same four steps; the
second runs step 0 eagerly, captures a ``DecodeStepGraph`` and replays it for
steps 1-3 with each step's batch copied in.  Every layer's output must be
bit-identical to the eager backend's (the same kernels on the same data),
whether the graph holds the fused selection + attention call (its epochs
renewed on the device at every replay) or the two separate calls.
"""

from __future__ import annotations

import pytest
import torch

import bench
from qwenquest_b200.graphs import DecodeStepGraph

pytestmark = pytest.mark.gpu

N_REQ, PREFIX, LAYERS, STEPS = 8, 4096, 3, 4


def _setup(dev, fused=False):
    backend, pool, r2t, max_ctx, qkv = bench.build_config1(dev, STEPS + 1, 7, n_req=N_REQ, prefix=PREFIX,
                                                           layers=LAYERS, resident=1)
    batches, layers = bench.make_batches(dev, backend, pool, r2t, max_ctx, STEPS + 1, n_req=N_REQ, prefix=PREFIX)
    backend.fused = fused
    return backend, batches, layers, qkv


def _eager_step(backend, batch, layers, qkv):
    qs, ks, vs = qkv
    backend.init_forward_metadata(batch)
    return [backend.forward(qs[layer.layer_id], ks[layer.layer_id], vs[layer.layer_id], layer, batch).clone()
            for layer in layers]


@pytest.mark.parametrize("fused", [True, False], ids=["fused-call", "two-calls"])
def test_graph_replay_equals_eager_steps(cuda_device, fused):
    dev = torch.device(cuda_device)
    eager, batches, layers, qkv = _setup(dev)
    ref = [_eager_step(eager, batches[s], layers, qkv) for s in range(STEPS)]
    torch.cuda.synchronize(dev)

    graphed, gbatches, glayers, gqkv = _setup(dev, fused)
    first = _eager_step(graphed, gbatches[0], glayers, gqkv)
    for a, b in zip(ref[0], first, strict=True):
        assert torch.equal(a, b)
    g = DecodeStepGraph(graphed, glayers, gbatches[1], *gqkv)
    for s in range(1, STEPS):
        outs = [o.clone() for o in g.replay(gbatches[s])]
        for li, (a, b) in enumerate(zip(ref[s], outs, strict=True)):
            assert torch.equal(a, b), (s, li)
    torch.cuda.synchronize(dev)
    graphed.check_errors()
    eager.check_errors()


def test_graph_rejects_traced_backend(cuda_device):
    from qwenquest_b200.quest import QuestTrace

    dev = torch.device(cuda_device)
    backend, batches, layers, qkv = _setup(dev)
    _eager_step(backend, batches[0], layers, qkv)
    backend.quest.trace = QuestTrace()
    with pytest.raises(ValueError):
        DecodeStepGraph(backend, layers, batches[1], *qkv)

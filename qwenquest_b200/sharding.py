"""Multi-GPU decode: requests sharded across ranks, no collective on the data path.

Decode requests are independent — their KV rows, Quest bounds, hot buffers
and host rows are all per request — so a batch is partitioned by request and
every rank runs the whole decode step for its own requests.  The only
cross-rank traffic is bookkeeping: the maximum of the ranks' timings (the
box is as fast as its slowest GPU) and optional statistics.

* :func:`shard_requests` — contiguous blocks of the batch (equal lengths), or a
  greedy longest-first assignment by the bytes a request moves per layer step
  when lengths are ragged (benchmark config 2).
* :func:`request_layer_bytes` — those bytes (the roofline unit of one request).
* :func:`max_over_ranks` — the slowest rank's value, via the default process
  group (NCCL on GPUs, gloo on the host).
"""

from __future__ import annotations

from collections.abc import Sequence

import torch

__all__ = ["request_layer_bytes", "shard_requests", "max_over_ranks"]


def request_layer_bytes(seq_len: int, top_k: int = 2048, page_size: int = 64, kv_heads: int = 4,
                        head_dim: int = 128, q_heads: int = 32, elem_bytes: int = 2) -> int:
    """Algorithmic bytes one request moves in one layer of one decode step.

    Long request (seq_len > top_k): q + new K/V + bounds append + the (min,
    max) bounds of every complete page + positions + req_to_token + top_k K/V
    rows + output; dense request (seq_len <= top_k): no scores, seq_len rows.
    """
    row = kv_heads * head_dim * elem_bytes          # one K or V row
    q = q_heads * head_dim * elem_bytes
    # q, new K/V, running bounds read + written, positions out, output
    fixed = q + 2 * row + 2 * 2 * row + 4 * top_k + q
    if seq_len > top_k:
        pages = seq_len // page_size               # (min, max) bounds: 2 rows per page
        return fixed + 2 * row * pages + 4 * top_k + 2 * row * top_k
    return fixed + 4 * seq_len + 2 * row * seq_len


def shard_requests(seq_lens: Sequence[int], rank: int, world: int, *, balance: bool = False,
                   **geometry) -> list[int]:
    """Indices of the requests rank ``rank`` of ``world`` decodes.

    Without ``balance``: contiguous blocks, the first ``len % world`` ranks
    one request larger.  With ``balance``: requests sorted by
    :func:`request_layer_bytes` (largest first, ties by index) each go to the
    rank with the fewest bytes so far (ties to the lower rank); each rank's
    list is in ascending request order.
    """
    if world <= 0 or not 0 <= rank < world:
        raise ValueError(f"rank {rank} out of range for world size {world}")
    n = len(seq_lens)
    if not balance:
        base, extra = divmod(n, world)
        start = rank * base + min(rank, extra)
        return list(range(start, start + base + (1 if rank < extra else 0)))
    cost = [request_layer_bytes(int(s), **geometry) for s in seq_lens]
    load = [0] * world
    owner = [0] * n
    for i in sorted(range(n), key=lambda i: (-cost[i], i)):
        r = min(range(world), key=lambda r: (load[r], r))
        owner[i] = r
        load[r] += cost[i]
    return [i for i in range(n) if owner[i] == rank]


def max_over_ranks(values: Sequence[float], device: torch.device | str = "cpu") -> list[float]:
    """Element-wise maximum of ``values`` over all ranks (identity without a process group)."""
    t = torch.tensor([float(v) for v in values], dtype=torch.float64, device=device)
    if torch.distributed.is_available() and torch.distributed.is_initialized():
        torch.distributed.all_reduce(t, op=torch.distributed.ReduceOp.MAX)
    return [float(x) for x in t.cpu()]


def box_totals(times: Sequence[float], counts: Sequence[float], device: torch.device | str = "cpu"
               ) -> tuple[list[float], list[float]]:
    """The box's view of per-rank shards: each of ``times`` as its maximum over the ranks
    (the slowest GPU sets the box's time) and each of ``counts`` summed over the ranks
    (the tokens all shards produced).  Identity without a process group."""
    slowest = max_over_ranks(times, device)
    t = torch.tensor([float(c) for c in counts], dtype=torch.float64, device=device)
    if torch.distributed.is_available() and torch.distributed.is_initialized():
        torch.distributed.all_reduce(t, op=torch.distributed.ReduceOp.SUM)
    return slowest, [float(x) for x in t.cpu()]

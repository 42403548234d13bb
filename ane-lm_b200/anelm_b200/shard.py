"""Multi-GPU plumbing for the attention core: one process per GPU.

Batched serving decode shards by sequence and needs no collective on the data
path: each rank owns whole sequences (their KV rings and DeltaNet states) and
decodes them with its own context.  This module holds the host-side pieces:

* `assign_sequences` -- which sequences a rank owns.  Weak scaling gives every
  rank its own set; strong scaling splits one global set with greedy
  longest-first bin packing on each sequence's bytes touched per decode step
  (KV rows + DeltaNet state), so ragged lengths still balance.
* `max_over_ranks` -- the step time reported for a multi-GPU run (the slowest
  rank), one all-reduce outside the timed region.
* `gather_heads` -- the single collective of head-sharded prefill: every rank
  computed the output columns of its heads; one all-gather and a transpose give
  every rank the full [tokens][Hq*d] output.

Works with any torch.distributed backend (NCCL on GPUs, gloo in the CPU tests).
"""
from __future__ import annotations

import heapq
from typing import Sequence


def seq_step_bytes(kv_len: int, n_fa_layers: int, n_kv_heads: int, head_dim: int, n_gdn_layers: int,
                   n_val_heads: int, key_dim: int = 128, val_dim: int = 128) -> int:
    """HBM bytes one decode step of one sequence touches: fp16 K and V rows of every
    full-attention layer plus the fp32 DeltaNet state read and written per linear layer."""
    kv = 2 * kv_len * n_kv_heads * head_dim * 2 * n_fa_layers
    state = 2 * n_val_heads * key_dim * val_dim * 4 * n_gdn_layers
    return kv + state


def assign_sequences(costs: Sequence[float], world: int, rank: int, mode: str = "strong") -> list[int]:
    """Indices of the sequences rank `rank` owns.

    mode "strong": the len(costs) sequences are split over `world` ranks by greedy
    longest-first bin packing (largest cost to the currently lightest rank; ties to
    the lower rank), so every rank's total cost is within one sequence of the mean.
    mode "weak": every rank owns all of them (its own copy of the per-GPU workload).
    """
    if world < 1 or not 0 <= rank < world:
        raise ValueError(f"rank {rank} of world {world}")
    n = len(costs)
    if mode == "weak":
        return list(range(n))
    if mode != "strong":
        raise ValueError(mode)
    order = sorted(range(n), key=lambda i: (-costs[i], i))
    heap = [(0.0, r) for r in range(world)]
    owned: list[list[int]] = [[] for _ in range(world)]
    for i in order:
        load, r = heapq.heappop(heap)
        owned[r].append(i)
        heapq.heappush(heap, (load + costs[i], r))
    return sorted(owned[rank])


def max_over_ranks(value: float, device=None) -> float:
    """The largest `value` over all ranks (identity without an initialised process group)."""
    import torch
    import torch.distributed as dist

    if not (dist.is_available() and dist.is_initialized()):
        return float(value)
    t = torch.tensor([float(value)], dtype=torch.float64, device=device)
    dist.all_reduce(t, op=dist.ReduceOp.MAX)
    return float(t.item())


def head_shard(n_q_heads: int, n_kv_heads: int, world: int, rank: int):
    """Query heads and kv head owned by `rank` for head-sharded prefill.

    KV-head groups are spread over the ranks; with more ranks than KV heads each
    group's query heads are split further and that group's K/V is duplicated.
    Returns (q_heads, kv_heads): lists of global head indices, in order."""
    G = n_q_heads // n_kv_heads
    if world <= n_kv_heads:
        if n_kv_heads % world:
            raise ValueError("kv heads must divide evenly over the ranks")
        per = n_kv_heads // world
        kvs = list(range(rank * per, (rank + 1) * per))
        return [kv * G + g for kv in kvs for g in range(G)], kvs
    if world % n_kv_heads or n_q_heads % world:
        raise ValueError("ranks must be a multiple of the kv heads and divide the q heads")
    split = world // n_kv_heads           # ranks per kv group
    kv = rank // split
    per = G // split
    part = rank % split
    return [kv * G + part * per + g for g in range(per)], [kv]


def value_head_shard(n_key_heads: int, n_val_heads: int, world: int, rank: int):
    """Key and value heads owned by `rank` for value-head-sharded Gated DeltaNet prefill.

    Value heads are split into `world` contiguous blocks; a rank also takes the key heads
    its value heads read (value head h reads key head h // (Hv / Hk), qwen3_5.cpp:880-890),
    so a key head is duplicated when its value heads land on different ranks.
    Returns (key_heads, val_heads): lists of global head indices, in order."""
    if n_val_heads % n_key_heads:
        raise ValueError("value heads must be a multiple of the key heads")
    if n_val_heads % world:
        raise ValueError("value heads must divide evenly over the ranks")
    ratio = n_val_heads // n_key_heads
    per = n_val_heads // world
    vals = list(range(rank * per, (rank + 1) * per))
    keys = sorted({h // ratio for h in vals})
    return keys, vals


def gather_heads(local_out, n_q_heads: int, n_kv_heads: int, head_dim: int, group=None):
    """All-gather of head-sharded outputs: local_out [tokens][len(my q heads) * head_dim]
    on every rank -> [tokens][n_q_heads * head_dim] in global head order.

    head_shard gives every rank a contiguous block of query heads, in rank order, all of the
    same size, so one all_gather_into_tensor ([world][tokens][cols]) and one transpose to
    [tokens][world][cols] put every column in place."""
    import torch
    import torch.distributed as dist

    world = dist.get_world_size(group)
    for r in range(world):  # the layout this relies on (cheap host-side check)
        qh, _ = head_shard(n_q_heads, n_kv_heads, world, r)
        assert qh == list(range(r * len(qh), (r + 1) * len(qh))), "head shards must be contiguous and in rank order"
    tokens, cols = local_out.shape
    parts = torch.empty(world * tokens, cols, dtype=local_out.dtype, device=local_out.device)
    dist.all_gather_into_tensor(parts, local_out.contiguous(), group=group)
    return parts.view(world, tokens, cols).transpose(0, 1).reshape(tokens, world * cols)

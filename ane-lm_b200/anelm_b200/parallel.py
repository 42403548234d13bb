"""Head-sharded causal prefill over several GPUs (one process per GPU).

A single long prompt does not split by sequence, so its full-attention prefill
splits by head: each rank computes the query heads of its KV-head groups
(`shard.head_shard`), on the columns of the projection rows that belong to
them, with its own context of `len(q heads)` / `len(kv heads)` heads.  The one
collective is the all-gather of the gated outputs (`shard.gather_heads`), after
which every rank holds the full [tokens][Hq * d] output.  Every rank also keeps
the K/V ring of its own KV heads for the decode that follows.
"""
from __future__ import annotations

import torch

from .shard import gather_heads, head_shard


def local_proj_columns(n_q_heads: int, n_kv_heads: int, head_dim: int, q_heads, kv_heads) -> torch.Tensor:
    """Indices of the projection columns [q_gate (Hq*2d) | k (Hkv*d) | v (Hkv*d)]
    (models/llm/qwen3_5.cpp:948-950) that a rank owning q_heads / kv_heads needs,
    in the order its own context expects."""
    d = head_dim
    cols = []
    for h in q_heads:
        cols.extend(range(h * 2 * d, (h + 1) * 2 * d))
    k0 = n_q_heads * 2 * d
    for kv in kv_heads:
        cols.extend(range(k0 + kv * d, k0 + (kv + 1) * d))
    v0 = k0 + n_kv_heads * d
    for kv in kv_heads:
        cols.extend(range(v0 + kv * d, v0 + (kv + 1) * d))
    return torch.tensor(cols, dtype=torch.long)


def sharded_full_attn_prefill(ctx, plan, layer: int, proj: torch.Tensor, n_q_heads: int, n_kv_heads: int,
                              head_dim: int, start_pos: int = 0, out_dtype=torch.float32, group=None):
    """proj: full projection rows [tokens][Hq*2d + 2*Hkv*d] (same on every rank).
    `ctx` is this rank's context built for its shard (head_shard) and `plan` a plan
    of one sequence in it.  Returns the full gated output [tokens][Hq*d] on every rank."""
    import torch.distributed as dist

    world = dist.get_world_size(group) if dist.is_initialized() else 1
    rank = dist.get_rank(group) if dist.is_initialized() else 0
    q_heads, kv_heads = head_shard(n_q_heads, n_kv_heads, world, rank)
    cols = local_proj_columns(n_q_heads, n_kv_heads, head_dim, q_heads, kv_heads).to(proj.device)
    local = proj.index_select(1, cols).unsqueeze(0).contiguous()
    out_local = ctx.full_attn_prefill(plan, layer, local, start_pos, out_dtype=out_dtype)[0]
    if world == 1:
        return out_local
    return gather_heads(out_local, n_q_heads, n_kv_heads, head_dim, group)

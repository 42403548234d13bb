"""Head-sharded prefill over several GPUs (one process per GPU).

A single long prompt does not split by sequence, so its full-attention prefill
splits by head: each rank computes the query heads of its KV-head groups
(`shard.head_shard`), on the columns of the projection rows that belong to
them, with its own context of `len(q heads)` / `len(kv heads)` heads.  The one
collective is the all-gather of the gated outputs (`shard.gather_heads`), after
which every rank holds the full [tokens][Hq * d] output.  Every rank also keeps
the K/V ring of its own KV heads for the decode that follows.

The chunked Gated DeltaNet prefill splits the same way by value head
(`shard.value_head_shard`): each rank runs the chunked delta rule on its value
heads (and the key heads they read) and updates its heads' state; one all-gather
rebuilds the outputs of all heads.
"""
from __future__ import annotations

import torch

from .shard import gather_heads, head_shard, value_head_shard


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


def sharded_gated_delta_chunked(q, k, v, log_decay, beta, state, delta_mode: int = 0, y_dtype=torch.float32,
                                group=None):
    """The chunked delta rule (core.gated_delta_chunked) sharded by value head over the ranks.

    Inputs are the full tensors on every rank: q, k [B][T][Hk][dk], v [B][T][Hv][dv], log_decay,
    beta [B][T][Hv] float32, state [B][Hv][dk][dv] float32.  Each rank computes its value heads and
    writes their final state into `state` in place (other heads' state is left as it was); the
    outputs of every head are all-gathered, so every rank returns y [B][T][Hv][dv]."""
    import torch.distributed as dist

    from .core import gated_delta_chunked

    world = dist.get_world_size(group) if dist.is_initialized() else 1
    rank = dist.get_rank(group) if dist.is_initialized() else 0
    Hk, Hv = q.shape[2], v.shape[2]
    keys, vals = value_head_shard(Hk, Hv, world, rank)
    k0, k1, v0, v1 = keys[0], keys[-1] + 1, vals[0], vals[-1] + 1
    st = state[:, v0:v1].contiguous()
    y = gated_delta_chunked(q[:, :, k0:k1].contiguous(), k[:, :, k0:k1].contiguous(), v[:, :, v0:v1].contiguous(),
                            log_decay[:, :, v0:v1].contiguous(), beta[:, :, v0:v1].contiguous(), st, delta_mode,
                            y_dtype=y_dtype)
    state[:, v0:v1] = st
    if world == 1:
        return y
    parts = [torch.empty_like(y) for _ in range(world)]
    dist.all_gather(parts, y.contiguous(), group=group)
    return torch.cat(parts, dim=2)

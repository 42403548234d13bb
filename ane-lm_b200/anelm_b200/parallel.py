"""Head-sharded prefill over several GPUs (one process per GPU).

A single long prompt does not split by sequence, so its full-attention prefill
splits by head: each rank computes the query heads of its KV-head groups
(`shard.head_shard`), on the columns of the projection rows that belong to
them, with its own context of `len(q heads)` / `len(kv heads)` heads.  The one
collective is the all-gather of the gated outputs (`shard.gather_heads`), after
which every rank holds the full [tokens][Hq * d] output.  Every rank also keeps
the K/V ring of its own KV heads for the decode that follows.

`PeerOutputs` + `fused_sharded_full_attn_prefill` do the same without a separate
collective moving the data: every rank's attention kernel stores its output tiles
straight into every rank's output buffer (CUDA IPC mappings of the peers' buffers,
TMA tile stores over NVLink, anelm_full_attn_prefill_gather), and one one-element
all-reduce on the same stream marks that all ranks' stores have completed.

The chunked Gated DeltaNet prefill splits the same way by value head
(`shard.value_head_shard`): each rank runs the chunked delta rule on its value
heads (and the key heads they read) and updates its heads' state; one all-gather
rebuilds the outputs of all heads.
"""
from __future__ import annotations

import ctypes

import torch

from ._lib import check, lib
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


class PeerOutputs:
    """One output buffer per rank, [B][tokens][cols] of a 16-bit dtype, with every peer's buffer
    mapped into this process (CUDA IPC over the process group).  `ptrs` lists, for ranks 0..world-1,
    the address this rank writes that rank's buffer through; `local` is this rank's own buffer."""

    def __init__(self, shape, dtype, device, group=None):
        import torch.distributed as dist

        self.group = group
        self.world = dist.get_world_size(group)
        self.rank = dist.get_rank(group)
        self.local = torch.empty(shape, dtype=dtype, device=device)
        self.flag = torch.zeros(1, dtype=torch.int32, device=device)
        handle = (ctypes.c_ubyte * 64)()
        off = ctypes.c_size_t()
        check(lib().anelm_ipc_handle(ctypes.c_void_p(self.local.data_ptr()), handle, ctypes.byref(off)),
              "anelm_ipc_handle")
        blob = torch.tensor(list(bytes(handle)) + list(off.value.to_bytes(8, "little")), dtype=torch.uint8,
                            device=device)
        blobs = torch.empty(self.world, blob.numel(), dtype=torch.uint8, device=device)
        dist.all_gather_into_tensor(blobs, blob, group=group)
        blobs = blobs.cpu().numpy()
        self.ptrs, self._opened = [], []
        dev = device.index if hasattr(device, "index") and device.index is not None else torch.cuda.current_device()
        for r in range(self.world):
            if r == self.rank:
                self.ptrs.append(self.local.data_ptr())
                continue
            h = (ctypes.c_ubyte * 64)(*blobs[r, :64].tolist())
            p = ctypes.c_void_p()
            check(lib().anelm_ipc_open(h, int.from_bytes(bytes(blobs[r, 64:72].tolist()), "little"), dev,
                                       ctypes.byref(p)), "anelm_ipc_open")
            self.ptrs.append(p.value)
            self._opened.append(p.value)
        self.arr = (ctypes.c_void_p * self.world)(*self.ptrs)

    def close(self):
        """Unmaps the peers' buffers (after a barrier: no rank may still be writing into them)."""
        import torch.distributed as dist

        torch.cuda.synchronize()
        dist.barrier(group=self.group)
        for p in self._opened:
            lib().anelm_ipc_close(ctypes.c_void_p(p))
        self._opened = []


def fused_sharded_full_attn_prefill(ctx, plan, layer: int, local_proj: torch.Tensor, peers: PeerOutputs,
                                    n_q_heads: int, n_kv_heads: int, head_dim: int, start_pos: int = 0):
    """Head-sharded prefill with the all-gather inside the attention kernel.  local_proj
    [B][tokens][this rank's projection columns] (parallel.local_proj_columns order); `peers` holds
    [B][tokens][n_q_heads * head_dim] outputs.  Returns this rank's full output (peers.local), valid
    once the returned call's stream reaches it."""
    import torch.distributed as dist

    from .core import _dtype_code, _stream

    world, rank = peers.world, peers.rank
    q_heads, _ = head_shard(n_q_heads, n_kv_heads, world, rank)
    n = local_proj.shape[1]
    check(lib().anelm_full_attn_prefill_gather(ctx.handle, plan.handle, layer, n, ctypes.c_void_p(local_proj.data_ptr()),
                                               _dtype_code(local_proj), start_pos, peers.arr, world,
                                               q_heads[0] * head_dim, n_q_heads * head_dim,
                                               _dtype_code(peers.local), _stream(local_proj.device)),
          "anelm_full_attn_prefill_gather")
    # stream-ordered: this all-reduce completes on a rank only after every rank's prefill kernels have
    # completed, and with them their stores into this rank's buffer
    dist.all_reduce(peers.flag, group=peers.group)
    return peers.local

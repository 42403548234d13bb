"""Worker for tests/test_gpu_multi.py, launched by torchrun (one process per GPU, NCCL):
head-sharded causal prefill of one sequence (anelm_b200.parallel), the output all-gathered
to every rank by NCCL, and the same with the gather fused into the attention kernel (every
rank's epilogue storing its tiles into every rank's buffer over NVLink); rank 0 also runs the
full-head prefill on its GPU and saves all three (every rank checks its fused copy)."""
import os
import sys
from datetime import timedelta

import numpy as np
import torch
import torch.distributed as dist

sys.path.insert(0, os.path.join(os.path.dirname(os.path.abspath(__file__)), "..", "ane-lm_b200"))
import anelm_b200 as ab  # noqa: E402
from anelm_b200.core import Context  # noqa: E402
from anelm_b200.parallel import (PeerOutputs, fused_sharded_full_attn_prefill, local_proj_columns,  # noqa: E402
                                 sharded_full_attn_prefill)
from anelm_b200.shard import head_shard  # noqa: E402

HQ, HKV, D, R, N = 16, 4, 256, 64, 300


def main(out_path):
    rank, world = int(os.environ["RANK"]), int(os.environ["WORLD_SIZE"])
    local = int(os.environ.get("LOCAL_RANK", rank))
    torch.cuda.set_device(local)
    dist.init_process_group("nccl", timeout=timedelta(seconds=60))
    rng = np.random.default_rng(9)
    qn = (1 + 0.02 * rng.standard_normal(D)).astype(np.float32)
    kn = (1 + 0.02 * rng.standard_normal(D)).astype(np.float32)
    proj = torch.tensor(rng.standard_normal((N, HQ * 2 * D + 2 * HKV * D)), dtype=torch.float32)
    proj = proj.to(torch.bfloat16).to(f"cuda:{local}")
    qh, kvh = head_shard(HQ, HKV, world, rank)
    with Context(device=local, layer_types=[ab.LAYER_FULL_ATTN], num_q_heads=len(qh), num_kv_heads=len(kvh),
                 head_dim=D, rot_dim=R, rope_theta=1e7, max_seqs=1, kv_capacity=N) as ctx:
        ctx.set_full_attn_weights(0, qn, kn)
        plan = ctx.plan([0])
        out = sharded_full_attn_prefill(ctx, plan, 0, proj, HQ, HKV, D)
        torch.cuda.synchronize()
        # the fused form, twice (the second call reuses the mapped buffers), bf16 output
        peers = PeerOutputs((1, N, HQ * D), torch.bfloat16, torch.device("cuda", local))
        cols = local_proj_columns(HQ, HKV, D, qh, kvh).to(proj.device)
        lp = proj.index_select(1, cols).unsqueeze(0).contiguous()
        fused = []
        for _ in range(2):
            ctx.reset(0)
            fused.append(fused_sharded_full_attn_prefill(ctx, plan, 0, lp, peers, HQ, HKV, D).float().cpu().numpy())
            dist.barrier()
        peers.close()
        plan.close()
    with Context(device=local, layer_types=[ab.LAYER_FULL_ATTN], num_q_heads=HQ, num_kv_heads=HKV, head_dim=D,
                 rot_dim=R, rope_theta=1e7, max_seqs=1, kv_capacity=N) as ctx:
        ctx.set_full_attn_weights(0, qn, kn)
        plan = ctx.plan([0])
        full = ctx.full_attn_prefill(plan, 0, proj[None].contiguous())[0]
        ctx.reset(0)
        full16 = ctx.full_attn_prefill(plan, 0, proj[None].contiguous(), out_dtype=torch.bfloat16)
        torch.cuda.synchronize()
        plan.close()
    ok = all(np.array_equal(f, full16.float().cpu().numpy()) for f in fused)
    oks = torch.tensor([int(ok)], device=f"cuda:{local}")
    dist.all_reduce(oks)
    if rank == 0:
        np.savez(out_path, sharded=out.cpu().numpy(), full=full.cpu().numpy(), world=world,
                 fused_ok_ranks=int(oks.item()), fused=fused[-1][0], full16=full16.float().cpu().numpy()[0])
    dist.barrier()
    dist.destroy_process_group()


if __name__ == "__main__":
    main(sys.argv[1])

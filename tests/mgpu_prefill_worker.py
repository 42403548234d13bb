"""Worker for tests/test_gpu_multi.py, launched by torchrun (one process per GPU, NCCL):
head-sharded causal prefill of one sequence (anelm_b200.parallel), the output all-gathered
to every rank; rank 0 also runs the full-head prefill on its GPU and saves both."""
import os
import sys
from datetime import timedelta

import numpy as np
import torch
import torch.distributed as dist

sys.path.insert(0, os.path.join(os.path.dirname(os.path.abspath(__file__)), "..", "ane-lm_b200"))
import anelm_b200 as ab  # noqa: E402
from anelm_b200.core import Context  # noqa: E402
from anelm_b200.parallel import sharded_full_attn_prefill  # noqa: E402
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
        plan.close()
    if rank == 0:
        with Context(device=local, layer_types=[ab.LAYER_FULL_ATTN], num_q_heads=HQ, num_kv_heads=HKV, head_dim=D,
                     rot_dim=R, rope_theta=1e7, max_seqs=1, kv_capacity=N) as ctx:
            ctx.set_full_attn_weights(0, qn, kn)
            plan = ctx.plan([0])
            full = ctx.full_attn_prefill(plan, 0, proj[None].contiguous())[0]
            torch.cuda.synchronize()
            plan.close()
        np.savez(out_path, sharded=out.cpu().numpy(), full=full.cpu().numpy(), world=world)
    dist.barrier()
    dist.destroy_process_group()


if __name__ == "__main__":
    main(sys.argv[1])

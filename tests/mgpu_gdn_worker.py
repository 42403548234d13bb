"""Worker for tests/test_gpu_multi.py, launched by torchrun (one process per GPU, NCCL):
value-head-sharded chunked Gated DeltaNet prefill (anelm_b200.parallel) of the config-4 head
shape, outputs all-gathered to every rank; rank 0 also runs the unsharded call on its GPU
and saves both (outputs and every rank's state slice)."""
import os
import sys
from datetime import timedelta

import numpy as np
import torch
import torch.distributed as dist

sys.path.insert(0, os.path.join(os.path.dirname(os.path.abspath(__file__)), "..", "ane-lm_b200"))
from anelm_b200.core import gated_delta_chunked  # noqa: E402
from anelm_b200.parallel import sharded_gated_delta_chunked  # noqa: E402
from anelm_b200.shard import value_head_shard  # noqa: E402

B, T, HK, HV, D = 1, 200, 16, 32, 128


def main(out_path):
    rank, world = int(os.environ["RANK"]), int(os.environ["WORLD_SIZE"])
    local = int(os.environ.get("LOCAL_RANK", rank))
    torch.cuda.set_device(local)
    dist.init_process_group("nccl", timeout=timedelta(seconds=60))
    g = torch.Generator().manual_seed(4)
    unit = lambda x: x / x.norm(dim=-1, keepdim=True)  # noqa: E731
    q = (unit(torch.randn(B, T, HK, D, generator=g)) / D ** 0.5).to(torch.bfloat16)
    k = unit(torch.randn(B, T, HK, D, generator=g)).to(torch.bfloat16)
    v = torch.randn(B, T, HV, D, generator=g).to(torch.bfloat16)
    lg = -0.1 * torch.rand(B, T, HV, generator=g)
    bt = torch.rand(B, T, HV, generator=g)
    s0 = 0.1 * torch.randn(B, HV, D, D, generator=g)
    dev = f"cuda:{local}"
    q, k, v, lg, bt = (t.to(dev).contiguous() for t in (q, k, v, lg, bt))
    st = s0.to(dev).contiguous()
    y = sharded_gated_delta_chunked(q, k, v, lg, bt, st)
    torch.cuda.synchronize()
    _, vals = value_head_shard(HK, HV, world, rank)
    mine = st[:, vals[0]:vals[-1] + 1].contiguous()
    parts = [torch.empty_like(mine) for _ in range(world)]
    dist.all_gather(parts, mine)
    if rank == 0:
        st_full = s0.to(dev).contiguous()
        want = gated_delta_chunked(q, k, v, lg, bt, st_full)
        torch.cuda.synchronize()
        np.savez(out_path, sharded=y.cpu().numpy(), full=want.cpu().numpy(),
                 state_sharded=torch.cat(parts, dim=1).cpu().numpy(), state_full=st_full.cpu().numpy(), world=world)
    dist.barrier()
    dist.destroy_process_group()


if __name__ == "__main__":
    main(sys.argv[1])

"""Host logic of the multi-GPU paths, on CPU: sequence assignment for batched
decode (no collective), head-sharded attention prefill and value-head-sharded
chunked DeltaNet prefill with their one all-gather, run as world-size 2 and 4
gloo process groups (127.0.0.1)."""
import os
import socket

import numpy as np
import pytest
import torch
import torch.distributed as dist
import torch.multiprocessing as mp

from anelm_b200.parallel import local_proj_columns
from anelm_b200.shard import (assign_sequences, gather_heads, head_shard, max_over_ranks, seq_step_bytes,
                               value_head_shard)


def test_strong_assignment_is_a_balanced_partition():
    rng = np.random.default_rng(0)
    lengths = rng.integers(512, 32768, size=256, endpoint=True)
    costs = [seq_step_bytes(int(L), 8, 4, 256, 24, 32) for L in lengths]
    for world in (1, 2, 4, 8):
        parts = [assign_sequences(costs, world, r) for r in range(world)]
        flat = sorted(i for p in parts for i in p)
        assert flat == list(range(256))
        loads = [sum(costs[i] for i in p) for p in parts]
        assert max(loads) - min(loads) <= max(costs)
        assert max(loads) / (sum(costs) / world) < 1.01
    assert assign_sequences(costs, 4, 2, mode="weak") == list(range(256))


def test_head_shards_cover_every_head_once():
    for world in (1, 2, 4, 8):
        seen = []
        for r in range(world):
            q, kv = head_shard(16, 4, world, r)
            assert all(h // 4 in kv for h in q)
            seen += q
        assert sorted(seen) == list(range(16))


def _free_port():
    s = socket.socket()
    s.bind(("127.0.0.1", 0))
    p = s.getsockname()[1]
    s.close()
    return p


def _reference_attention(proj, Hq, Hkv, d):
    """Plain fp32 causal GQA attention with sigmoid gate (no norm / RoPE): the
    stand-in for the CUDA prefill in this host-logic test."""
    n = proj.shape[0]
    qg = proj[:, :Hq * 2 * d].view(n, Hq, 2 * d)
    q, gate = qg[..., :d], qg[..., d:]
    k = proj[:, Hq * 2 * d:Hq * 2 * d + Hkv * d].view(n, Hkv, d)
    v = proj[:, Hq * 2 * d + Hkv * d:].view(n, Hkv, d)
    G = Hq // Hkv
    out = torch.empty(n, Hq, d)
    mask = torch.ones(n, n, dtype=torch.bool).tril()
    for h in range(Hq):
        s = (q[:, h] @ k[:, h // G].T) / d ** 0.5
        out[:, h] = s.masked_fill(~mask, float("-inf")).softmax(-1) @ v[:, h // G]
    return (out * torch.sigmoid(gate)).reshape(n, Hq * d)


class _FakeCtx:
    """Host-only stand-in with the Context.full_attn_prefill signature."""

    def __init__(self, Hq, Hkv, d):
        self.Hq, self.Hkv, self.d = Hq, Hkv, d

    def full_attn_prefill(self, plan, layer, proj, start_pos, out_dtype=torch.float32):
        return _reference_attention(proj[0], self.Hq, self.Hkv, self.d)[None].to(out_dtype)


def _worker(rank, world, port, Hq, Hkv, d, n, q):
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
    dist.init_process_group("gloo", rank=rank, world_size=world)
    try:
        from anelm_b200.parallel import sharded_full_attn_prefill
        g = torch.Generator().manual_seed(0)
        proj = torch.randn(n, Hq * 2 * d + 2 * Hkv * d, generator=g)
        qh, kvh = head_shard(Hq, Hkv, world, rank)
        out = sharded_full_attn_prefill(_FakeCtx(len(qh), len(kvh), d), None, 0, proj, Hq, Hkv, d)
        want = _reference_attention(proj, Hq, Hkv, d)
        err = float((out - want).abs().max())
        t = max_over_ranks(float(rank))
        q.put((rank, err, t, tuple(out.shape)))
    finally:
        dist.destroy_process_group()


@pytest.mark.parametrize("world", [2, 4])
def test_head_sharded_prefill_gloo(world):
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=_worker, args=(r, world, port, 8, 2 if world == 2 else 4, 16, 24, q))
             for r in range(world)]
    for p in procs:
        p.start()
    res = [q.get(timeout=120) for _ in procs]
    for p in procs:
        p.join(timeout=60)
        assert p.exitcode == 0
    for rank, err, t, shape in res:
        assert err < 1e-5, (rank, err)
        assert t == world - 1
        assert shape == (24, 8 * 16)


def test_local_proj_columns_order():
    cols = local_proj_columns(4, 2, 2, [2, 3], [1]).tolist()
    # q_gate of heads 2, 3 (4 columns each), then k of kv head 1, then v of kv head 1
    assert cols == list(range(8, 16)) + [18, 19] + [22, 23]


def test_value_head_shards_cover_every_head_once():
    for Hk, Hv in ((16, 32), (16, 16), (2, 8)):
        ratio = Hv // Hk
        for world in (1, 2, 4, 8, 16):
            if Hv % world:
                continue
            seen = []
            for r in range(world):
                keys, vals = value_head_shard(Hk, Hv, world, r)
                assert keys == sorted({h // ratio for h in vals})
                assert vals == list(range(vals[0], vals[-1] + 1))
                seen += vals
            assert sorted(seen) == list(range(Hv))
    with pytest.raises(ValueError):
        value_head_shard(16, 32, 3, 0)


def _delta_rule_reference(q, k, v, log_decay, beta, state, delta_mode=0, y_dtype=torch.float32):
    """Host stand-in with the gated_delta_chunked signature: the token recurrence of
    cpu_ops.cpp:131-146 (Sk from the undecayed state), state updated in place."""
    B, T, Hk, _ = q.shape
    Hv = v.shape[2]
    ratio = Hv // Hk
    y = torch.empty(B, T, Hv, v.shape[3], dtype=torch.float64)
    for b in range(B):
        for h in range(Hv):
            S = state[b, h].double()
            for t in range(T):
                kk, qq, vv = k[b, t, h // ratio].double(), q[b, t, h // ratio].double(), v[b, t, h].double()
                d = vv - S.T @ kk
                S = torch.exp(log_decay[b, t, h].double()) * S + beta[b, t, h].double() * torch.outer(kk, d)
                y[b, t, h] = S.T @ qq
            state[b, h] = S.float()
    return y.to(y_dtype)


def _gdn_worker(rank, world, port, q):
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
    dist.init_process_group("gloo", rank=rank, world_size=world)
    try:
        import anelm_b200.core as core
        core.gated_delta_chunked = _delta_rule_reference
        from anelm_b200.parallel import sharded_gated_delta_chunked
        g = torch.Generator().manual_seed(1)
        B, T, Hk, Hv, d = 1, 5, 2, 8, 4
        qq = torch.randn(B, T, Hk, d, generator=g)
        kk = torch.randn(B, T, Hk, d, generator=g)
        vv = torch.randn(B, T, Hv, d, generator=g)
        lg = -0.1 * torch.rand(B, T, Hv, generator=g)
        bt = torch.rand(B, T, Hv, generator=g)
        s0 = torch.randn(B, Hv, d, d, generator=g)
        st = s0.clone()
        y = sharded_gated_delta_chunked(qq, kk, vv, lg, bt, st)
        st_full = s0.clone()
        want = _delta_rule_reference(qq, kk, vv, lg, bt, st_full)
        _, vals = value_head_shard(Hk, Hv, world, rank)
        q.put((rank, bool(torch.equal(y, want)), bool(torch.equal(st[:, vals], st_full[:, vals])),
               bool(torch.equal(st[:, [h for h in range(Hv) if h not in vals]],
                                s0[:, [h for h in range(Hv) if h not in vals]]))))
    finally:
        dist.destroy_process_group()


@pytest.mark.parametrize("world", [2, 4])
def test_value_head_sharded_delta_rule_gloo(world):
    """Outputs all-gathered in head order; each rank's heads' state updated, the others untouched."""
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=_gdn_worker, args=(r, world, port, q)) for r in range(world)]
    for p in procs:
        p.start()
    res = [q.get(timeout=120) for _ in procs]
    for p in procs:
        p.join(timeout=60)
        assert p.exitcode == 0
    for rank, y_ok, own_ok, other_ok in res:
        assert y_ok and own_ok and other_ok, rank

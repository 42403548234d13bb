"""GPU parity of the causal prefill (tcgen05 attention) through the C ABI.

Small sizes: against the CPU oracle's per-token loop (the reference's
forward_full_attn_from_proj, qwen3_5.cpp:944-1002, called once per prompt token
as in qwen3_5.cpp:1205-1217), including padding rows and a decode step after the
prefill.  BASELINE config 3 size (4096 tokens, 16/4 heads, d=256): against a
plain PyTorch fp32 restatement of the same math.  Tolerance 2e-3 abs + 1e-2 rel."""
import numpy as np
import pytest

torch = pytest.importorskip("torch")

import anelm_b200 as ab  # noqa: E402
from anelm_b200.core import Context  # noqa: E402
from helpers import assert_close, fa_shape  # noqa: E402
from oracle import pyoracle as po  # noqa: E402

pytestmark = pytest.mark.gpu

HQ, HKV, D, R = 16, 4, 256, 64
PROJ = HQ * 2 * D + 2 * HKV * D


def ctx_for(n_seqs, cap, **kw):
    return Context(layer_types=[ab.LAYER_FULL_ATTN], num_q_heads=HQ, num_kv_heads=HKV, head_dim=D, rot_dim=R,
                   rope_theta=1e7, max_seqs=n_seqs, kv_capacity=cap, **kw)


def bf16_proj(gen, B, n):
    return torch.randn(B, n, PROJ, generator=gen, device="cuda").to(torch.bfloat16)


def weights(rng):
    return ((1 + 0.02 * rng.standard_normal(D)).astype(np.float32),
            (1 + 0.02 * rng.standard_normal(D)).astype(np.float32))


def torch_reference(proj, qn, kn, start_pos, rope):
    """fp32 restatement: per-head RMSNorm (cpu_ops.cpp:24-30), interleaved RoPE
    (cpu_ops.cpp:40-63), causal GQA softmax attention (cpu_ops.cpp:148-204),
    sigmoid gate (cpu_ops.cpp:15-22)."""
    B, n, _ = proj.shape
    x = proj.float()
    qg = x[..., :HQ * 2 * D].reshape(B, n, HQ, 2 * D)
    q, gate = qg[..., :D], qg[..., D:]
    k = x[..., HQ * 2 * D:HQ * 2 * D + HKV * D].reshape(B, n, HKV, D)
    v = x[..., HQ * 2 * D + HKV * D:].reshape(B, n, HKV, D)
    qn_t, kn_t = torch.tensor(qn, device="cuda"), torch.tensor(kn, device="cuda")
    q = q * torch.rsqrt(q.pow(2).mean(-1, keepdim=True) + 1e-6) * qn_t
    k = k * torch.rsqrt(k.pow(2).mean(-1, keepdim=True) + 1e-6) * kn_t
    cos = torch.tensor(rope[0][start_pos:start_pos + n], device="cuda")[None, :, None, :]
    sin = torch.tensor(rope[1][start_pos:start_pos + n], device="cuda")[None, :, None, :]

    def rot(t):
        t = t.clone()
        a, b = t[..., 0:R:2].clone(), t[..., 1:R:2].clone()
        t[..., 0:R:2] = a * cos - b * sin
        t[..., 1:R:2] = a * sin + b * cos
        return t

    q, k = rot(q), rot(k)
    out = torch.empty(B, n, HQ, D, device="cuda")
    mask = torch.ones(n, n, device="cuda", dtype=torch.bool).tril()
    G = HQ // HKV
    for b in range(B):
        for g in range(HKV):
            qq = q[b, :, g * G:(g + 1) * G].permute(1, 0, 2)           # [G][n][D]
            s = (qq @ k[b, :, g].T[None]) / (D ** 0.5)                  # [G][n][n]
            s = s.masked_fill(~mask, float("-inf"))
            out[b, :, g * G:(g + 1) * G] = (s.softmax(-1) @ v[b, :, g][None]).permute(1, 0, 2)
    out = out / (1 + torch.exp(-gate))
    return out.reshape(B, n, HQ * D)


@pytest.mark.parametrize("out_dtype", ["float32", "bfloat16", "float16"])
def test_prefill_matches_oracle_with_padding_and_decode_after(out_dtype):
    """fp32 output takes the row-store epilogue; 16-bit outputs take the TMA tile store, whose rows past
    each sequence's end (200 of a 256-row tile) must not spill into the next sequence's rows."""
    rng = np.random.default_rng(5)
    gen = torch.Generator(device="cuda")
    gen.manual_seed(5)
    B, n, cap = 2, 200, 256
    qn, kn = weights(rng)
    proj = bf16_proj(gen, B, n)
    rope = po.rope_table(4096, R, 1e7)
    shape = fa_shape(HQ, HKV, D, R, 1e7)
    with ctx_for(B, cap) as ctx:
        ctx.set_full_attn_weights(0, qn, kn)
        plan = ctx.plan([1, 0])
        out = ctx.full_attn_prefill(plan, 0, proj, start_pos=0, out_dtype=getattr(torch, out_dtype))
        out = out.float().cpu().numpy()
        # one more decode token for sequence 1 (row 0 of the plan)
        nxt = torch.randn(PROJ, generator=gen, device="cuda").to(torch.bfloat16)
        dec = ctx.full_attn_from_proj(0, 1, nxt, n).cpu().numpy()
        exported = [ctx.kv_export(0, s) for s in (1, 0)]
        plan.close()
    p32 = proj.float().cpu().numpy()
    for i in range(B):
        ring = po.KVRing.empty(cap, HKV, D)
        want = po.full_attn_tokens("oracle", shape, po.make_variant(kv_round_f16=1), qn, kn, ring, p32[i], 0, rope)
        assert_close(out[i], want, what=f"prefill row {i}")
        if i == 0:  # plan row 0 (sequence 1) got one more decode token
            want_dec = po.full_attn_tokens("oracle", shape, po.make_variant(kv_round_f16=1), qn, kn, ring,
                                           nxt.float().cpu().numpy()[None], n, rope)
            assert_close(dec, want_dec[0], what="decode after prefill")
        k, v, ln, st = exported[i]
        assert (ln, st) == (ring.len, ring.start) == (n + (i == 0), 0)
        np.testing.assert_array_equal(v[:ring.len], ring.v[:ring.len])
        assert_close(k[:ring.len], ring.k[:ring.len], atol=2e-3, rtol=2e-3, what="K ring after prefill")


@pytest.mark.parametrize("n,out_dtype", [(520, "float32"), (700, "bfloat16"), (256, "float16")])
def test_prefill_ragged_query_tiles(n, out_dtype):
    """Several 128-row query tiles per head with a ragged last one: n = 520 leaves the last tile 8
    rows, n = 700 leaves it 60, n = 256 fills two tiles exactly; tiles are dispatched longest first
    across heads and sequences (B = 2).  Row-store (fp32) and TMA tile-store (16-bit) epilogues,
    against the fp32 PyTorch restatement."""
    gen = torch.Generator(device="cuda")
    gen.manual_seed(n)
    rng = np.random.default_rng(n)
    B = 2
    qn, kn = weights(rng)
    proj = bf16_proj(gen, B, n)
    rope = po.rope_table(4096, R, 1e7)
    with ctx_for(B, n) as ctx:
        ctx.set_full_attn_weights(0, qn, kn)
        plan = ctx.plan([0, 1])
        out = ctx.full_attn_prefill(plan, 0, proj, start_pos=0, out_dtype=getattr(torch, out_dtype))
        torch.cuda.synchronize()
        plan.close()
    want = torch_reference(proj, qn, kn, 0, rope)
    assert_close(out.float().cpu().numpy(), want.cpu().numpy(), what=f"prefill n={n}")


@pytest.mark.parametrize("B,out_dtype", [(1, "float32"), (8, "bfloat16")])
def test_prefill_config3_full_size(B, out_dtype):
    """Qwen3.5-4B shape, seq 4096, bf16 inputs N(0,1)."""
    rng = np.random.default_rng(3)
    gen = torch.Generator(device="cuda")
    gen.manual_seed(3 + B)
    n = 4096
    qn, kn = weights(rng)
    proj = bf16_proj(gen, B, n)
    rope = po.rope_table(4096, R, 1e7)
    with ctx_for(B, n) as ctx:
        ctx.set_full_attn_weights(0, qn, kn)
        plan = ctx.plan(list(range(B)))
        out = ctx.full_attn_prefill(plan, 0, proj, start_pos=0, out_dtype=getattr(torch, out_dtype))
        torch.cuda.synchronize()
        assert ctx.device_error() == 0
        plan.close()
    check = [0, B - 1] if B > 1 else [0]
    want = torch_reference(proj[check], qn, kn, 0, rope)
    assert_close(out[check].float().cpu().numpy(), want.cpu().numpy(), what=f"config-3 prefill B={B}")


def test_prefill_state_errors():
    with ctx_for(1, 64, qk_norm_in_core=0) as ctx:
        plan = ctx.plan([0])
        p = torch.zeros(1, 65, PROJ, device="cuda")
        with pytest.raises(ab.AnelmError) as e:
            ctx.full_attn_prefill(plan, 0, p)        # more tokens than the ring holds
        assert e.value.status == 2
        ctx.full_attn_prefill(plan, 0, p[:, :10].contiguous())
        with pytest.raises(ab.AnelmError) as e:
            ctx.full_attn_prefill(plan, 0, p[:, :10].contiguous())   # ring is no longer empty
        assert e.value.status == 6
        ctx.reset(0)
        ctx.full_attn_prefill(plan, 0, p[:, :10].contiguous())
        torch.cuda.synchronize()
        plan.close()


@pytest.mark.parametrize("case", ["rope_half_f32_proj", "rope_half_bf16_proj", "rot40_fallback_prep",
                                  "past_table_bf16_proj"])
def test_prefill_prep_variants(case):
    """The projection prep (RMSNorm, RoPE, fp16 Q/K/V, ring append) has a streaming path (16-bit
    projection rows staged by bulk copies), a vectorised one (16-byte rows, rot_dim % 16 == 0) and a
    general one: rotate-half RoPE on a bf16 projection exercises the streaming kernel's lane-pair
    shuffle, on an fp32 projection the vectorised kernel's, rot_dim 40 the general kernel; positions
    4000-4149 cross the end of the 4096-row RoPE table (computed angles past it, cpu_ops.cpp:51-56).
    All against the oracle."""
    rng = np.random.default_rng(11)
    gen = torch.Generator(device="cuda")
    gen.manual_seed(11)
    n, cap = 150, 160
    half = case.startswith("rope_half")
    rot = 64 if half else 40
    qn, kn = weights(rng)
    proj = torch.randn(1, n, PROJ, generator=gen, device="cuda")
    if not case.endswith("f32_proj"):
        proj = proj.to(torch.bfloat16)
    rope = po.rope_table(4096, rot, 1e7)
    shape = fa_shape(HQ, HKV, D, rot, 1e7)
    variant = po.make_variant(rope_half=int(half), kv_round_f16=1)
    start = 4000 if case.startswith("past_table") else 0
    with Context(layer_types=[ab.LAYER_FULL_ATTN], num_q_heads=HQ, num_kv_heads=HKV, head_dim=D, rot_dim=rot,
                 rope_theta=1e7, max_seqs=1, kv_capacity=cap,
                 rope_mode=ab.ROPE_HALF if half else ab.ROPE_INTERLEAVED) as ctx:
        ctx.set_full_attn_weights(0, qn, kn)
        plan = ctx.plan([0])
        out = ctx.full_attn_prefill(plan, 0, proj, start_pos=start, out_dtype=torch.float16).float().cpu().numpy()
        k, v, ln, st = ctx.kv_export(0, 0)
        plan.close()
    ring = po.KVRing.empty(cap, HKV, D)
    want = po.full_attn_tokens("oracle", shape, variant, qn, kn, ring, proj.float().cpu().numpy()[0], start, rope)
    assert_close(out[0], want, what=f"prefill {case}")
    assert (ln, st) == (n, 0)
    np.testing.assert_array_equal(v[:n], ring.v[:n])
    assert_close(k[:n], ring.k[:n], atol=2e-3, rtol=2e-3, what=f"K ring {case}")


@pytest.mark.parametrize("hq,hkv", [(8, 2), (6, 2), (4, 1)])
def test_prefill_other_head_counts(hq, hkv):
    """Head counts other than the 4B shape's: 8/2 (the 0.8B shape; q and gate segments interleaved
    across the prep's warps), 6/2 and 4/1 (head counts that are not a multiple of 8 keep the
    prep's segment order), bf16 projections through the streaming prep, against the oracle."""
    rng = np.random.default_rng(40 + hq)
    gen = torch.Generator(device="cuda")
    gen.manual_seed(40 + hq)
    n, cap = 140, 160
    qn, kn = weights(rng)
    proj = torch.randn(1, n, hq * 2 * D + 2 * hkv * D, generator=gen, device="cuda").to(torch.bfloat16)
    rope = po.rope_table(4096, R, 1e7)
    shape = fa_shape(hq, hkv, D, R, 1e7)
    with Context(layer_types=[ab.LAYER_FULL_ATTN], num_q_heads=hq, num_kv_heads=hkv, head_dim=D, rot_dim=R,
                 rope_theta=1e7, max_seqs=1, kv_capacity=cap) as ctx:
        ctx.set_full_attn_weights(0, qn, kn)
        plan = ctx.plan([0])
        out = ctx.full_attn_prefill(plan, 0, proj, out_dtype=torch.bfloat16).float().cpu().numpy()
        k, v, ln, st = ctx.kv_export(0, 0)
        plan.close()
    ring = po.KVRing.empty(cap, hkv, D)
    want = po.full_attn_tokens("oracle", shape, po.make_variant(kv_round_f16=1), qn, kn, ring,
                               proj.float().cpu().numpy()[0], 0, rope)
    assert_close(out[0], want, what=f"prefill {hq}/{hkv} heads")
    assert (ln, st) == (n, 0)
    np.testing.assert_array_equal(v[:n], ring.v[:n])
    assert_close(k[:n], ring.k[:n], atol=2e-3, rtol=2e-3, what=f"K ring {hq}/{hkv} heads")

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
from helpers import assert_close, f16, fa_shape  # noqa: E402
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


def test_prefill_linear_cache_errors():
    """A linear cache (slot = position, serve_hybrid.py:105-108) is filled from position 0 of an
    empty cache and never slides: longer prompts, later starts and second prefills are errors."""
    with ctx_for(1, 64, qk_norm_in_core=0, kv_mode=ab.KV_LINEAR) as ctx:
        plan = ctx.plan([0])
        p = torch.zeros(1, 65, PROJ, device="cuda")
        with pytest.raises(ab.AnelmError) as e:
            ctx.full_attn_prefill(plan, 0, p)        # more tokens than the cache has positions
        assert e.value.status == 2
        with pytest.raises(ab.AnelmError) as e:
            ctx.full_attn_prefill(plan, 0, p[:, :10].contiguous(), start_pos=10)
        assert e.value.status == 5
        ctx.full_attn_prefill(plan, 0, p[:, :10].contiguous())
        with pytest.raises(ab.AnelmError) as e:
            ctx.full_attn_prefill(plan, 0, p[:, :10].contiguous())   # the cache is no longer empty
        assert e.value.status == 2
        ctx.reset(0)
        ctx.full_attn_prefill(plan, 0, p[:, :10].contiguous())
        torch.cuda.synchronize()
        assert ctx.device_error() == 0
        plan.close()


def generate_chunks(n):
    """Chunk sizes of generate.cpp:57-73: the largest of 8 / 4 / 2 / 1 that fits what remains."""
    out = []
    while n > 0:
        c = next(b for b in (8, 4, 2, 1) if b <= n)
        out.append(c)
        n -= c
    return out


def test_prefill_continues_rings_in_generate_chunks():
    """Prefill on top of existing KV: generate.cpp:57-73 feeds the prompt to forward_batch in
    chunks of 8 / 4 / 2 / 1 at a running start_pos (qwen3_5.cpp:1164-1217), each chunk attending
    to every earlier token still in the ring.  Two sequences (rings of 512 and 200 slots) start
    from prompts of 100 and 37 tokens, continue together in one plan through 45 tokens of such
    chunks (their old-token prefixes differ), decode 3 tokens, then take a 150-token second turn
    that overflows the 200-slot ring mid-call (it slides: its oldest tokens leave the window of
    later queries) and a last 8-token chunk over a wrapped ring.  Everything against the
    oracle's per-token loop over the same positions; ring len / start and V bit-exact."""
    rng = np.random.default_rng(77)
    gen = torch.Generator(device="cuda")
    gen.manual_seed(77)
    caps = [512, 200]
    qn, kn = weights(rng)
    rope = po.rope_table(4096, R, 1e7)
    shape = fa_shape(HQ, HKV, D, R, 1e7)
    var = po.make_variant(kv_round_f16=1)
    rings = [po.KVRing.empty(c, HKV, D) for c in caps]
    got = [[], []]
    want = [[], []]

    def oracle(s, proj, pos):
        want[s].append(po.full_attn_tokens("oracle", shape, var, qn, kn, rings[s], proj.float().cpu().numpy(),
                                           pos, rope))

    with Context(layer_types=[ab.LAYER_FULL_ATTN], num_q_heads=HQ, num_kv_heads=HKV, head_dim=D, rot_dim=R,
                 rope_theta=1e7, seq_kv_capacity=caps) as ctx:
        ctx.set_full_attn_weights(0, qn, kn)
        plans = [ctx.plan([0]), ctx.plan([1]), ctx.plan([0, 1])]
        # first prompts, one sequence each
        for s, n in ((0, 100), (1, 37)):
            p = bf16_proj(gen, 1, n)
            got[s].append(ctx.full_attn_prefill(plans[s], 0, p, start_pos=0)[0].cpu().numpy())
            oracle(s, p[0], 0)
        # both sequences continue in generate.cpp's chunks (one start position for the plan)
        pos = 200
        for c in generate_chunks(45):
            p = bf16_proj(gen, 2, c)
            out = ctx.full_attn_prefill(plans[2], 0, p, start_pos=pos).cpu().numpy()
            for s in (0, 1):
                got[s].append(out[s])
                oracle(s, p[s], pos)
            pos += c
        # decode
        for _ in range(3):
            p = bf16_proj(gen, 2, 1)[:, 0].contiguous()
            out = ctx.full_attn_decode(plans[2], 0, p, torch.tensor([pos, pos], dtype=torch.int32,
                                                                     device="cuda")).cpu().numpy()
            for s in (0, 1):
                got[s].append(out[s:s + 1])
                oracle(s, p[s:s + 1], pos)
            pos += 1
        # second turn: 150 tokens (sequence 1's ring overflows), then 8 more over a wrapped ring
        for n in (150, 8):
            p = bf16_proj(gen, 2, n)
            out = ctx.full_attn_prefill(plans[2], 0, p, start_pos=pos).cpu().numpy()
            for s in (0, 1):
                got[s].append(out[s])
                oracle(s, p[s], pos)
            pos += n
        torch.cuda.synchronize()
        assert ctx.device_error() == 0
        exported = [ctx.kv_export(0, s) for s in (0, 1)]
        for pl in plans:
            pl.close()
    assert rings[1].start != 0 and rings[1].len == caps[1]  # the small ring slid and wrapped
    for s in (0, 1):
        assert_close(np.concatenate(got[s]), np.concatenate(want[s]), what=f"sequence {s}")
        k, v, ln, st = exported[s]
        assert (ln, st) == (rings[s].len, rings[s].start), f"sequence {s} ring metadata"
        np.testing.assert_array_equal(v, rings[s].v)
        assert_close(k, rings[s].k, atol=2e-3, rtol=2e-3, what=f"sequence {s} K ring")


@pytest.mark.parametrize("n,cap,start_len", [(3000, 2048, 0), (700, 300, 250)])
def test_prefill_longer_than_ring(n, cap, start_len):
    """A prompt longer than the ring: the reference's ring slides once full (qwen3_5.cpp:974-983),
    so token t sees only the last `cap` tokens and the ring ends holding the last `cap` of the
    prompt with start = (old start + overflow) mod cap.  3,000 tokens into the reference's
    2,048-slot ring (0.8B shape, fresh ring), and 700 tokens into a 300-slot ring that already
    holds 250 (wrapped at slot 123).  Against the oracle's per-token loop; metadata and V exact."""
    hq, hkv = 8, 2
    rng = np.random.default_rng(n)
    gen = torch.Generator(device="cuda")
    gen.manual_seed(n)
    qn, kn = weights(rng)
    rope = po.rope_table(4096, R, 1e7)
    shape = fa_shape(hq, hkv, D, R, 1e7)
    ring = po.KVRing.empty(cap, hkv, D)
    if start_len:
        ring.k[:] = f16(rng.standard_normal(ring.k.shape))
        ring.v[:] = f16(rng.standard_normal(ring.v.shape))
        ring.len, ring.start = start_len, 123
    proj = torch.randn(1, n, hq * 2 * D + 2 * hkv * D, generator=gen, device="cuda").to(torch.bfloat16)
    with Context(layer_types=[ab.LAYER_FULL_ATTN], num_q_heads=hq, num_kv_heads=hkv, head_dim=D, rot_dim=R,
                 rope_theta=1e7, max_seqs=1, kv_capacity=cap) as ctx:
        ctx.set_full_attn_weights(0, qn, kn)
        if start_len:
            ctx.kv_import(0, 0, ring.k, ring.v, ring.len, ring.start)
        plan = ctx.plan([0])
        out = ctx.full_attn_prefill(plan, 0, proj, start_pos=start_len).cpu().numpy()[0]
        assert ctx.device_error() == 0
        k, v, ln, st = ctx.kv_export(0, 0)
        plan.close()
    want = po.full_attn_tokens("oracle", shape, po.make_variant(kv_round_f16=1), qn, kn, ring,
                               proj.float().cpu().numpy()[0], start_len, rope)
    assert_close(out, want, what=f"{n} tokens into a {cap}-slot ring")
    assert (ln, st) == (ring.len, ring.start) == (cap, (123 * bool(start_len) + start_len + n - cap) % cap)
    np.testing.assert_array_equal(v, ring.v)
    assert_close(k, ring.k, atol=2e-3, rtol=2e-3, what="K ring")


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

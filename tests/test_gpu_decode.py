"""GPU parity of the fused decode kernels against the CPU oracle and the golden
fixtures made from the reference (tolerance: 2e-3 abs / 1e-2 rel, fp32
accumulation from fp16 inputs; ring/conv indexing bit-exact).  Every call goes
through the C ABI of libanelm_b200.so via the ctypes host mirror."""
import numpy as np
import pytest

torch = pytest.importorskip("torch")

import anelm_b200 as ab  # noqa: E402
from anelm_b200.core import Context  # noqa: E402
from helpers import (assert_close, f16, fa_inputs, fa_shape, gdn_inputs, gdn_shape,  # noqa: E402
                     random_ring)
from oracle import pyoracle as po  # noqa: E402

pytestmark = pytest.mark.gpu


def fa_ctx(shape, cap=None, caps=None, max_seqs=1, **kw):
    extra = dict(kv_capacity=cap) if cap else {}
    return Context(layer_types=[ab.LAYER_FULL_ATTN], num_q_heads=shape.num_q_heads,
                   num_kv_heads=shape.num_kv_heads, head_dim=shape.head_dim, rot_dim=shape.rot_dim,
                   rope_theta=shape.rope_theta, max_seqs=max_seqs, seq_kv_capacity=caps, **extra, **kw)


def gdn_ctx(shape, max_seqs=1, **kw):
    return Context(layer_types=[ab.LAYER_LINEAR_ATTN], lin_num_key_heads=shape.lin_num_key_heads,
                   lin_num_val_heads=shape.lin_num_val_heads, max_seqs=max_seqs, **kw)


def dev(a, dtype=torch.float32):
    return torch.from_numpy(np.ascontiguousarray(a)).to(device="cuda", dtype=dtype)


# ---------------------------------------------------------------- golden fixtures

@pytest.mark.parametrize("proj_dtype,out_dtype", [(torch.float32, torch.float32), (torch.float16, torch.float16)])
def test_full_attn_matches_reference_golden(golden, proj_dtype, out_dtype):
    g = golden("full_attn_ref.npz")
    shape = fa_shape()
    T, cap, p0 = g["proj"].shape[0], int(g["cap"]), int(g["start_pos"])
    with fa_ctx(shape, cap=cap) as ctx:
        ctx.set_full_attn_weights(0, g["q_norm"], g["k_norm"])
        proj = dev(g["proj"].astype(np.float32), proj_dtype)
        out = torch.stack([ctx.full_attn_from_proj(0, 0, proj[t].contiguous(), p0 + t, out_dtype=out_dtype)
                           for t in range(T)])
        got = out.float().cpu().numpy()
        k, v, ln, st = ctx.kv_export(0, 0)
    assert_close(got, g["out_f16kv"], what="attention output vs reference (fp16 KV)")
    # the ring layout: same tokens in the same slots, same len/start (bit-exact indexing)
    assert (ln, st) == (int(g["len"]), int(g["start"]))
    assert_close(k, g["k_cache_f16kv"], atol=2e-3, rtol=2e-3, what="K ring")
    np.testing.assert_array_equal(v, g["v_cache_f16kv"])  # V is copied, so it is exact


def test_deltanet_matches_reference_golden(golden):
    g = golden("deltanet_ref.npz")
    Hv, dk = g["ssm0"].shape[:2]
    Hk = (g["conv0"].shape[0] - Hv * dk) // (2 * dk)
    shape = gdn_shape(Hk=Hk, Hv=Hv)
    with gdn_ctx(shape) as ctx:
        ctx.set_deltanet_weights(0, g["conv_w"], g["A"], g["dt_bias"], g["norm_w"])
        ctx.deltanet_state_import(0, 0, g["ssm0"], g["conv0"], int(g["conv_pos0"]))
        proj = dev(g["proj"].astype(np.float32))
        got = torch.stack([ctx.deltanet_from_proj(0, 0, proj[t].contiguous()) for t in range(proj.shape[0])])
        got = got.cpu().numpy()
        ssm, conv, pos = ctx.deltanet_state_export(0, 0)
    assert_close(got, g["out"], what="DeltaNet output vs reference")
    assert_close(ssm, g["ssm"], what="DeltaNet state vs reference")
    np.testing.assert_array_equal(conv, g["conv"])
    assert pos == int(g["conv_pos"])


# ---------------------------------------------------------------- BASELINE config 1 / 2 shapes

@pytest.mark.parametrize("length,start", [(2048, 700), (2047, 1500), (5, 0), (1, 2047)])
def test_full_attn_config1_ring(length, start):
    """0.8B shape, KV ring of 2048: full + wrapped, nearly full across the edge, short."""
    rng = np.random.default_rng(length + start)
    shape = fa_shape(8, 2, 256, 64, 1e7)
    cap, T = 2048, 6
    proj, qn, kn = fa_inputs(rng, shape, T)
    ring = random_ring(rng, cap, 2, 256, length, start)
    rope = po.rope_table(4096, 64, 1e7)
    with fa_ctx(shape, cap=cap) as ctx:
        ctx.set_full_attn_weights(0, qn, kn)
        ctx.kv_import(0, 0, ring.k, ring.v, ring.len, ring.start)
        p = dev(proj, torch.float16)
        got = torch.stack([ctx.full_attn_from_proj(0, 0, p[t].contiguous(), 3000 + t) for t in range(T)])
        got = got.cpu().numpy()
        k, v, ln, st = ctx.kv_export(0, 0)
    want = po.full_attn_tokens("oracle", shape, po.make_variant(kv_round_f16=1), qn, kn, ring, proj, 3000, rope)
    assert_close(got, want, what="config-1 decode")
    assert (ln, st) == (ring.len, ring.start)
    assert_close(k, ring.k, atol=2e-3, rtol=2e-3, what="K ring")
    np.testing.assert_array_equal(v, ring.v)


@pytest.mark.parametrize("Hq,Hkv,d,cap", [(8, 2, 256, 100), (8, 2, 256, 160), (8, 2, 256, 300),
                                           (16, 4, 256, 500), (4, 4, 128, 900), (6, 2, 128, 2048),
                                           (2, 2, 256, 1500)])
def test_full_attn_one_row_cluster_merge(Hq, Hkv, d, cap):
    """One-row plans merge their splits inside a thread-block cluster: each split pushes every owner
    CTA its slice of the G * d / 4 output float4s and its (m, l).  Ring capacities giving 2, 3, 5, 8,
    15 and 16 splits (the last owner's slice shorter than the others at most of them), G = 4, 1, 3 and
    1 query heads per kv head, head_dim 256 and 128; full and partly filled rings, against the oracle."""
    rng = np.random.default_rng(cap + Hq)
    shape = fa_shape(Hq, Hkv, d, 64, 1e7)
    T = 3
    proj, qn, kn = fa_inputs(rng, shape, T)
    length = cap if cap % 2 == 0 else cap - 7
    ring = random_ring(rng, cap, Hkv, d, length, cap // 3)
    rope = po.rope_table(4096, 64, 1e7)
    with fa_ctx(shape, cap=cap) as ctx:
        ctx.set_full_attn_weights(0, qn, kn)
        ctx.kv_import(0, 0, ring.k, ring.v, ring.len, ring.start)
        p = dev(proj, torch.float16)
        got = torch.stack([ctx.full_attn_from_proj(0, 0, p[t].contiguous(), 900 + t) for t in range(T)])
        got = got.cpu().numpy()
        assert ctx.device_error() == 0
        k, v, ln, st = ctx.kv_export(0, 0)
    want = po.full_attn_tokens("oracle", shape, po.make_variant(kv_round_f16=1), qn, kn, ring, proj, 900, rope)
    assert_close(got, want, what=f"one-row decode, {Hq}/{Hkv} heads, d {d}, ring {cap}")
    assert (ln, st) == (ring.len, ring.start)
    np.testing.assert_array_equal(v, ring.v)


@pytest.mark.parametrize("Hk,Hv,T", [(16, 16, 64), (16, 32, 24)])
def test_deltanet_successive_tokens(Hk, Hv, T):
    """Config-2 (16/16 heads) and the 4B GQA shape (32 value / 16 key heads):
    successive tokens from a random state N(0, 0.1)."""
    rng = np.random.default_rng(Hv * 1000 + T)
    shape = gdn_shape(Hk=Hk, Hv=Hv)
    proj, conv_w, A, dt_bias, norm_w = gdn_inputs(rng, shape, T)
    C = conv_w.shape[0]
    st = po.DeltaState((0.1 * rng.standard_normal((Hv, 128, 128))).astype(np.float32),
                       rng.standard_normal((C, 3)).astype(np.float32), 2)
    with gdn_ctx(shape) as ctx:
        ctx.set_deltanet_weights(0, conv_w, A, dt_bias, norm_w)
        ctx.deltanet_state_import(0, 0, st.ssm, st.conv, st.conv_pos)
        p = dev(proj, torch.float16)
        got = torch.stack([ctx.deltanet_from_proj(0, 0, p[t].contiguous()) for t in range(T)]).cpu().numpy()
        ssm, conv, pos = ctx.deltanet_state_export(0, 0)
    want = po.deltanet_tokens("oracle", shape, po.make_variant(), conv_w, A, dt_bias, norm_w, st, proj)
    assert_close(got, want, what="DeltaNet outputs")
    assert_close(ssm, st.ssm, what="DeltaNet state")
    np.testing.assert_array_equal(conv, st.conv)
    assert pos == st.conv_pos


def test_deltanet_long_run_state_stays_close():
    """BASELINE config 2 over its full length: 4096 successive tokens through one 16/16-head
    layer from a state N(0, 0.1), every output and the final state / conv ring / position
    against the oracle -- no drift beyond tolerance."""
    rng = np.random.default_rng(7)
    shape = gdn_shape(16, 16)
    T = 4096
    proj, conv_w, A, dt_bias, norm_w = gdn_inputs(rng, shape, T)
    st = po.DeltaState.zeros(shape)
    st.ssm[:] = (0.1 * rng.standard_normal(st.ssm.shape)).astype(np.float32)
    with gdn_ctx(shape) as ctx:
        ctx.set_deltanet_weights(0, conv_w, A, dt_bias, norm_w)
        ctx.deltanet_state_import(0, 0, st.ssm, st.conv, 0)
        p = dev(proj, torch.float16)
        got = torch.stack([ctx.deltanet_from_proj(0, 0, p[t].contiguous()) for t in range(T)]).cpu().numpy()
        ssm, conv, pos = ctx.deltanet_state_export(0, 0)
    want = po.deltanet_tokens("oracle", shape, po.make_variant(), conv_w, A, dt_bias, norm_w, st, proj)
    assert_close(got, want, what=f"outputs over {T} tokens")
    assert_close(ssm, st.ssm, what=f"state after {T} tokens")
    np.testing.assert_array_equal(conv, st.conv)
    assert pos == st.conv_pos


# ---------------------------------------------------------------- batched / ragged serving decode

def test_full_attn_batched_ragged():
    rng = np.random.default_rng(11)
    shape = fa_shape(16, 4, 256, 64, 1e7)   # 4B shape
    caps = [300, 1000, 64, 2048, 700, 129]
    lens = [(300, 17), (640, 0), (64, 63), (1999, 100), (1, 5), (128, 120)]
    order = [3, 0, 5, 4, 1]                  # seq 2 idle; rows out of id order
    steps = 3
    rope = po.rope_table(4096, 64, 1e7)
    rings = [random_ring(rng, c, 4, 256, l, s) for c, (l, s) in zip(caps, lens)]
    _, qn, kn = fa_inputs(rng, shape, 1)
    projs = [f16(rng.standard_normal((steps, len(order), shape.num_q_heads * 512 + 2 * 4 * 256)))][0]
    pos0 = np.array([5000, 10, 77, 4090, 0, 129], np.int32)
    with fa_ctx(shape, caps=caps) as ctx:
        ctx.set_full_attn_weights(0, qn, kn)
        for s, r in enumerate(rings):
            ctx.kv_import(0, s, r.k, r.v, r.len, r.start)
        plan = ctx.plan(order)
        outs = []
        for t in range(steps):
            pos = dev(pos0[order] + t, torch.int32)
            outs.append(ctx.full_attn_decode(plan, 0, dev(projs[t], torch.float16), pos))
        got = torch.stack(outs).cpu().numpy()
        exported = [ctx.kv_export(0, s) for s in range(len(caps))]
        plan.close()
    for i, s in enumerate(order):
        want = po.full_attn_tokens("oracle", shape, po.make_variant(kv_round_f16=1), qn, kn, rings[s],
                                   projs[:, i], int(pos0[s]), rope)
        assert_close(got[:, i], want, what=f"row {i} (seq {s})")
        k, v, ln, st = exported[s]
        assert (ln, st) == (rings[s].len, rings[s].start), f"seq {s} ring metadata"
        np.testing.assert_array_equal(v, rings[s].v)
    # the idle sequence was not touched
    k, v, ln, st = exported[2]
    assert (ln, st) == lens[2]
    np.testing.assert_array_equal(v, rings[2].v)


def test_full_attn_batched_serving_lengths():
    """The multi-row plan at the serving workload's KV lengths (U[512, 32768]):
    a full 32,768-slot ring wrapped at slot 5000, one just short of full, lengths down to 512, and
    one ring that fills and starts evicting during the steps.  These are the long splits and the
    global-memory merge that the serving bench times; every row vs the oracle, ring metadata and
    V rows bit-exact."""
    rng = np.random.default_rng(21)
    shape = fa_shape(16, 4, 256, 64, 1e7)
    caps = [32768, 512, 20003, 32768, 8193, 700]
    lens = [(32768, 5000), (512, 0), (20001, 3), (31000, 0), (8191, 8000), (600, 650)]
    order = [2, 0, 5, 3, 1, 4]
    steps = 3
    rope = po.rope_table(4096, 64, 1e7)
    rings = [random_ring(rng, c, 4, 256, l, s) for c, (l, s) in zip(caps, lens)]
    _, qn, kn = fa_inputs(rng, shape, 1)
    projs = f16(rng.standard_normal((steps, len(order), shape.num_q_heads * 512 + 2 * 4 * 256)))
    pos0 = np.array([40000, 512, 20001, 31000, 8191, 600], np.int32)
    with fa_ctx(shape, caps=caps, max_seqs=len(caps)) as ctx:
        ctx.set_full_attn_weights(0, qn, kn)
        for s, r in enumerate(rings):
            ctx.kv_import(0, s, r.k, r.v, r.len, r.start)
        plan = ctx.plan(order)
        outs = []
        for t in range(steps):
            pos = dev(pos0[order] + t, torch.int32)
            outs.append(ctx.full_attn_decode(plan, 0, dev(projs[t], torch.float16), pos))
        got = torch.stack(outs).cpu().numpy()
        exported = [ctx.kv_export(0, s) for s in range(len(caps))]
        plan.close()
    for i, s in enumerate(order):
        want = po.full_attn_tokens("oracle", shape, po.make_variant(kv_round_f16=1), qn, kn, rings[s],
                                   projs[:, i], int(pos0[s]), rope)
        assert_close(got[:, i], want, what=f"row {i} (seq {s}, len {lens[s][0]})")
        k, v, ln, st = exported[s]
        assert (ln, st) == (rings[s].len, rings[s].start), f"seq {s} ring metadata"
        np.testing.assert_array_equal(v, rings[s].v)


def test_deltanet_batched():
    rng = np.random.default_rng(12)
    shape = gdn_shape(4, 8)
    n_seq, steps = 5, 3
    order = [4, 1, 3, 0]
    proj, conv_w, A, dt_bias, norm_w = gdn_inputs(rng, shape, steps * len(order))
    proj = proj.reshape(steps, len(order), -1)
    C = conv_w.shape[0]
    states = [po.DeltaState((0.1 * rng.standard_normal((8, 128, 128))).astype(np.float32),
                            rng.standard_normal((C, 3)).astype(np.float32), s % 3) for s in range(n_seq)]
    with gdn_ctx(shape, max_seqs=n_seq) as ctx:
        ctx.set_deltanet_weights(0, conv_w, A, dt_bias, norm_w)
        for s, st in enumerate(states):
            ctx.deltanet_state_import(0, s, st.ssm, st.conv, st.conv_pos)
        plan = ctx.plan(order)
        got = torch.stack([ctx.deltanet_decode(plan, 0, dev(proj[t], torch.float16)) for t in range(steps)])
        got = got.cpu().numpy()
        exported = [ctx.deltanet_state_export(0, s) for s in range(n_seq)]
        plan.close()
    for i, s in enumerate(order):
        want = po.deltanet_tokens("oracle", shape, po.make_variant(), conv_w, A, dt_bias, norm_w, states[s],
                                  proj[:, i])
        assert_close(got[:, i], want, what=f"row {i}")
        ssm, conv, pos = exported[s]
        assert_close(ssm, states[s].ssm, what=f"state {s}")
        np.testing.assert_array_equal(conv, states[s].conv)
        assert pos == states[s].conv_pos
    ssm, conv, pos = exported[2]
    np.testing.assert_array_equal(ssm, states[2].ssm)


@pytest.mark.parametrize("form", ["register", "staged"])
@pytest.mark.parametrize("Hv,n_seq", [(32, 40), (16, 24)])
@pytest.mark.parametrize("delta_mode", [ab.DELTA_CPUOPS, ab.DELTA_HF])
def test_deltanet_batched_gqa(delta_mode, Hv, n_seq, form, monkeypatch):
    """Larger batches, both forms of the wide-batch kernel (the state block in registers, or in and
    out by TMA tiles through shared memory -- the library picks by batch size, ANELM_GDN_STAGED
    forces one): 40 rows x 16 key heads in the 4B GQA shape (two value heads per key head) and 24
    rows of the 0.8B shape (one), 3 steps, rows in shuffled order, both delta-rule orders: every
    row's outputs / state / conv ring / position vs the oracle."""
    monkeypatch.setenv("ANELM_GDN_STAGED", "1" if form == "staged" else "0")
    rng = np.random.default_rng(40 + delta_mode + Hv)
    shape = gdn_shape(16, Hv)
    steps = 3
    order = list(rng.permutation(n_seq))
    proj, conv_w, A, dt_bias, norm_w = gdn_inputs(rng, shape, steps * n_seq)
    proj = proj.reshape(steps, n_seq, -1)
    C = conv_w.shape[0]
    states = [po.DeltaState((0.1 * rng.standard_normal((Hv, 128, 128))).astype(np.float32),
                            rng.standard_normal((C, 3)).astype(np.float32), s % 3) for s in range(n_seq)]
    var = po.make_variant(delta_hf=int(delta_mode == ab.DELTA_HF))
    with gdn_ctx(shape, max_seqs=n_seq, delta_mode=delta_mode) as ctx:
        ctx.set_deltanet_weights(0, conv_w, A, dt_bias, norm_w)
        for s, st in enumerate(states):
            ctx.deltanet_state_import(0, s, st.ssm, st.conv, st.conv_pos)
        plan = ctx.plan(order)
        got = torch.stack([ctx.deltanet_decode(plan, 0, dev(proj[t], torch.float16)) for t in range(steps)])
        got = got.cpu().numpy()
        exported = [ctx.deltanet_state_export(0, s) for s in range(n_seq)]
        plan.close()
    for i, s in enumerate(order):
        want = po.deltanet_tokens("oracle", shape, var, conv_w, A, dt_bias, norm_w, states[s], proj[:, i])
        assert_close(got[:, i], want, what=f"row {i} (seq {s})")
        ssm, conv, pos = exported[s]
        assert_close(ssm, states[s].ssm, what=f"state {s}")
        np.testing.assert_array_equal(conv, states[s].conv)
        assert pos == states[s].conv_pos


# ---------------------------------------------------------------- variants

def test_deltanet_hf_variant():
    """Decay-first delta rule with L2 eps 1e-6 (export_hybrid_chunks.py:142-147)."""
    rng = np.random.default_rng(13)
    shape = gdn_shape(2, 4)
    T = 12
    proj, conv_w, A, dt_bias, norm_w = gdn_inputs(rng, shape, T)
    st = po.DeltaState.zeros(shape)
    st.ssm[:] = (0.1 * rng.standard_normal(st.ssm.shape)).astype(np.float32)
    with gdn_ctx(shape, delta_mode=ab.DELTA_HF, l2_eps=1e-6) as ctx:
        ctx.set_deltanet_weights(0, conv_w, A, dt_bias, norm_w)
        ctx.deltanet_state_import(0, 0, st.ssm, st.conv, 0)
        p = dev(proj)
        got = torch.stack([ctx.deltanet_from_proj(0, 0, p[t].contiguous()) for t in range(T)]).cpu().numpy()
    want = po.deltanet_tokens("oracle", shape, po.make_variant(delta_hf=1, l2_eps=1e-6), conv_w, A, dt_bias,
                              norm_w, st, proj)
    assert_close(got, want, what="HF-order DeltaNet")


@pytest.mark.parametrize("route", ["decode", "prefill"])
def test_deltanet_hf_variant_matches_reference_layer(golden, route):
    """The decay-first variant against the hybrid v2 export's own DeltaNetLayer
    (scripts/export_hybrid_chunks.py:83-160, run from the reference source into
    tests/golden/deltanet_hf_ref.npz): its shift-register conv state converted to the
    context's ring, 16 tokens token by token (decode) or as one chunked prefill."""
    from anelm_b200.state_layout import conv_ring_to_shift, conv_shift_to_ring

    g = golden("deltanet_hf_ref.npz")
    Hk, Hv, dk, dv, K = (int(x) for x in g["dims"])
    shape = gdn_shape(Hk, Hv, dk, dv)
    ring, pos0 = conv_shift_to_ring(g["shift0"])
    proj = g["proj"].astype(np.float32)
    with gdn_ctx(shape, delta_mode=ab.DELTA_HF) as ctx:
        ctx.set_deltanet_weights(0, g["conv_w"], g["A"], g["dt_bias"], g["norm_w"])
        ctx.deltanet_state_import(0, 0, g["ssm0"], ring, pos0)
        p = dev(proj, torch.float16)
        if route == "decode":
            got = torch.stack([ctx.deltanet_from_proj(0, 0, p[t].contiguous()) for t in range(p.shape[0])])
        else:
            plan = ctx.plan([0])
            got = ctx.deltanet_prefill(plan, 0, p[None].contiguous())[0]
            plan.close()
        got = got.cpu().numpy()
        ssm, conv, pos = ctx.deltanet_state_export(0, 0)
    assert_close(got, g["out"], what=f"HF-order {route} vs export_hybrid_chunks DeltaNetLayer")
    assert_close(ssm, g["ssm"], what="HF-order state")
    np.testing.assert_array_equal(conv_ring_to_shift(conv, pos)[:, 1:], g["shift"][:, 1:])


def test_full_attn_python_route_variant():
    """Rotate-half RoPE, no QK-norm in the core, linear KV at pos (serve_hybrid.py:85-132)."""
    rng = np.random.default_rng(14)
    shape = fa_shape(16, 4, 256, 64, 1e7)
    T, cap = 20, 64
    proj, qn, kn = fa_inputs(rng, shape, T)
    ring = po.KVRing.empty(cap, 4, 256)
    rope = po.rope_table(cap, 64, 1e7)
    with fa_ctx(shape, cap=cap, rope_table_len=cap, rope_mode=ab.ROPE_HALF, qk_norm_in_core=0,
                kv_mode=ab.KV_LINEAR) as ctx:
        p = dev(proj, torch.float16)
        got = torch.stack([ctx.full_attn_from_proj(0, 0, p[t].contiguous(), t) for t in range(T)]).cpu().numpy()
    want = po.full_attn_tokens("oracle", shape, po.make_variant(rope_half=1, no_qk_norm=1, kv_linear=1,
                                                                kv_round_f16=1), qn, kn, ring, proj, 0, rope)
    assert_close(got, want, what="python-route attention")


def test_serve_hybrid_dropin_matches_reference_golden(golden):
    from anelm_b200.serve_hybrid import CudaAttention
    g = golden("serve_hybrid_ref.npz")
    H, KVH, HD, RD, CTX = (int(v) for v in g["consts"])
    attn = CudaAttention(n_layers=2, num_heads=H, num_kv_heads=KVH, head_dim=HD, rope_dim=RD, context=CTX,
                         rope_theta=float(g["rope_theta"]))
    kv = attn.new_kv_caches()
    outs = [attn.cpu_attention(g["q_gate"][t], g["k"][t], g["v"][t], t, kv, 1) for t in range(g["q_gate"].shape[0])]
    got = np.concatenate(outs, 0)
    assert got.dtype == np.float16 and got.shape == g["out"].shape
    assert_close(got.astype(np.float32), g["out"].astype(np.float32), what="serve_hybrid cpu_attention")
    attn.ctx.close()


# ---------------------------------------------------------------- errors (no fault, status codes)

def test_errors_are_status_codes():
    shape = fa_shape()
    with fa_ctx(shape, cap=16, kv_mode=ab.KV_LINEAR, qk_norm_in_core=0) as ctx:
        p = torch.zeros(ctx.fa_proj_dim, device="cuda")
        with pytest.raises(ab.AnelmError) as e:
            ctx.full_attn_from_proj(0, 0, p, 16)          # position beyond the linear cache
        assert e.value.status == 2
        with pytest.raises(ab.AnelmError) as e:
            ctx.full_attn_from_proj(0, 3, p, 0)           # no such sequence
        assert e.value.status == 1
        plan = ctx.plan([0])
        pos = torch.tensor([99], dtype=torch.int32, device="cuda")
        proj = torch.zeros((1, ctx.fa_proj_dim), device="cuda")
        ctx.full_attn_decode(plan, 0, proj, pos)          # device-side position check
        assert ctx.device_error() == 2
        assert ctx.device_error() == 0
        k, v, ln, st = ctx.kv_export(0, 0)
        assert ln == 0 and not k.any()                    # nothing was written
        plan.close()
    with gdn_ctx(gdn_shape(2, 2)) as ctx:
        with pytest.raises(ab.AnelmError) as e:
            ctx.deltanet_from_proj(0, 0, torch.zeros(ctx.gdn_proj_dim, device="cuda"))
        assert e.value.status == 6                        # weights not set


def test_bounded_wait_gives_up_and_the_context_stays_usable():
    """The failure path of every mbarrier wait in the tensor-core kernels: a wait on a barrier that
    nothing arrives on gives up after its poll budget, records ANELM_ERR_TIMEOUT in the context's
    error word and returns (no trap, no hang); the status is read on the host and cleared, and the
    context then decodes correctly."""
    from anelm_b200._lib import lib

    rng = np.random.default_rng(31)
    shape = fa_shape()
    proj, qn, kn = fa_inputs(rng, shape, 2)
    with fa_ctx(shape, cap=64) as ctx:
        ctx.set_full_attn_weights(0, qn, kn)
        assert ctx.device_error() == 0
        assert lib().anelm_selftest_wait_timeout(ctx.handle, 4096, None) == 0
        assert ctx.device_error() == ab._lib.ERR_TIMEOUT
        assert ctx.device_error() == 0                      # read and cleared
        assert lib().anelm_selftest_wait_timeout(ctx.handle, 0, None) == ab._lib.ERR_INVALID_ARG
        p = dev(proj, torch.float16)
        got = torch.stack([ctx.full_attn_from_proj(0, 0, p[t].contiguous(), t) for t in range(2)]).cpu().numpy()
        assert ctx.device_error() == 0
    want = po.full_attn_tokens("oracle", shape, po.make_variant(kv_round_f16=1), qn, kn, po.KVRing.empty(64, 2, 256),
                               proj, 0, po.rope_table(4096, 64, 1e7))
    assert_close(got, want, what="decode after a timed-out wait")

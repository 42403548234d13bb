"""Pins the CPU oracle (oracle/liboracle.so, oracle/serve_hybrid_oracle.py) against
the reference: the golden fixtures made from the reference's own cpu_ops.cpp and
serve_hybrid.cpu_attention, and -- where oracle/_ref was built -- the reference
library live on fresh seeded inputs.  CPU only."""
import numpy as np
import pytest

from oracle import pyoracle as po
from oracle import serve_hybrid_oracle as sho

P = po.P


def test_ops_match_golden(golden):
    g = golden("cpu_ops_ref.npz")
    L = po.lib("oracle")
    x, z, w = g["x"], g["z"], g["w"]
    tmp = np.zeros(256, np.float32)
    o = np.zeros(256, np.float32); L.orc_rmsnorm(P(o), P(x), P(w), 256, 1e-6)
    np.testing.assert_array_equal(o, g["rmsnorm"])
    o = np.zeros(256, np.float32); L.orc_rmsnorm_gated(P(o), P(x), P(z), P(w), 256)
    np.testing.assert_array_equal(o, g["rmsnorm_gated"])
    o = x.copy(); L.orc_l2_normalize(P(o), 256); np.testing.assert_array_equal(o, g["l2_normalize"])
    o = x.copy(); L.orc_silu_vec_inplace(P(o), 256, P(tmp)); np.testing.assert_array_equal(o, g["silu"])
    o = x.copy(); L.orc_mul_sigmoid_inplace(P(o), P(z), 256, P(tmp))
    np.testing.assert_array_equal(o, g["mul_sigmoid"])
    o = x.copy(); L.orc_softmax(P(o), 256); np.testing.assert_array_equal(o, g["softmax"])
    o = np.zeros(64, np.float32); L.orc_matvec(P(o), P(g["matvec_W"]), P(x), 64, 256)
    np.testing.assert_array_equal(o, g["matvec"])


def test_rope_matches_golden(golden):
    g = golden("cpu_ops_ref.npz")
    L = po.lib("oracle")
    cos, sin = po.rope_table(4096, 64, 1e7)
    for tag, pos, c, s in (("table", 1234, cos[1234].copy(), sin[1234].copy()), ("fly", 5000, None, None)):
        q, k = g["rope_q_in"].copy(), g["rope_k_in"].copy()
        L.orc_apply_rope_cached(P(q), P(k), 4, 2, 256, 512, 256, 64, pos, 1e7, P(c), P(s))
        np.testing.assert_array_equal(q, g[f"rope_{tag}_q"])
        np.testing.assert_array_equal(k, g[f"rope_{tag}_k"])


def test_conv_ssm_gqa_match_golden(golden):
    g = golden("cpu_ops_ref.npz")
    L = po.lib("oracle")
    C = g["conv_w"].shape[0]
    cs = g["conv_state0"].copy()
    pos = np.zeros(1, np.int32)
    ys = np.zeros_like(g["conv_y"])
    for t in range(ys.shape[0]):
        L.orc_conv1d_update(P(ys[t]), P(cs), P(pos), P(g["conv_x"][t].copy()), P(g["conv_w"]), C, 4)
    np.testing.assert_array_equal(ys, g["conv_y"])
    np.testing.assert_array_equal(cs, g["conv_state"])
    assert pos[0] == g["conv_pos"][0]

    S = g["ssm_S0"].copy()
    y = np.zeros(128, np.float32)
    L.orc_ssm_step(P(y), P(S), P(g["ssm_q"]), P(g["ssm_k"]), P(g["ssm_v"]), 0.9, 0.3, 128, 128)
    np.testing.assert_array_equal(y, g["ssm_y"])
    np.testing.assert_array_equal(S, g["ssm_S"])

    for tag, start, ln in (("wrap", 17, 24), ("part", 5, 11), ("empty", 0, 0)):
        o = np.full((4, 256), 7.0, np.float32)
        L.orc_gqa_attention(P(o), P(g["gqa_q"]), P(g["gqa_k"]), P(g["gqa_v"]), 4, 2, 256, 512, start, ln, 24)
        np.testing.assert_array_equal(o, g[f"gqa_{tag}"])


def test_full_attn_glue_matches_golden(golden):
    g = golden("full_attn_ref.npz")
    shape = po.make_shape(num_q_heads=8, num_kv_heads=2, head_dim=256, rot_dim=64, rope_theta=1e7)
    ring = po.KVRing.empty(int(g["cap"]), 2, 256)
    out = po.full_attn_tokens("oracle", shape, po.make_variant(), g["q_norm"], g["k_norm"], ring,
                              g["proj"].astype(np.float32), int(g["start_pos"]), po.rope_table(4096, 64, 1e7))
    np.testing.assert_array_equal(out, g["out"])
    np.testing.assert_array_equal(ring.k, g["k_cache"])
    np.testing.assert_array_equal(ring.v, g["v_cache"])
    assert (ring.len, ring.start) == (int(g["len"]), int(g["start"]))


def test_deltanet_glue_matches_golden(golden):
    g = golden("deltanet_ref.npz")
    Hv, dk = g["ssm0"].shape[0], g["ssm0"].shape[1]
    C = g["conv0"].shape[0]
    Hk = (C - Hv * dk) // (2 * dk)
    shape = po.make_shape(lin_num_key_heads=Hk, lin_num_val_heads=Hv, lin_key_dim=dk, lin_val_dim=dk)
    st = po.DeltaState(g["ssm0"].copy(), g["conv0"].copy(), int(g["conv_pos0"]))
    out = po.deltanet_tokens("oracle", shape, po.make_variant(), g["conv_w"], g["A"], g["dt_bias"],
                             g["norm_w"], st, g["proj"].astype(np.float32))
    np.testing.assert_array_equal(out, g["out"])
    np.testing.assert_array_equal(st.ssm, g["ssm"])
    np.testing.assert_array_equal(st.conv, g["conv"])
    assert st.conv_pos == int(g["conv_pos"])


def test_serve_hybrid_restatement_matches_golden(golden):
    g = golden("serve_hybrid_ref.npz")
    H, KVH, HD, RD, CTX = (int(v) for v in g["consts"])
    cfg = sho.HybridAttnConfig(H, KVH, HD, RD, CTX, float(g["rope_theta"]))
    kv = cfg.new_kv_caches(1)
    outs = [sho.cpu_attention(cfg, g["q_gate"][t], g["k"][t], g["v"][t], t, kv, 0)
            for t in range(g["q_gate"].shape[0])]
    got = np.concatenate(outs, 0).astype(np.float32)
    np.testing.assert_allclose(got, g["out"].astype(np.float32), atol=2e-3, rtol=1e-2)


@pytest.mark.skipif(not po.available("ref"), reason="reference sources were not present to build oracle/_ref")
@pytest.mark.parametrize("seed", [0, 1])
def test_oracle_equals_reference_live(seed):
    """C restatement vs the reference's cpu_ops.cpp on fresh inputs (bit-exact)."""
    rng = np.random.default_rng(100 + seed)
    shape = po.make_shape(num_q_heads=4, num_kv_heads=1, head_dim=256, lin_num_key_heads=2,
                          lin_num_val_heads=4)
    var = po.make_variant()
    qn = (1 + 0.02 * rng.standard_normal(256)).astype(np.float32)
    kn = (1 + 0.02 * rng.standard_normal(256)).astype(np.float32)
    proj = rng.standard_normal((20, 4 * 512 + 2 * 256)).astype(np.float32)
    outs = []
    for kind in ("oracle", "ref"):
        ring = po.KVRing.empty(8, 1, 256)
        outs.append((po.full_attn_tokens(kind, shape, var, qn, kn, ring, proj, 3), ring.k.copy()))
    np.testing.assert_array_equal(outs[0][0], outs[1][0])
    np.testing.assert_array_equal(outs[0][1], outs[1][1])

    C = 2 * 2 * 128 + 4 * 128
    proj = rng.standard_normal((6, C + 4 * 128 + 8)).astype(np.float32)
    cw = rng.standard_normal((C, 4)).astype(np.float32)
    A = np.ones(4, np.float32); dtb = np.zeros(4, np.float32); nw = np.ones(128, np.float32)
    res = []
    for kind in ("oracle", "ref"):
        st = po.DeltaState((0.1 * np.random.default_rng(seed).standard_normal((4, 128, 128))).astype(np.float32),
                           np.zeros((C, 3), np.float32), 0)
        res.append((po.deltanet_tokens(kind, shape, var, cw, A, dtb, nw, st, proj), st.ssm.copy()))
    np.testing.assert_array_equal(res[0][0], res[1][0])
    np.testing.assert_array_equal(res[0][1], res[1][1])


# ---------------------------------------------------------------- decay-first (HF-order) DeltaNet

def _hf_oracle_run(g, l2_eps):
    from anelm_b200.state_layout import conv_shift_to_ring

    Hk, Hv, dk, dv, K = (int(x) for x in g["dims"])
    shape = po.make_shape(lin_num_key_heads=Hk, lin_num_val_heads=Hv, lin_key_dim=dk, lin_val_dim=dv,
                          conv_kernel=K)
    ring, pos = conv_shift_to_ring(g["shift0"])
    st = po.DeltaState(g["ssm0"].copy(), ring.copy(), pos)
    out = po.deltanet_tokens("oracle", shape, po.make_variant(delta_hf=1, l2_eps=l2_eps), g["conv_w"], g["A"],
                             g["dt_bias"], g["norm_w"], st, g["proj"].astype(np.float32))
    return out, st


@pytest.mark.parametrize("l2_eps", [0.0, 1e-6])
def test_oracle_hf_order_matches_reference_layer(golden, l2_eps):
    """The oracle's decay-first branch against the hybrid v2 export's own DeltaNetLayer
    (scripts/export_hybrid_chunks.py:83-160, run from the reference source by
    tests/golden/make_golden.py): outputs and state within the parity tolerance, the conv
    shift register bit-exact.  Both L2 forms agree with F.normalize here: cpu_ops's
    sqrt(sum + 1e-12) (l2_eps 0) and the validators' rsqrt(sum + 1e-6)."""
    from anelm_b200.state_layout import conv_ring_to_shift
    from helpers import assert_close

    g = golden("deltanet_hf_ref.npz")
    out, st = _hf_oracle_run(g, l2_eps)
    assert_close(out, g["out"], what="HF-order outputs vs export_hybrid_chunks DeltaNetLayer")
    assert_close(st.ssm, g["ssm"], what="HF-order state")
    np.testing.assert_array_equal(conv_ring_to_shift(st.conv, st.conv_pos)[:, 1:], g["shift"][:, 1:])
    # much closer than the tolerance: the same fp32 math in another order
    assert np.abs(out - g["out"]).max() < 1e-4


def test_oracle_hf_order_is_not_the_cpuops_order(golden):
    """The fixture separates the two delta-rule orders: the cpu_ops order misses it."""
    from anelm_b200.state_layout import conv_shift_to_ring

    g = golden("deltanet_hf_ref.npz")
    Hk, Hv, dk, dv, K = (int(x) for x in g["dims"])
    shape = po.make_shape(lin_num_key_heads=Hk, lin_num_val_heads=Hv, lin_key_dim=dk, lin_val_dim=dv)
    ring, pos = conv_shift_to_ring(g["shift0"])
    st = po.DeltaState(g["ssm0"].copy(), ring.copy(), pos)
    out = po.deltanet_tokens("oracle", shape, po.make_variant(), g["conv_w"], g["A"], g["dt_bias"], g["norm_w"],
                             st, g["proj"].astype(np.float32))
    assert np.abs(out - g["out"]).max() > 1e-2


@pytest.mark.parametrize("Hk,Hv,T", [(2, 4, 70), (1, 2, 130)])
def test_oracle_delta_rule_matches_transformers(Hk, Hv, T):
    """The bare decay-first delta rule (oracle gated_delta_tokens, delta_hf=1) against the
    installed transformers Qwen3.5 implementation, called as a library:
    torch_recurrent_gated_delta_rule and the chunked torch_chunk_gated_delta_rule (chunk 64,
    T not a multiple of it), from a nonzero initial state.  transformers scales q by
    1/sqrt(dk) itself and wants q/k repeated to the value heads."""
    torch = pytest.importorskip("torch")
    mq = pytest.importorskip("transformers.models.qwen3_5.modeling_qwen3_5")
    from helpers import assert_close

    rng = np.random.default_rng(T)
    dk = dv = 128
    q = rng.standard_normal((T, Hk, dk)).astype(np.float32)
    q /= np.linalg.norm(q, axis=-1, keepdims=True)
    k = rng.standard_normal((T, Hk, dk)).astype(np.float32)
    k /= np.linalg.norm(k, axis=-1, keepdims=True)
    v = rng.standard_normal((T, Hv, dv)).astype(np.float32)
    lg = (-0.1 * rng.random((T, Hv)) - 0.01).astype(np.float32)
    beta = rng.random((T, Hv)).astype(np.float32)
    s0 = (0.1 * rng.standard_normal((Hv, dk, dv))).astype(np.float32)
    st = s0.copy()
    y = po.gated_delta_tokens("oracle", q / np.sqrt(dk), k, v, lg, beta, st, delta_hf=1)

    rep = Hv // Hk
    tq = torch.from_numpy(np.repeat(q, rep, axis=1))[None]
    tk = torch.from_numpy(np.repeat(k, rep, axis=1))[None]
    tv, tg, tb = (torch.from_numpy(a)[None] for a in (v, lg, beta))
    init = torch.from_numpy(s0)[None]
    y_rec, s_rec = mq.torch_recurrent_gated_delta_rule(tq, tk, tv, tg, tb, init.clone(), True)
    assert_close(y, y_rec[0].numpy(), what="vs torch_recurrent_gated_delta_rule")
    assert_close(st, s_rec[0].numpy(), what="state vs torch_recurrent_gated_delta_rule")
    y_ch, s_ch = mq.torch_chunk_gated_delta_rule(tq, tk, tv, tg, tb, initial_state=init.clone(),
                                                 output_final_state=True)
    assert_close(y, y_ch[0].numpy(), what="vs torch_chunk_gated_delta_rule")
    assert_close(st, s_ch[0].numpy(), what="state vs torch_chunk_gated_delta_rule")

"""GPU parity of the op-level entry points (the core/cpu_ops.h mirror on device
pointers) against the golden fixtures made from the reference's cpu_ops.cpp."""
import ctypes

import numpy as np
import pytest

torch = pytest.importorskip("torch")

import anelm_b200 as ab  # noqa: E402
from anelm_b200._lib import check, lib  # noqa: E402
from helpers import assert_close, f16  # noqa: E402
from oracle import pyoracle as po  # noqa: E402

pytestmark = pytest.mark.gpu


def D(a):
    return torch.from_numpy(np.ascontiguousarray(a, np.float32)).cuda()


def P(t):
    return ctypes.c_void_p(t.data_ptr()) if t is not None else None


def test_vector_ops(golden):
    g = golden("cpu_ops_ref.npz")
    L = lib()
    x, z, w = D(g["x"]), D(g["z"]), D(g["w"])
    o = torch.empty_like(x)
    check(L.anelm_rmsnorm(P(o), P(x), P(w), 256, 1e-6, 1, None), "rmsnorm")
    assert_close(o.cpu(), g["rmsnorm"], atol=1e-6, rtol=1e-5, what="rmsnorm")
    check(L.anelm_rmsnorm_gated(P(o), P(x), P(z), P(w), 256, 1, None), "rmsnorm_gated")
    assert_close(o.cpu(), g["rmsnorm_gated"], atol=1e-6, rtol=1e-5, what="rmsnorm_gated")
    o = x.clone(); check(L.anelm_l2_normalize(P(o), 256, 1, None), "l2")
    assert_close(o.cpu(), g["l2_normalize"], atol=1e-7, rtol=1e-5, what="l2")
    o = x.clone(); check(L.anelm_silu_vec_inplace(P(o), 256, None), "silu")
    assert_close(o.cpu(), g["silu"], atol=1e-6, rtol=1e-5, what="silu")
    o = x.clone(); check(L.anelm_mul_sigmoid_inplace(P(o), P(z), 256, None), "mul_sigmoid")
    assert_close(o.cpu(), g["mul_sigmoid"], atol=1e-6, rtol=1e-5, what="mul_sigmoid")
    o = x.clone(); check(L.anelm_softmax(P(o), 256, 1, None), "softmax")
    assert_close(o.cpu(), g["softmax"], atol=1e-7, rtol=1e-5, what="softmax")
    W = D(g["matvec_W"]); y = torch.empty(64, device="cuda")
    check(L.anelm_matvec(P(y), P(W), P(x), 64, 256, None), "matvec")
    assert_close(y.cpu(), g["matvec"], atol=1e-4, rtol=1e-5, what="matvec")


def test_rope_op(golden):
    g = golden("cpu_ops_ref.npz")
    L = lib()
    cos, sin = po.rope_table(4096, 64, 1e7)
    for tag, pos, c, s in (("table", 1234, D(cos[1234]), D(sin[1234])), ("fly", 5000, None, None)):
        q, k = D(g["rope_q_in"]), D(g["rope_k_in"])
        check(L.anelm_apply_rope_cached(P(q), P(k), 4, 2, 256, 512, 256, 64, pos, 1e7, P(c), P(s), None), "rope")
        assert_close(q.cpu(), g[f"rope_{tag}_q"], atol=1e-5, rtol=1e-5, what=f"rope {tag} q")
        assert_close(k.cpu(), g[f"rope_{tag}_k"], atol=1e-5, rtol=1e-5, what=f"rope {tag} k")


def test_conv_ssm_ops(golden):
    g = golden("cpu_ops_ref.npz")
    L = lib()
    C = g["conv_w"].shape[0]
    st, w = D(g["conv_state0"]), D(g["conv_w"])
    pos = ctypes.c_int(0)
    ys = []
    for t in range(g["conv_x"].shape[0]):
        y = torch.empty(C, device="cuda")
        x = D(g["conv_x"][t])  # keep a reference: the kernel runs asynchronously
        check(L.anelm_conv1d_update(P(y), P(st), ctypes.byref(pos), P(x), P(w), C, 4, None), "conv")
        ys.append((y, x))
    ys = [y for y, _ in ys]
    assert_close(torch.stack(ys).cpu(), g["conv_y"], atol=1e-6, rtol=1e-6, what="conv y")
    np.testing.assert_array_equal(st.cpu().numpy(), g["conv_state"])
    assert pos.value == int(g["conv_pos"][0])
    S, y = D(g["ssm_S0"]), torch.empty(128, device="cuda")
    q, k, v = D(g["ssm_q"]), D(g["ssm_k"]), D(g["ssm_v"])
    check(L.anelm_ssm_step(P(y), P(S), P(q), P(k), P(v), 0.9, 0.3, 128, 128, None), "ssm_step")
    assert_close(y.cpu(), g["ssm_y"], atol=1e-5, rtol=1e-4, what="ssm y")
    assert_close(S.cpu(), g["ssm_S"], atol=1e-6, rtol=1e-5, what="ssm S")


@pytest.mark.parametrize("kv_dtype", [ab.F32, ab.F16])
def test_gqa_attention_op(golden, kv_dtype):
    g = golden("cpu_ops_ref.npz")
    L = lib()
    tdt = torch.float32 if kv_dtype == ab.F32 else torch.float16
    kc = torch.from_numpy(g["gqa_k"]).to("cuda", tdt)
    vc = torch.from_numpy(g["gqa_v"]).to("cuda", tdt)
    q = D(g["gqa_q"])
    for tag, start, ln in (("wrap", 17, 24), ("part", 5, 11), ("empty", 0, 0)):
        o = torch.full((4, 256), 7.0, device="cuda")
        check(L.anelm_gqa_attention(P(o), P(q), P(kc), P(vc), kv_dtype, 4, 2, 256, 512, start, ln, 24, None), tag)
        assert_close(o.cpu(), g[f"gqa_{tag}"], what=f"gqa {tag}")


def test_gqa_attention_op_long_fp16():
    """A 30000-slot fp16 ring, wrapped: many splits merged."""
    rng = np.random.default_rng(21)
    cap, Hq, Hkv, d = 30000, 8, 2, 256
    kc = f16(rng.standard_normal((cap, Hkv, d)))
    vc = f16(rng.standard_normal((cap, Hkv, d)))
    q = (3 * rng.standard_normal((Hq, 2 * d))).astype(np.float32)
    want = np.zeros((Hq, d), np.float32)
    po.lib("oracle").orc_gqa_attention(po.P(want), po.P(q), po.P(kc), po.P(vc), Hq, Hkv, d, 2 * d, 12345, 29999, cap)
    o = torch.empty((Hq, d), device="cuda")
    qd, kd, vd = D(q), torch.from_numpy(kc).half().cuda(), torch.from_numpy(vc).half().cuda()
    check(lib().anelm_gqa_attention(P(o), P(qd), P(kd), P(vd), ab.F16, Hq, Hkv, d, 2 * d, 12345, 29999, cap, None),
          "gqa long")
    assert_close(o.cpu(), want, what="long wrapped ring")

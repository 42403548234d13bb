"""The link-compatible cpu_ops replacement (include/cpu_ops_compat/cpu_ops.h, namespace ane_lm,
host pointers) on the GPU.  The oracle's layer glue, written against the reference's
core/cpu_ops.h, is compiled against the shim instead of core/cpu_ops.cpp (exactly what a
reference build relinked against libanelm_b200.so does); every op and both per-token layer
loops (qwen3_5.cpp:849-1002 as restated in oracle/glue_impl.h) then run through the B200
kernels and are compared with the oracle.  Tolerance 2e-3 abs + 1e-2 rel; ring / conv position
bookkeeping bit-exact."""
import ctypes
import os
import shutil
import subprocess

import numpy as np
import pytest

torch = pytest.importorskip("torch")

import anelm_b200 as ab  # noqa: E402
from helpers import assert_close, f16, fa_inputs, fa_shape, gdn_inputs, gdn_shape, random_ring  # noqa: E402
from oracle import pyoracle as po  # noqa: E402

pytestmark = pytest.mark.gpu

REPO = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))


@pytest.fixture(scope="module")
def shim(tmp_path_factory):
    gxx = shutil.which("g++")
    if not gxx:
        pytest.skip("no g++")
    libdir = os.path.dirname(ab.LIB_PATH)
    out = tmp_path_factory.mktemp("shim") / "libshim_glue.so"
    r = subprocess.run([gxx, "-O2", "-fPIC", "-shared", "-std=c++17", f"-I{REPO}/include/cpu_ops_compat",
                        f"-I{REPO}/oracle", f"{REPO}/oracle/ref_glue.cpp", f"-L{libdir}", "-lanelm_b200",
                        f"-Wl,-rpath,{libdir}", "-o", str(out)], capture_output=True, text=True)
    assert r.returncode == 0, r.stderr[-3000:]
    po.LIBS["shim"] = str(out)
    po.PREFIX["shim"] = "ref_"
    return "shim"


P = po.P


def test_elementwise_and_norm_ops(shim):
    rng = np.random.default_rng(1)
    x = rng.standard_normal(300).astype(np.float32)
    z = rng.standard_normal(300).astype(np.float32)
    w = (1 + 0.1 * rng.standard_normal(300)).astype(np.float32)
    tmp = np.zeros(300, np.float32)
    for name, args in [("silu_vec_inplace", None), ("l2_normalize", None), ("softmax", None)]:
        a, b = x.copy(), x.copy()
        if name == "silu_vec_inplace":
            po.fn(shim, name)(P(a), 300, P(tmp))
            po.fn("oracle", name)(P(b), 300, P(tmp))
        else:
            po.fn(shim, name)(P(a), 300)
            po.fn("oracle", name)(P(b), 300)
        assert_close(a, b, what=name)
    a, b = x.copy(), x.copy()
    po.fn(shim, "mul_sigmoid_inplace")(P(a), P(z), 300, P(tmp))
    po.fn("oracle", "mul_sigmoid_inplace")(P(b), P(z), 300, P(tmp))
    assert_close(a, b, what="mul_sigmoid_inplace")
    o1, o2 = np.zeros(300, np.float32), np.zeros(300, np.float32)
    po.fn(shim, "rmsnorm")(P(o1), P(x), P(w), 300, 1e-6)
    po.fn("oracle", "rmsnorm")(P(o2), P(x), P(w), 300, 1e-6)
    assert_close(o1, o2, what="rmsnorm")
    po.fn(shim, "rmsnorm_gated")(P(o1), P(x), P(z), P(w), 300)
    po.fn("oracle", "rmsnorm_gated")(P(o2), P(x), P(z), P(w), 300)
    assert_close(o1, o2, what="rmsnorm_gated")
    W = rng.standard_normal((40, 300)).astype(np.float32)
    y1, y2 = np.zeros(40, np.float32), np.zeros(40, np.float32)
    po.fn(shim, "matvec")(P(y1), P(W), P(x), 40, 300)
    po.fn("oracle", "matvec")(P(y2), P(W), P(x), 40, 300)
    assert_close(y1, y2, what="matvec")


def test_rope_conv_ssm_attention_ops(shim):
    rng = np.random.default_rng(2)
    q = rng.standard_normal((4, 512)).astype(np.float32)
    k = rng.standard_normal((2, 256)).astype(np.float32)
    c, s = po.rope_table(64, 64, 1e7)
    for cos_row, sin_row in [(c[37].copy(), s[37].copy()), (None, None)]:
        q1, k1, q2, k2 = q.copy(), k.copy(), q.copy(), k.copy()
        po.fn(shim, "apply_rope_cached")(P(q1), P(k1), 4, 2, 256, 512, 256, 64, 37, 1e7, P(cos_row), P(sin_row))
        po.fn("oracle", "apply_rope_cached")(P(q2), P(k2), 4, 2, 256, 512, 256, 64, 37, 1e7, P(cos_row), P(sin_row))
        assert_close(q1, q2, what="rope q")
        assert_close(k1, k2, what="rope k")
    C = 96
    st1 = rng.standard_normal((C, 3)).astype(np.float32)
    st2 = st1.copy()
    wts = rng.standard_normal((C, 4)).astype(np.float32)
    p1, p2 = ctypes.c_int(2), ctypes.c_int(2)
    for _ in range(4):
        x = rng.standard_normal(C).astype(np.float32)
        y1, y2 = np.zeros(C, np.float32), np.zeros(C, np.float32)
        po.fn(shim, "conv1d_update")(P(y1), P(st1), ctypes.byref(p1), P(x), P(wts), C, 4)
        po.fn("oracle", "conv1d_update")(P(y2), P(st2), ctypes.byref(p2), P(x), P(wts), C, 4)
        assert_close(y1, y2, what="conv1d_update")
        np.testing.assert_array_equal(st1, st2)
        assert p1.value == p2.value
    S1 = (0.1 * rng.standard_normal((128, 128))).astype(np.float32)
    S2 = S1.copy()
    for _ in range(3):
        qq = rng.standard_normal(128).astype(np.float32)
        kk = rng.standard_normal(128).astype(np.float32)
        vv = rng.standard_normal(128).astype(np.float32)
        y1, y2 = np.zeros(128, np.float32), np.zeros(128, np.float32)
        po.fn(shim, "ssm_step")(P(y1), P(S1), P(qq), P(kk), P(vv), 0.9, 0.4, 128, 128)
        po.fn("oracle", "ssm_step")(P(y2), P(S2), P(qq), P(kk), P(vv), 0.9, 0.4, 128, 128)
        assert_close(y1, y2, what="ssm_step y")
        assert_close(S1, S2, what="ssm_step state")
    ring = random_ring(rng, 300, 2, 256, 300, 123)
    o1, o2 = np.zeros((8, 256), np.float32), np.zeros((8, 256), np.float32)
    qa = rng.standard_normal((8, 512)).astype(np.float32)
    for args in [(8, 2, 256, 512, ring.start, ring.len, 300), (8, 2, 256, 512, 0, 0, 300)]:
        po.fn(shim, "gqa_attention")(P(o1), P(qa), P(ring.k), P(ring.v), *args)
        po.fn("oracle", "gqa_attention")(P(o2), P(qa), P(ring.k), P(ring.v), *args)
        assert_close(o1, o2, what=f"gqa_attention len={args[5]}")


def test_layer_loops_through_shim(shim):
    """forward_deltanet_from_proj and forward_full_attn_from_proj per token, their every cpu_ops
    call served by the GPU."""
    rng = np.random.default_rng(3)
    shape = gdn_shape(2, 4)
    proj, conv_w, A, dt_bias, norm_w = gdn_inputs(rng, shape, 6)
    C = conv_w.shape[0]
    s1 = po.DeltaState((0.1 * rng.standard_normal((4, 128, 128))).astype(np.float32),
                       rng.standard_normal((C, 3)).astype(np.float32), 1)
    s2 = s1.copy()
    got = po.deltanet_tokens(shim, shape, po.make_variant(), conv_w, A, dt_bias, norm_w, s1, proj)
    want = po.deltanet_tokens("oracle", shape, po.make_variant(), conv_w, A, dt_bias, norm_w, s2, proj)
    assert_close(got, want, what="DeltaNet layer through the shim")
    assert_close(s1.ssm, s2.ssm, what="DeltaNet state through the shim")
    np.testing.assert_array_equal(s1.conv, s2.conv)
    assert s1.conv_pos == s2.conv_pos
    fshape = fa_shape(8, 2, 256, 64, 1e7)
    fproj, qn, kn = fa_inputs(rng, fshape, 5)
    r1 = random_ring(rng, 64, 2, 256, 60, 10)
    r2 = po.KVRing(r1.k.copy(), r1.v.copy(), r1.len, r1.start)
    rope = po.rope_table(4096, 64, 1e7)
    got = po.full_attn_tokens(shim, fshape, po.make_variant(), qn, kn, r1, fproj, 900, rope)
    want = po.full_attn_tokens("oracle", fshape, po.make_variant(), qn, kn, r2, fproj, 900, rope)
    assert_close(got, want, what="attention layer through the shim")
    assert (r1.len, r1.start) == (r2.len, r2.start)
    assert_close(r1.k, r2.k, what="K ring through the shim")

"""Generates the golden fixtures in tests/golden/ from the REFERENCE itself.

Run where the reference sources are present (--ref, or ANELM_REFERENCE) and
after ``make -C oracle`` has built oracle/_ref/libref_core.so from the
reference's unmodified core/cpu_ops.cpp:

    python tests/golden/make_golden.py --ref <ANE-LM root> [--only deltanet_hf ...]

Fixtures written (seeded, numpy default_rng):

* ``cpu_ops_ref.npz``      -- each core/cpu_ops.h entry point on small inputs;
* ``full_attn_ref.npz``    -- forward_full_attn_from_proj (qwen3_5.cpp:944-1002) over
  40 tokens of a 32-slot ring (so the ring wraps), 8 q / 2 kv heads, d=256; once with
  the reference's fp32 cache and once with K/V rounded to fp16 as they are written
  (``*_f16kv``: the storage format of the GPU ring);
* ``deltanet_ref.npz``     -- forward_deltanet_from_proj (qwen3_5.cpp:849-910) over
  16 tokens, 4 value / 2 key heads, dk=dv=128, random initial state;
* ``serve_hybrid_ref.npz`` -- scripts/serve_hybrid.py:85-132 ``cpu_attention`` run from
  the reference file's own source (parsed with ast; the two Accelerate sgemm
  calls replaced by numpy matmul, the only Apple dependency of that function)
  over 12 positions at the reference's Qwen3.5-4B constants;
* ``deltanet_hf_ref.npz``  -- the decay-first (HF-order) DeltaNet layer of the hybrid v2
  export, scripts/export_hybrid_chunks.py:83-160 ``DeltaNetLayer``, run from the
  reference file's own class source (parsed with ast; coremltools, which that file
  imports at module level, is not needed by the class) over 16 tokens, 4 value / 2 key
  heads, dk=dv=128: its shift-register conv state, F.normalize of q/k, decay-first
  update and [y, -y] LayerNorm.  The layer's own input norm and in_proj are replaced by
  identities so that it consumes the projection row directly, and its out_proj by a
  module that records the core output (y_normed) and returns zeros.

The C++ glue around cpu_ops is the restatement in oracle/glue_impl.h (the
reference's qwen3_5.cpp cannot be compiled off macOS); the ops it calls are the
reference's.  Nothing on the GPU box reads the reference: these files travel.
"""
from __future__ import annotations

import argparse
import ast
import os
import sys

import numpy as np

REPO = os.path.dirname(os.path.dirname(os.path.dirname(os.path.abspath(__file__))))
sys.path.insert(0, REPO)
from oracle import pyoracle as po  # noqa: E402

OUT = os.path.dirname(os.path.abspath(__file__))


def f16(x):
    return np.asarray(x, np.float32).astype(np.float16).astype(np.float32)


def gen_cpu_ops(rng):
    L = po.lib("ref")
    P = po.P
    d = {}
    # rmsnorm / rmsnorm_gated / l2 / silu / mul_sigmoid / softmax on one 256-vector
    x = rng.standard_normal(256).astype(np.float32)
    z = rng.standard_normal(256).astype(np.float32)
    w = (1 + 0.02 * rng.standard_normal(256)).astype(np.float32)
    tmp = np.zeros(256, np.float32)
    d["x"], d["z"], d["w"] = x, z, w
    o = np.zeros(256, np.float32); L.ref_rmsnorm(P(o), P(x), P(w), 256, 1e-6); d["rmsnorm"] = o
    o = np.zeros(256, np.float32); L.ref_rmsnorm_gated(P(o), P(x), P(z), P(w), 256); d["rmsnorm_gated"] = o
    o = x.copy(); L.ref_l2_normalize(P(o), 256); d["l2_normalize"] = o
    o = x.copy(); L.ref_silu_vec_inplace(P(o), 256, P(tmp)); d["silu"] = o
    o = x.copy(); L.ref_mul_sigmoid_inplace(P(o), P(z), 256, P(tmp)); d["mul_sigmoid"] = o
    o = x.copy(); L.ref_softmax(P(o), 256); d["softmax"] = o
    W = rng.standard_normal((64, 256)).astype(np.float32)
    o = np.zeros(64, np.float32); L.ref_matvec(P(o), P(W), P(x), 64, 256)
    d["matvec_W"], d["matvec"] = W, o
    # rope (interleaved), table row and on-the-fly branch
    q = rng.standard_normal((4, 512)).astype(np.float32)
    k = rng.standard_normal((2, 256)).astype(np.float32)
    cos, sin = po.rope_table(4096, 64, 1e7)
    for tag, pos, c, s in (("table", 1234, cos[1234].copy(), sin[1234].copy()), ("fly", 5000, None, None)):
        qq, kk = q.copy(), k.copy()
        L.ref_apply_rope_cached(P(qq), P(kk), 4, 2, 256, 512, 256, 64, pos, 1e7, P(c), P(s))
        d[f"rope_{tag}_q"], d[f"rope_{tag}_k"] = qq, kk
    d["rope_q_in"], d["rope_k_in"] = q, k
    # conv1d_update over 5 steps (ring wraps)
    C = 96
    cw = (0.5 * rng.standard_normal((C, 4))).astype(np.float32)
    cs = rng.standard_normal((C, 3)).astype(np.float32)
    xs = rng.standard_normal((5, C)).astype(np.float32)
    d["conv_w"], d["conv_state0"], d["conv_x"] = cw, cs.copy(), xs
    pos = np.zeros(1, np.int32)
    ys = np.zeros((5, C), np.float32)
    for t in range(5):
        L.ref_conv1d_update(P(ys[t]), P(cs), P(pos), P(xs[t].copy()), P(cw), C, 4)
    d["conv_y"], d["conv_state"], d["conv_pos"] = ys, cs, pos
    # ssm_step
    S = (0.1 * rng.standard_normal((128, 128))).astype(np.float32)
    qv = rng.standard_normal(128).astype(np.float32); qv /= np.linalg.norm(qv)
    kv = rng.standard_normal(128).astype(np.float32); kv /= np.linalg.norm(kv)
    vv = rng.standard_normal(128).astype(np.float32)
    d["ssm_S0"], d["ssm_q"], d["ssm_k"], d["ssm_v"] = S.copy(), qv, kv, vv
    y = np.zeros(128, np.float32)
    L.ref_ssm_step(P(y), P(S), P(qv), P(kv), P(vv), 0.9, 0.3, 128, 128)
    d["ssm_y"], d["ssm_S"] = y, S
    # gqa_attention on a wrapped ring: cap 24, start 17, len 24
    cap, Hq, Hkv, hd = 24, 4, 2, 256
    kc = f16(rng.standard_normal((cap, Hkv, hd)))
    vc = f16(rng.standard_normal((cap, Hkv, hd)))
    qa = rng.standard_normal((Hq, 2 * hd)).astype(np.float32)
    d["gqa_k"], d["gqa_v"], d["gqa_q"] = kc, vc, qa
    for tag, start, ln in (("wrap", 17, 24), ("part", 5, 11), ("empty", 0, 0)):
        o = np.full((Hq, hd), 7.0, np.float32)
        L.ref_gqa_attention(P(o), P(qa), P(kc), P(vc), Hq, Hkv, hd, 2 * hd, start, ln, cap)
        d[f"gqa_{tag}"] = o
    np.savez_compressed(os.path.join(OUT, "cpu_ops_ref.npz"), **d)


def gen_full_attn(rng):
    shape = po.make_shape(num_q_heads=8, num_kv_heads=2, head_dim=256, rot_dim=64, rope_theta=1e7)
    var = po.make_variant()
    T, cap, d_ = 40, 32, 256
    proj_dim = 8 * 2 * d_ + 2 * 2 * d_
    proj = f16(rng.standard_normal((T, proj_dim)))
    q_norm = (1 + 0.02 * rng.standard_normal(d_)).astype(np.float32)
    k_norm = (1 + 0.02 * rng.standard_normal(d_)).astype(np.float32)
    cos, sin = po.rope_table(4096, 64, 1e7)
    ring = po.KVRing.empty(cap, 2, d_)
    start_pos = 4070  # crosses the 4096-row table edge -> on-the-fly RoPE branch too
    out = po.full_attn_tokens("ref", shape, var, q_norm, k_norm, ring, proj, start_pos, (cos, sin))
    # same run with the K/V written to the cache rounded to fp16 (the GPU's storage format)
    ring16 = po.KVRing.empty(cap, 2, d_)
    out16 = po.full_attn_tokens("ref", shape, po.make_variant(kv_round_f16=1), q_norm, k_norm, ring16, proj,
                                start_pos, (cos, sin))
    np.savez_compressed(os.path.join(OUT, "full_attn_ref.npz"), proj=proj.astype(np.float16),
                        q_norm=q_norm, k_norm=k_norm, start_pos=np.int32(start_pos), cap=np.int32(cap),
                        out=out, k_cache=ring.k, v_cache=ring.v, len=np.int32(ring.len),
                        start=np.int32(ring.start), out_f16kv=out16, k_cache_f16kv=ring16.k,
                        v_cache_f16kv=ring16.v)


def gen_deltanet(rng):
    Hv, Hk, dk, dv = 4, 2, 128, 128
    shape = po.make_shape(lin_num_key_heads=Hk, lin_num_val_heads=Hv, lin_key_dim=dk, lin_val_dim=dv)
    var = po.make_variant()
    C = 2 * Hk * dk + Hv * dv
    T = 16
    proj_dim = C + Hv * dv + 2 * Hv
    proj = f16(rng.standard_normal((T, proj_dim)))
    conv_w = f16(0.5 * rng.standard_normal((C, 4)))
    A = np.exp(0.3 * rng.standard_normal(Hv)).astype(np.float32)
    dt_bias = (0.5 * rng.standard_normal(Hv)).astype(np.float32)
    norm_w = (1 + 0.1 * rng.standard_normal(dv)).astype(np.float32)
    st = po.DeltaState((0.1 * rng.standard_normal((Hv, dk, dv))).astype(np.float32),
                       rng.standard_normal((C, 3)).astype(np.float32), 1)
    s0 = st.copy()
    out = po.deltanet_tokens("ref", shape, var, conv_w, A, dt_bias, norm_w, st, proj)
    np.savez_compressed(os.path.join(OUT, "deltanet_ref.npz"), proj=proj.astype(np.float16),
                        conv_w=conv_w, A=A, dt_bias=dt_bias, norm_w=norm_w,
                        ssm0=s0.ssm, conv0=s0.conv, conv_pos0=np.int32(s0.conv_pos),
                        out=out, ssm=st.ssm, conv=st.conv, conv_pos=np.int32(st.conv_pos))


def load_reference_cpu_attention(ref_root):
    """Executes the reference's own serve_hybrid.py constants and cpu_attention body.

    Only module-level assignments to the listed constants and the two function
    definitions are taken from the file; ``_cblas_sgemm`` (Accelerate) is replaced
    by a numpy stand-in with the same row-major CBLAS contract."""
    path = os.path.join(ref_root, "scripts", "serve_hybrid.py")
    tree = ast.parse(open(path).read(), path)
    keep_names = {"HIDDEN", "NUM_HEADS", "NUM_KV_HEADS", "HEAD_DIM", "GROUPS", "ROPE_DIM", "HALF_ROT",
                  "ATTN_DIM", "CONTEXT", "ROPE_THETA", "_inv_freq", "_positions", "_freqs", "ROPE_COS",
                  "ROPE_SIN", "CblasRowMajor", "CblasNoTrans", "CblasTrans"}
    body = []
    for node in tree.body:
        if isinstance(node, ast.Assign) and all(isinstance(t, ast.Name) and t.id in keep_names
                                                for t in node.targets):
            body.append(node)
        elif isinstance(node, ast.FunctionDef) and node.name in ("sgemm", "cpu_attention"):
            body.append(node)
    mod = ast.Module(body=body, type_ignores=[])
    import ctypes
    import math

    def fake_sgemm(order, ta, tb, M, N, K, alpha, A, lda, B, ldb, beta, C, ldc):
        a = np.ctypeslib.as_array(A, shape=(M, lda))[:, :K]
        if tb == 112:
            b = np.ctypeslib.as_array(B, shape=(N, ldb))[:, :K].T
        else:
            b = np.ctypeslib.as_array(B, shape=(K, ldb))[:, :N]
        c = np.ctypeslib.as_array(C, shape=(M, ldc))
        c[:, :N] = alpha.value * (a @ b) + (beta.value * c[:, :N] if beta.value != 0 else 0)

    g = {"np": np, "math": math, "ctypes": ctypes, "_cblas_sgemm": fake_sgemm}
    exec(compile(mod, path, "exec"), g)
    return g


def gen_serve_hybrid(rng, ref_root):
    g = load_reference_cpu_attention(ref_root)
    H, KVH, HD, CTX = g["NUM_HEADS"], g["NUM_KV_HEADS"], g["HEAD_DIM"], g["CONTEXT"]
    T = 12
    kv = [(np.zeros((KVH, CTX, HD), np.float32), np.zeros((KVH, CTX, HD), np.float32))]
    qg = rng.standard_normal((T, H, 2 * HD)).astype(np.float16)
    k = rng.standard_normal((T, KVH, HD)).astype(np.float16)
    v = rng.standard_normal((T, KVH, HD)).astype(np.float16)
    outs = [g["cpu_attention"](qg[t], k[t], v[t], t, kv, 0) for t in range(T)]
    np.savez_compressed(os.path.join(OUT, "serve_hybrid_ref.npz"), q_gate=qg, k=k, v=v,
                        out=np.concatenate(outs, 0),
                        consts=np.array([H, KVH, HD, g["ROPE_DIM"], CTX], np.int32),
                        rope_theta=np.float32(g["ROPE_THETA"]))


def load_reference_deltanet_layer(ref_root):
    """Executes the reference's RMSNorm, SwiGLUFFN and DeltaNetLayer class definitions from
    scripts/export_hybrid_chunks.py (nothing else of that file) and returns DeltaNetLayer."""
    import torch
    import torch.nn as nn
    import torch.nn.functional as F

    path = os.path.join(ref_root, "scripts", "export_hybrid_chunks.py")
    tree = ast.parse(open(path).read(), path)
    body = [n for n in tree.body if isinstance(n, ast.ClassDef) and n.name in ("RMSNorm", "SwiGLUFFN",
                                                                              "DeltaNetLayer")]
    assert len(body) == 3, "expected RMSNorm, SwiGLUFFN and DeltaNetLayer in export_hybrid_chunks.py"
    g = {"torch": torch, "nn": nn, "F": F, "math": __import__("math")}
    exec(compile(ast.Module(body=body, type_ignores=[]), path, "exec"), g)
    return g["DeltaNetLayer"]


def gen_deltanet_hf(rng, ref_root):
    import torch
    import torch.nn as nn

    Layer = load_reference_deltanet_layer(ref_root)
    Hv, Hk, dk, dv, K, T = 4, 2, 128, 128, 4, 16
    C = 2 * Hk * dk + Hv * dv
    proj_dim = C + Hv * dv + 2 * Hv
    proj = f16(rng.standard_normal((T, proj_dim)))
    conv_w = f16(0.5 * rng.standard_normal((C, K)))
    A_log = (0.3 * rng.standard_normal(Hv)).astype(np.float32)
    dt_bias = (0.5 * rng.standard_normal(Hv)).astype(np.float32)
    norm_w = (1 + 0.1 * rng.standard_normal(dv)).astype(np.float32)
    shift0 = rng.standard_normal((C, K)).astype(np.float32)
    ssm0 = (0.1 * rng.standard_normal((Hv, dk, dv))).astype(np.float32)

    layer = Layer(hidden_size=proj_dim, intermediate_size=8, lin_qkv_dim=C, lin_total_val=Hv * dv,
                  lin_num_val_heads=Hv, lin_key_dim=dk, lin_val_dim=dv, lin_num_key_heads=Hk, conv_kernel=K)
    captured = []

    class Capture(nn.Module):  # stands in for out_proj: keeps the core output, adds nothing
        def forward(self, x):
            captured.append(x.detach().clone())
            return torch.zeros(x.shape[0], proj_dim)

    layer.input_layernorm = nn.Identity()
    layer.in_proj = nn.Identity()
    layer.out_proj = Capture()
    with torch.no_grad():
        layer.conv_weight.copy_(torch.from_numpy(conv_w))
        layer.A_log.copy_(torch.from_numpy(A_log))
        layer.dt_bias.copy_(torch.from_numpy(dt_bias))
        layer.norm_weight.copy_(torch.from_numpy(norm_w))
        conv, ssm = torch.from_numpy(shift0), torch.from_numpy(ssm0)
        for t in range(T):
            _, conv, ssm = layer(torch.from_numpy(proj[t:t + 1]), conv, ssm)
    out = torch.cat(captured, 0).numpy()
    assert out.shape == (T, Hv * dv)
    np.savez_compressed(os.path.join(OUT, "deltanet_hf_ref.npz"), proj=proj.astype(np.float16), conv_w=conv_w,
                        A=np.exp(A_log).astype(np.float32), A_log=A_log, dt_bias=dt_bias, norm_w=norm_w,
                        shift0=shift0, ssm0=ssm0, out=out, ssm=ssm.numpy(), shift=conv.numpy(),
                        dims=np.array([Hk, Hv, dk, dv, K], np.int32))


GENERATORS = ("cpu_ops", "full_attn", "deltanet", "serve_hybrid", "deltanet_hf")


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--ref", default=os.environ.get("ANELM_REFERENCE"),
                    help="root of the ANE-LM sources (or set ANELM_REFERENCE)")
    ap.add_argument("--only", nargs="*", choices=GENERATORS, help="regenerate only these fixtures")
    a = ap.parse_args()
    if not a.ref or not os.path.isdir(a.ref):
        sys.exit("give the ANE-LM source root with --ref or ANELM_REFERENCE")
    only = set(a.only or GENERATORS)
    if not po.available("ref") and only & {"cpu_ops", "full_attn", "deltanet"}:
        sys.exit("oracle/_ref/libref_core.so missing: run make -C oracle REF=<ANE-LM root>")
    if "cpu_ops" in only:
        gen_cpu_ops(np.random.default_rng(0))
    if "full_attn" in only:
        gen_full_attn(np.random.default_rng(1))
    if "deltanet" in only:
        gen_deltanet(np.random.default_rng(2))
    if "serve_hybrid" in only:
        gen_serve_hybrid(np.random.default_rng(3), a.ref)
    if "deltanet_hf" in only:
        gen_deltanet_hf(np.random.default_rng(4), a.ref)
    for f in sorted(os.listdir(OUT)):
        if f.endswith(".npz"):
            print(f, os.path.getsize(os.path.join(OUT, f)))


if __name__ == "__main__":
    main()

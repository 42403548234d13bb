"""Shared helpers for the parity tests: seeded inputs in the reference's layouts
and oracle runs (oracle/ is the checker, never the thing under test)."""
from __future__ import annotations

import numpy as np

from oracle import pyoracle as po

# Tolerance of the parity contract: fp32 accumulate from fp16/bf16 inputs.
ATOL, RTOL = 2e-3, 1e-2


def assert_close(got, want, atol=ATOL, rtol=RTOL, what=""):
    got = np.asarray(got, np.float32)
    want = np.asarray(want, np.float32)
    assert got.shape == want.shape, (what, got.shape, want.shape)
    err = np.abs(got - want)
    bad = err > atol + rtol * np.abs(want)
    if bad.any():
        i = np.unravel_index(np.argmax(err - (atol + rtol * np.abs(want))), err.shape)
        raise AssertionError(f"{what}: {bad.sum()} / {bad.size} outside atol={atol} rtol={rtol}; "
                             f"max abs err {err.max():.3e} at {i}: got {got[i]:.6f} want {want[i]:.6f}")


def f16(x):
    return np.asarray(x, np.float32).astype(np.float16).astype(np.float32)


def fa_shape(Hq=8, Hkv=2, d=256, R=64, theta=1e7):
    return po.make_shape(num_q_heads=Hq, num_kv_heads=Hkv, head_dim=d, rot_dim=R, rope_theta=theta)


def gdn_shape(Hk=16, Hv=16, dk=128, dv=128):
    return po.make_shape(lin_num_key_heads=Hk, lin_num_val_heads=Hv, lin_key_dim=dk, lin_val_dim=dv)


def fa_inputs(rng, shape, T):
    """q/k/v/gate fp16 N(0,1) projections, QK-norm weights N(1, 0.02)."""
    d = shape.head_dim
    proj_dim = shape.num_q_heads * 2 * d + 2 * shape.num_kv_heads * d
    proj = f16(rng.standard_normal((T, proj_dim)))
    qn = (1 + 0.02 * rng.standard_normal(d)).astype(np.float32)
    kn = (1 + 0.02 * rng.standard_normal(d)).astype(np.float32)
    return proj, qn, kn


def gdn_inputs(rng, shape, T):
    """DeltaNet projections and weights: conv w fp16 N(0,0.5); a, b N(0,1) so that
    g = exp(-softplus(a)) and beta = sigmoid(b) with A = 1, dt_bias = 0."""
    Hv, dv = shape.lin_num_val_heads, shape.lin_val_dim
    C = 2 * shape.lin_num_key_heads * shape.lin_key_dim + Hv * dv
    proj = f16(rng.standard_normal((T, C + Hv * dv + 2 * Hv)))
    conv_w = f16(0.5 * rng.standard_normal((C, 4)))
    A = np.ones(Hv, np.float32)
    dt_bias = np.zeros(Hv, np.float32)
    norm_w = (1 + 0.1 * rng.standard_normal(dv)).astype(np.float32)
    return proj, conv_w, A, dt_bias, norm_w


def random_ring(rng, cap, Hkv, d, length, start):
    """A KV ring holding `length` fp16-representable N(0,1) rows starting at slot `start`."""
    ring = po.KVRing.empty(cap, Hkv, d)
    ring.k[:] = f16(rng.standard_normal(ring.k.shape))
    ring.v[:] = f16(rng.standard_normal(ring.v.shape))
    ring.len, ring.start = length, start
    return ring

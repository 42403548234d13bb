"""anelm oracle, Python side -- TEST INFRASTRUCTURE ONLY.

ctypes bindings for the CPU oracle libraries built by ``oracle/Makefile``:

* ``liboracle.so``          -- the plain-C restatement of core/cpu_ops.cpp and of the
  layer glue in models/llm/qwen3_5.cpp:849-1002;
* ``_ref/libref_core.so``   -- the reference's own core/cpu_ops.cpp compiled here
  (unmodified) under the same glue; present only where the reference sources were;
* ``_ref/libref_core_fast.so`` -- the same reference sources built for speed (the
  timed CPU baseline).

Only tests/, __graft_entry__.smoke() and bench.py's CPU-baseline / reference leg
may import this module.  The product library never does.
"""
from __future__ import annotations

import ctypes
import os
from dataclasses import dataclass

import numpy as np

HERE = os.path.dirname(os.path.abspath(__file__))
LIBS = {
    "oracle": os.path.join(HERE, "liboracle.so"),
    "ref": os.path.join(HERE, "_ref", "libref_core.so"),
    "ref_fast": os.path.join(HERE, "_ref", "libref_core_fast.so"),
}
PREFIX = {"oracle": "orc_", "ref": "ref_", "ref_fast": "ref_"}

_fp = ctypes.POINTER(ctypes.c_float)
_ip = ctypes.POINTER(ctypes.c_int)


class Shape(ctypes.Structure):
    """orc_shape (oracle/anelm_oracle.h); fields follow Qwen35Args, models/llm/qwen3_5.h:51-80."""

    _fields_ = [
        ("num_q_heads", ctypes.c_int), ("num_kv_heads", ctypes.c_int),
        ("head_dim", ctypes.c_int), ("rot_dim", ctypes.c_int),
        ("rope_theta", ctypes.c_float), ("rms_eps", ctypes.c_float),
        ("attn_output_gate", ctypes.c_int),
        ("lin_num_key_heads", ctypes.c_int), ("lin_num_val_heads", ctypes.c_int),
        ("lin_key_dim", ctypes.c_int), ("lin_val_dim", ctypes.c_int),
        ("conv_kernel", ctypes.c_int),
    ]


class Variant(ctypes.Structure):
    """orc_variant: all zero = the C++ cpu_ops path."""

    _fields_ = [
        ("rope_half", ctypes.c_int), ("no_qk_norm", ctypes.c_int),
        ("kv_linear", ctypes.c_int), ("kv_round_f16", ctypes.c_int),
        ("delta_hf", ctypes.c_int), ("l2_eps", ctypes.c_float),
    ]


def make_shape(num_q_heads=8, num_kv_heads=2, head_dim=256, rot_dim=64, rope_theta=1e7,
               rms_eps=1e-6, attn_output_gate=1, lin_num_key_heads=16, lin_num_val_heads=16,
               lin_key_dim=128, lin_val_dim=128, conv_kernel=4) -> Shape:
    return Shape(num_q_heads, num_kv_heads, head_dim, rot_dim, rope_theta, rms_eps,
                 attn_output_gate, lin_num_key_heads, lin_num_val_heads, lin_key_dim,
                 lin_val_dim, conv_kernel)


def make_variant(rope_half=0, no_qk_norm=0, kv_linear=0, kv_round_f16=0, delta_hf=0,
                 l2_eps=0.0) -> Variant:
    return Variant(rope_half, no_qk_norm, kv_linear, kv_round_f16, delta_hf, l2_eps)


def available(kind: str) -> bool:
    return os.path.exists(LIBS[kind])


_cache: dict[str, ctypes.CDLL] = {}


def lib(kind: str = "oracle") -> ctypes.CDLL:
    if kind in _cache:
        return _cache[kind]
    path = LIBS[kind]
    if not os.path.exists(path):
        raise FileNotFoundError(f"oracle library {path} not built (run make -C oracle)")
    L = ctypes.CDLL(path)
    p = PREFIX[kind]
    sp, vp = ctypes.POINTER(Shape), ctypes.POINTER(Variant)
    sig = {
        "full_attn_from_proj": (ctypes.c_int, [sp, vp, _fp, _fp, _fp, _fp, _ip, _ip, ctypes.c_int,
                                               _fp, _fp, ctypes.c_int, _fp, ctypes.c_int, _fp, _fp]),
        "deltanet_from_proj": (ctypes.c_int, [sp, vp, _fp, _fp, _fp, _fp, _fp, _fp, _ip, _fp, _fp, _fp]),
        "deltanet_tokens": (ctypes.c_int, [sp, vp, _fp, _fp, _fp, _fp, _fp, _fp, _ip, _fp,
                                           ctypes.c_int, _fp]),
        "full_attn_tokens": (ctypes.c_int, [sp, vp, _fp, _fp, _fp, _fp, _ip, _ip, ctypes.c_int,
                                            _fp, _fp, ctypes.c_int, _fp, ctypes.c_int, ctypes.c_int, _fp]),
        "silu_vec_inplace": (None, [_fp, ctypes.c_int, _fp]),
        "mul_sigmoid_inplace": (None, [_fp, _fp, ctypes.c_int, _fp]),
        "rmsnorm": (None, [_fp, _fp, _fp, ctypes.c_int, ctypes.c_float]),
        "rmsnorm_gated": (None, [_fp, _fp, _fp, _fp, ctypes.c_int]),
        "apply_rope_cached": (None, [_fp, _fp] + [ctypes.c_int] * 7 + [ctypes.c_float, _fp, _fp]),
        "softmax": (None, [_fp, ctypes.c_int]),
        "matvec": (None, [_fp, _fp, _fp, ctypes.c_int, ctypes.c_int]),
        "l2_normalize": (None, [_fp, ctypes.c_int]),
        "conv1d_update": (None, [_fp, _fp, _ip, _fp, _fp, ctypes.c_int, ctypes.c_int]),
        "ssm_step": (None, [_fp, _fp, _fp, _fp, _fp, ctypes.c_float, ctypes.c_float,
                            ctypes.c_int, ctypes.c_int]),
        "gqa_attention": (None, [_fp, _fp, _fp, _fp] + [ctypes.c_int] * 7),
    }
    for name, (res, args) in sig.items():
        f = getattr(L, p + name)
        f.restype = res
        f.argtypes = args
    if kind == "oracle":
        f = L.orc_rope_table
        f.restype = None
        f.argtypes = [_fp, _fp, ctypes.c_int, ctypes.c_int, ctypes.c_float]
    _cache[kind] = L
    return L


def fn(kind: str, name: str):
    return getattr(lib(kind), PREFIX[kind] + name)


def P(a: np.ndarray | None):
    """float32 / int32 C-contiguous numpy array -> ctypes pointer (None -> NULL)."""
    if a is None:
        return None
    assert a.flags["C_CONTIGUOUS"], "oracle arrays must be C-contiguous"
    if a.dtype == np.float32:
        return a.ctypes.data_as(_fp)
    if a.dtype == np.int32:
        return a.ctypes.data_as(_ip)
    raise TypeError(a.dtype)


def rope_table(n_pos: int, rot_dim: int, theta: float):
    """qwen3_5.cpp:309-324 cos/sin table [n_pos][rot_dim/2]."""
    c = np.zeros((n_pos, rot_dim // 2), np.float32)
    s = np.zeros((n_pos, rot_dim // 2), np.float32)
    lib("oracle").orc_rope_table(P(c), P(s), n_pos, rot_dim, theta)
    return c, s


@dataclass
class KVRing:
    """KVCache of models/llm/qwen3_5.h:165-171: slot-major [capacity][Hkv][d] fp32."""

    k: np.ndarray
    v: np.ndarray
    len: int = 0
    start: int = 0

    @classmethod
    def empty(cls, capacity: int, n_kv_heads: int, head_dim: int):
        z = np.zeros((capacity, n_kv_heads, head_dim), np.float32)
        return cls(z.copy(), z.copy())

    @property
    def capacity(self) -> int:
        return self.k.shape[0]


@dataclass
class DeltaState:
    """DeltaNetState of models/llm/qwen3_5.h:158-162."""

    ssm: np.ndarray    # [Hv][dk][dv] fp32
    conv: np.ndarray   # [C][K-1] fp32
    conv_pos: int = 0

    @classmethod
    def zeros(cls, shape: Shape):
        C = 2 * shape.lin_num_key_heads * shape.lin_key_dim + shape.lin_num_val_heads * shape.lin_val_dim
        return cls(np.zeros((shape.lin_num_val_heads, shape.lin_key_dim, shape.lin_val_dim), np.float32),
                   np.zeros((C, shape.conv_kernel - 1), np.float32), 0)

    def copy(self):
        return DeltaState(self.ssm.copy(), self.conv.copy(), self.conv_pos)


def full_attn_tokens(kind: str, shape: Shape, var: Variant, q_norm, k_norm, ring: KVRing,
                     proj: np.ndarray, start_pos: int, rope=None):
    """Runs len(proj) successive full-attention core steps; updates ring in place."""
    proj = np.ascontiguousarray(proj, np.float32).reshape(-1, proj.shape[-1])
    n = proj.shape[0]
    out = np.zeros((n, shape.num_q_heads * shape.head_dim), np.float32)
    ln, st = ctypes.c_int(ring.len), ctypes.c_int(ring.start)
    cos, sin = rope if rope is not None else (None, None)
    tl = 0 if cos is None else cos.shape[0]
    rc = fn(kind, "full_attn_tokens")(ctypes.byref(shape), ctypes.byref(var), P(q_norm), P(k_norm),
                                      P(ring.k), P(ring.v), ctypes.byref(ln), ctypes.byref(st),
                                      ring.capacity, P(cos), P(sin), tl, P(proj), start_pos, n, P(out))
    if rc != 0:
        raise RuntimeError(f"oracle full_attn_tokens failed rc={rc}")
    ring.len, ring.start = ln.value, st.value
    return out


def gated_delta_tokens(kind: str, q, k, v, log_decay, beta, state, delta_hf: int = 0):
    """The bare delta-rule recurrence over T tokens: q, k [T][Hk][dk], v [T][Hv][dv], log_decay,
    beta [T][Hv]; state [Hv][dk][dv] float32, updated in place.  Returns y [T][Hv][dv]."""
    q, k, v = (np.ascontiguousarray(a, np.float32) for a in (q, k, v))
    log_decay, beta = np.ascontiguousarray(log_decay, np.float32), np.ascontiguousarray(beta, np.float32)
    T, Hk, dk = q.shape
    Hv, dv = v.shape[1], v.shape[2]
    assert state.dtype == np.float32 and state.flags["C_CONTIGUOUS"] and state.shape == (Hv, dk, dv)
    y = np.zeros((T, Hv, dv), np.float32)
    rc = fn(kind, "gated_delta_tokens")(T, Hk, Hv, dk, dv, int(delta_hf), P(q), P(k), P(v), P(log_decay),
                                        P(beta), P(state), P(y))
    if rc != 0:
        raise RuntimeError(f"oracle gated_delta_tokens failed rc={rc}")
    return y


def deltanet_tokens(kind: str, shape: Shape, var: Variant, conv_w, A, dt_bias, norm_w,
                    state: DeltaState, proj: np.ndarray):
    """Runs len(proj) successive DeltaNet core steps; updates state in place."""
    proj = np.ascontiguousarray(proj, np.float32).reshape(-1, proj.shape[-1])
    n = proj.shape[0]
    out = np.zeros((n, shape.lin_num_val_heads * shape.lin_val_dim), np.float32)
    cp = ctypes.c_int(state.conv_pos)
    rc = fn(kind, "deltanet_tokens")(ctypes.byref(shape), ctypes.byref(var), P(conv_w), P(A),
                                     P(dt_bias), P(norm_w), P(state.ssm), P(state.conv),
                                     ctypes.byref(cp), P(proj), n, P(out))
    if rc != 0:
        raise RuntimeError(f"oracle deltanet_tokens failed rc={rc}")
    state.conv_pos = cp.value
    return out

"""Drop-in for scripts/serve_hybrid.py's CPU attention (serve_hybrid.py:85-132).

    from anelm_b200.serve_hybrid import CudaAttention
    attn = CudaAttention()                 # Qwen3.5-4B constants, serve_hybrid.py:32-55
    kv_caches = attn.new_kv_caches()       # replaces the numpy caches of _reset_state (228-236)
    out = attn.cpu_attention(q_gate_fp16, k_fp16, v_fp16, pos, kv_caches, layer_idx)

`cpu_attention` keeps the reference signature and return value (fp16 [1, Hq*d]).
The KV cache lives on the GPU inside the library context; `kv_caches` is a
handle naming the sequence slot.  The math is the reference's: rotate-half RoPE
on the first 64 dims, linear KV write at `pos`, GQA softmax attention over
[0, pos], sigmoid gate.  There is no CPU fallback.
"""
from __future__ import annotations

import ctypes

import numpy as np

from . import _lib
from .core import Context
from ._lib import check, lib


class KVHandle:
    """Stands in for the per-layer (k_cache, v_cache) list of serve_hybrid.py:232-235."""

    def __init__(self, owner: "CudaAttention", seq: int):
        self.owner = owner
        self.seq = seq

    def __getitem__(self, layer_idx):
        return (self, layer_idx)


class CudaAttention:
    def __init__(self, n_layers=8, num_heads=16, num_kv_heads=4, head_dim=256, rope_dim=64, context=4096,
                 rope_theta=10000000.0, max_seqs=1, device=0):
        self.num_heads, self.num_kv_heads, self.head_dim = num_heads, num_kv_heads, head_dim
        self.context = context
        self.ctx = Context(device=device, layer_types=[_lib.LAYER_FULL_ATTN] * n_layers,
                           num_q_heads=num_heads, num_kv_heads=num_kv_heads, head_dim=head_dim, rot_dim=rope_dim,
                           rope_theta=rope_theta, attn_output_gate=1, max_seqs=max_seqs, kv_capacity=context,
                           rope_table_len=context, rope_mode=_lib.ROPE_HALF, qk_norm_in_core=0,
                           kv_mode=_lib.KV_LINEAR)
        self._free = list(range(max_seqs))
        self._out = np.empty(num_heads * head_dim, np.float16)

    def new_kv_caches(self) -> KVHandle:
        """serve_hybrid.py:228-236 (_reset_state): a zeroed cache for one generation."""
        if not self._free:
            raise RuntimeError("no free sequence slot; create CudaAttention(max_seqs=...)")
        seq = self._free.pop(0)
        self.ctx.reset(seq)
        return KVHandle(self, seq)

    def release(self, kv: KVHandle):
        self._free.append(kv.seq)

    def cpu_attention(self, q_gate_fp16, k_fp16, v_fp16, pos, kv_caches, layer_idx):
        q = np.ascontiguousarray(q_gate_fp16, np.float16).reshape(-1)
        k = np.ascontiguousarray(k_fp16, np.float16).reshape(-1)
        v = np.ascontiguousarray(v_fp16, np.float16).reshape(-1)
        H, KV, D = self.num_heads, self.num_kv_heads, self.head_dim
        if q.size != H * 2 * D or k.size != KV * D or v.size != KV * D:
            raise ValueError("q_gate / k / v sizes do not match the configured heads")
        seq = kv_caches.seq if isinstance(kv_caches, KVHandle) else int(kv_caches)
        out = np.empty(H * D, np.float16)
        check(lib().anelm_py_cpu_attention(self.ctx.handle, int(layer_idx), seq, ctypes.c_void_p(q.ctypes.data),
                                           ctypes.c_void_p(k.ctypes.data), ctypes.c_void_p(v.ctypes.data),
                                           int(pos), ctypes.c_void_p(out.ctypes.data), None),
              "anelm_py_cpu_attention")
        return out.reshape(1, H * D)

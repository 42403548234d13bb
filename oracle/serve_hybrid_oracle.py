"""numpy restatement of scripts/serve_hybrid.py:85-132 (``cpu_attention``) --
TEST INFRASTRUCTURE ONLY.

The reference module cannot be imported here (it loads coremltools and Apple's
Accelerate at import time, serve_hybrid.py:22, 58), so its CPU attention is
restated with numpy matmuls standing in for the two ``cblas_sgemm`` calls
(serve_hybrid.py:65-82, 119, 127).  tests/golden/make_golden.py runs the
reference's own function body (with the same stand-in) to pin this restatement.

Shapes follow the reference's hard-coded Qwen3.5-4B constants
(serve_hybrid.py:32-55) but are parameters here.
"""
from __future__ import annotations

import math

import numpy as np


class HybridAttnConfig:
    """serve_hybrid.py:32-55."""

    def __init__(self, num_heads=16, num_kv_heads=4, head_dim=256, rope_dim=64, context=4096,
                 rope_theta=10000000.0):
        self.num_heads = num_heads
        self.num_kv_heads = num_kv_heads
        self.head_dim = head_dim
        self.groups = num_heads // num_kv_heads
        self.rope_dim = rope_dim
        self.half_rot = rope_dim // 2
        self.context = context
        self.rope_theta = rope_theta
        # serve_hybrid.py:51-55 (float32 table built by numpy)
        inv_freq = 1.0 / (rope_theta ** (np.arange(0, rope_dim, 2, dtype=np.float32) / rope_dim))
        positions = np.arange(context, dtype=np.float32)
        freqs = np.outer(positions, inv_freq)
        self.rope_cos = np.cos(freqs).astype(np.float32)
        self.rope_sin = np.sin(freqs).astype(np.float32)

    def new_kv_caches(self, n_layers):
        """serve_hybrid.py:232-235: per layer (k, v) [Hkv][context][d] fp32."""
        return [(np.zeros((self.num_kv_heads, self.context, self.head_dim), np.float32),
                 np.zeros((self.num_kv_heads, self.context, self.head_dim), np.float32))
                for _ in range(n_layers)]


def cpu_attention(cfg: HybridAttnConfig, q_gate_fp16, k_fp16, v_fp16, pos, kv_caches, layer_idx):
    """serve_hybrid.py:85-132."""
    HD, HR, RD = cfg.head_dim, cfg.half_rot, cfg.rope_dim
    k_cache, v_cache = kv_caches[layer_idx]
    q_gate = np.asarray(q_gate_fp16).reshape(cfg.num_heads, 2 * HD).astype(np.float32)
    k = np.asarray(k_fp16).reshape(cfg.num_kv_heads, HD).astype(np.float32)
    v = np.asarray(v_fp16).reshape(cfg.num_kv_heads, HD).astype(np.float32)
    q = q_gate[:, :HD]
    gate = q_gate[:, HD:]
    cos = cfg.rope_cos[pos]
    sin = cfg.rope_sin[pos]
    q1 = q[:, :HR].copy()
    q2 = q[:, HR:RD].copy()
    q[:, :HR] = q1 * cos - q2 * sin
    q[:, HR:RD] = q2 * cos + q1 * sin
    k1 = k[:, :HR].copy()
    k2 = k[:, HR:RD].copy()
    k[:, :HR] = k1 * cos - k2 * sin
    k[:, HR:RD] = k2 * cos + k1 * sin
    k_cache[:, pos, :] = k
    v_cache[:, pos, :] = v
    seq_len = pos + 1
    scale = 1.0 / math.sqrt(HD)
    attn_out = np.empty((cfg.num_heads, HD), np.float32)
    G = cfg.groups
    for g in range(cfg.num_kv_heads):
        q_block = q[g * G:(g + 1) * G]
        k_block = k_cache[g, :seq_len, :]
        v_block = v_cache[g, :seq_len, :]
        scores = (q_block @ k_block.T).astype(np.float32)
        scores *= np.float32(scale)
        scores -= scores.max(axis=-1, keepdims=True)
        exp_scores = np.exp(scores)
        w = exp_scores / exp_scores.sum(axis=-1, keepdims=True)
        attn_out[g * G:(g + 1) * G] = w @ v_block
    sigmoid_gate = 1.0 / (1.0 + np.exp(-gate))
    attn_out *= sigmoid_gate
    return attn_out.astype(np.float16).reshape(1, cfg.num_heads * HD)

"""Python host mirror of the anelm_b200 context API over torch device tensors.

`Context` wraps an anelm_ctx: the device-resident KV rings and DeltaNet states
that models/llm/qwen3_5.{h,cpp} keeps per layer (KVCache / DeltaNetState,
qwen3_5.h:158-171), plus the glue entry points

    Context.full_attn_from_proj  <->  Qwen35Model::forward_full_attn_from_proj (qwen3_5.cpp:944)
    Context.deltanet_from_proj   <->  Qwen35Model::forward_deltanet_from_proj  (qwen3_5.cpp:849)

and their batched (ragged) serving forms through a `Plan`.  Tensors are torch
CUDA tensors; calls are asynchronous on torch's current stream.
"""
from __future__ import annotations

import ctypes

import numpy as np
import torch

from . import _lib
from ._lib import check, lib

_DT = {torch.float32: _lib.F32, torch.float16: _lib.F16, torch.bfloat16: _lib.BF16}


def _dtype_code(t: torch.Tensor) -> int:
    try:
        return _DT[t.dtype]
    except KeyError:
        raise TypeError(f"unsupported dtype {t.dtype}") from None


def _stream(device) -> ctypes.c_void_p:
    return ctypes.c_void_p(torch.cuda.current_stream(device).cuda_stream)


def _fp(a: np.ndarray) -> ctypes.c_void_p:
    assert a.dtype == np.float32 and a.flags["C_CONTIGUOUS"]
    return ctypes.c_void_p(a.ctypes.data)


class Plan:
    """A fixed batch of sequence ids for batched decode (anelm_plan)."""

    def __init__(self, ctx: "Context", seq_ids):
        self.ctx = ctx
        self.seq_ids = [int(s) for s in seq_ids]
        arr = (ctypes.c_int * len(self.seq_ids))(*self.seq_ids)
        h = ctypes.c_void_p()
        check(lib().anelm_plan_create(ctx.handle, len(self.seq_ids), arr, ctypes.byref(h)), "anelm_plan_create")
        self.handle = h

    @property
    def n(self) -> int:
        return len(self.seq_ids)

    def info(self):
        ch, nb = ctypes.c_int(), ctypes.c_int()
        check(lib().anelm_plan_info(self.handle, ctypes.byref(ch), ctypes.byref(nb)), "anelm_plan_info")
        return ch.value, nb.value

    def close(self):
        if self.handle:
            lib().anelm_plan_destroy(self.handle)
            self.handle = None

    def __del__(self):
        try:
            self.close()
        except Exception:
            pass


class Context:
    """anelm_ctx: device KV rings + DeltaNet state for up to max_seqs sequences."""

    def __init__(self, device: int = 0, layer_types=None, seq_kv_capacity=None, **fields):
        L = lib()
        cfg = _lib.Config()
        check(L.anelm_config_default(ctypes.byref(cfg)), "anelm_config_default")
        for k, v in fields.items():
            if not hasattr(cfg, k):
                raise TypeError(f"unknown config field {k}")
            setattr(cfg, k, v)
        self._keep = []
        if layer_types is not None:
            lt = (ctypes.c_int * len(layer_types))(*[int(x) for x in layer_types])
            cfg.num_layers = len(layer_types)
            cfg.layer_types = ctypes.cast(lt, ctypes.POINTER(ctypes.c_int))
            self._keep.append(lt)
        if seq_kv_capacity is not None:
            caps = (ctypes.c_int * len(seq_kv_capacity))(*[int(x) for x in seq_kv_capacity])
            cfg.max_seqs = len(seq_kv_capacity)
            cfg.seq_kv_capacity = ctypes.cast(caps, ctypes.POINTER(ctypes.c_int))
            self._keep.append(caps)
            self.capacities = [int(x) for x in seq_kv_capacity]
        else:
            self.capacities = [cfg.kv_capacity] * cfg.max_seqs
        self.cfg = cfg
        self.device = device
        h = ctypes.c_void_p()
        check(L.anelm_create(ctypes.byref(cfg), device, ctypes.byref(h)), "anelm_create")
        self.handle = h
        if layer_types is None:
            iv = cfg.full_attention_interval or 4
            layer_types = [_lib.LAYER_FULL_ATTN if (l + 1) % iv == 0 else _lib.LAYER_LINEAR_ATTN
                           for l in range(cfg.num_layers)]
        self.layer_types = list(layer_types)
        c = cfg
        self.conv_channels = 2 * c.lin_num_key_heads * c.lin_key_dim + c.lin_num_val_heads * c.lin_val_dim
        self.gdn_proj_dim = self.conv_channels + c.lin_num_val_heads * c.lin_val_dim + 2 * c.lin_num_val_heads
        self.gdn_out_dim = c.lin_num_val_heads * c.lin_val_dim
        self.fa_proj_dim = c.num_q_heads * 2 * c.head_dim + 2 * c.num_kv_heads * c.head_dim
        self.fa_out_dim = c.num_q_heads * c.head_dim

    # ---- lifetime ----
    def close(self):
        if getattr(self, "handle", None):
            lib().anelm_destroy(self.handle)
            self.handle = None

    def __del__(self):
        try:
            self.close()
        except Exception:
            pass

    def __enter__(self):
        return self

    def __exit__(self, *a):
        self.close()

    # ---- weights / state ----
    def set_full_attn_weights(self, layer: int, q_norm, k_norm):
        q = np.ascontiguousarray(q_norm, np.float32)
        k = np.ascontiguousarray(k_norm, np.float32)
        check(lib().anelm_set_full_attn_weights(self.handle, layer, _fp(q), _fp(k)), "set_full_attn_weights")

    def set_deltanet_weights(self, layer: int, conv_w, A, dt_bias, norm_w):
        arrs = [np.ascontiguousarray(x, np.float32) for x in (conv_w, A, dt_bias, norm_w)]
        check(lib().anelm_set_deltanet_weights(self.handle, layer, *[_fp(a) for a in arrs]), "set_deltanet_weights")

    def reset(self, seq: int = -1):
        check(lib().anelm_reset(self.handle, seq), "anelm_reset")

    def kv_export(self, layer: int, seq: int):
        c = self.cfg
        shape = (self.capacities[seq], c.num_kv_heads, c.head_dim)
        k = np.zeros(shape, np.float32)
        v = np.zeros(shape, np.float32)
        ln, st = ctypes.c_int(), ctypes.c_int()
        check(lib().anelm_kv_export(self.handle, layer, seq, _fp(k), _fp(v), ctypes.byref(ln), ctypes.byref(st)),
              "anelm_kv_export")
        return k, v, ln.value, st.value

    def kv_import(self, layer: int, seq: int, k, v, length: int, start: int):
        k = np.ascontiguousarray(k, np.float32)
        v = np.ascontiguousarray(v, np.float32)
        check(lib().anelm_kv_import(self.handle, layer, seq, _fp(k), _fp(v), length, start), "anelm_kv_import")

    def kv_write(self, layer: int, seq: int, slot0: int, k: torch.Tensor, v: torch.Tensor):
        assert k.dtype == torch.float16 and v.dtype == torch.float16 and k.is_contiguous() and v.is_contiguous()
        n = k.shape[0]
        check(lib().anelm_kv_write(self.handle, layer, seq, slot0, n, ctypes.c_void_p(k.data_ptr()),
                                   ctypes.c_void_p(v.data_ptr()), _stream(k.device)), "anelm_kv_write")

    def kv_set_meta(self, layer: int, seq: int, length: int, start: int):
        check(lib().anelm_kv_set_meta(self.handle, layer, seq, length, start), "anelm_kv_set_meta")

    def deltanet_state_export(self, layer: int, seq: int):
        c = self.cfg
        ssm = np.zeros((c.lin_num_val_heads, c.lin_key_dim, c.lin_val_dim), np.float32)
        conv = np.zeros((self.conv_channels, c.conv_kernel - 1), np.float32)
        pos = ctypes.c_int()
        check(lib().anelm_deltanet_state_export(self.handle, layer, seq, _fp(ssm), _fp(conv), ctypes.byref(pos)),
              "anelm_deltanet_state_export")
        return ssm, conv, pos.value

    def deltanet_state_import(self, layer: int, seq: int, ssm, conv, conv_pos: int):
        ssm = np.ascontiguousarray(ssm, np.float32)
        conv = np.ascontiguousarray(conv, np.float32)
        check(lib().anelm_deltanet_state_import(self.handle, layer, seq, _fp(ssm), _fp(conv), conv_pos),
              "anelm_deltanet_state_import")

    def deltanet_state_write(self, layer: int, seq: int, ssm: torch.Tensor):
        assert ssm.dtype == torch.float32 and ssm.is_contiguous()
        check(lib().anelm_deltanet_state_write(self.handle, layer, seq, ctypes.c_void_p(ssm.data_ptr()),
                                               _stream(ssm.device)), "anelm_deltanet_state_write")

    def device_error(self) -> int:
        code = ctypes.c_int()
        check(lib().anelm_get_device_error(self.handle, ctypes.byref(code)), "anelm_get_device_error")
        return code.value

    # ---- compute ----
    def _out(self, out, n_rows, width, dtype, device):
        if out is None:
            out = torch.empty((n_rows, width) if n_rows > 1 else (width,), dtype=dtype, device=device)
        assert out.is_contiguous()
        return out

    def full_attn_from_proj(self, layer: int, seq: int, proj: torch.Tensor, pos: int, out=None,
                            out_dtype=torch.float32):
        assert proj.is_cuda and proj.is_contiguous() and proj.numel() == self.fa_proj_dim
        out = self._out(out, 1, self.fa_out_dim, out_dtype, proj.device)
        check(lib().anelm_full_attn_from_proj(self.handle, layer, seq, ctypes.c_void_p(proj.data_ptr()),
                                              _dtype_code(proj), pos, ctypes.c_void_p(out.data_ptr()),
                                              _dtype_code(out), _stream(proj.device)), "anelm_full_attn_from_proj")
        return out

    def deltanet_from_proj(self, layer: int, seq: int, proj: torch.Tensor, out=None, out_dtype=torch.float32):
        assert proj.is_cuda and proj.is_contiguous() and proj.numel() == self.gdn_proj_dim
        out = self._out(out, 1, self.gdn_out_dim, out_dtype, proj.device)
        check(lib().anelm_deltanet_from_proj(self.handle, layer, seq, ctypes.c_void_p(proj.data_ptr()),
                                             _dtype_code(proj), ctypes.c_void_p(out.data_ptr()), _dtype_code(out),
                                             _stream(proj.device)), "anelm_deltanet_from_proj")
        return out

    def plan(self, seq_ids) -> Plan:
        return Plan(self, seq_ids)

    def full_attn_decode(self, plan: Plan, layer: int, proj: torch.Tensor, pos: torch.Tensor, out=None,
                         out_dtype=torch.float32):
        assert proj.is_cuda and proj.is_contiguous() and proj.shape == (plan.n, self.fa_proj_dim)
        assert pos.dtype == torch.int32 and pos.is_cuda and pos.numel() == plan.n
        if out is None:
            out = torch.empty((plan.n, self.fa_out_dim), dtype=out_dtype, device=proj.device)
        check(lib().anelm_full_attn_decode(self.handle, plan.handle, layer, ctypes.c_void_p(proj.data_ptr()),
                                           _dtype_code(proj), ctypes.c_void_p(pos.data_ptr()),
                                           ctypes.c_void_p(out.data_ptr()), _dtype_code(out), _stream(proj.device)),
              "anelm_full_attn_decode")
        return out

    def full_attn_prefill(self, plan: Plan, layer: int, proj: torch.Tensor, start_pos: int = 0, out=None,
                          out_dtype=torch.float32):
        """Causal prefill of fresh rings: proj [B][n][fa_proj_dim] for the plan's B sequences;
        returns out [B][n][Hq*d].  Leaves each ring holding the n tokens (len n, start 0)."""
        assert proj.is_cuda and proj.is_contiguous() and proj.dim() == 3 and proj.shape[0] == plan.n
        assert proj.shape[2] == self.fa_proj_dim
        n = proj.shape[1]
        if out is None:
            out = torch.empty((plan.n, n, self.fa_out_dim), dtype=out_dtype, device=proj.device)
        check(lib().anelm_full_attn_prefill(self.handle, plan.handle, layer, n, ctypes.c_void_p(proj.data_ptr()),
                                            _dtype_code(proj), start_pos, ctypes.c_void_p(out.data_ptr()),
                                            _dtype_code(out), _stream(proj.device)), "anelm_full_attn_prefill")
        return out

    def deltanet_prefill(self, plan: Plan, layer: int, proj: torch.Tensor, out=None, out_dtype=torch.float32):
        """Chunkwise prefill of a DeltaNet layer: proj [B][n][gdn_proj_dim] for the plan's B sequences;
        returns out [B][n][Hv*dv].  Continues from (and updates) each sequence's state and conv ring."""
        assert proj.is_cuda and proj.is_contiguous() and proj.dim() == 3 and proj.shape[0] == plan.n
        assert proj.shape[2] == self.gdn_proj_dim
        n = proj.shape[1]
        if out is None:
            out = torch.empty((plan.n, n, self.gdn_out_dim), dtype=out_dtype, device=proj.device)
        check(lib().anelm_deltanet_prefill(self.handle, plan.handle, layer, n, ctypes.c_void_p(proj.data_ptr()),
                                           _dtype_code(proj), ctypes.c_void_p(out.data_ptr()), _dtype_code(out),
                                           _stream(proj.device)), "anelm_deltanet_prefill")
        return out

    def set_layer_projections(self, layer: int, w_in: torch.Tensor, w_out: torch.Tensor):
        """bf16 projection weights of a layer (anelm_set_layer_projections): w_in [proj_dim][hidden],
        w_out [hidden][core out], CPU or CUDA tensors."""
        assert w_in.dtype == torch.bfloat16 and w_out.dtype == torch.bfloat16
        w_in, w_out = w_in.contiguous(), w_out.contiguous()
        check(lib().anelm_set_layer_projections(self.handle, layer, w_in.shape[1], ctypes.c_void_p(w_in.data_ptr()),
                                                ctypes.c_void_p(w_out.data_ptr())), "anelm_set_layer_projections")

    def layer_decode(self, plan: Plan, layer: int, x: torch.Tensor, pos: torch.Tensor = None, y=None):
        """One decode layer on the device (anelm_layer_decode): x [n][hidden] bf16 -> in-projection,
        core, out-projection -> y [n][hidden] bf16; pos [n] int32 for attention layers."""
        assert x.is_cuda and x.is_contiguous() and x.dtype == torch.bfloat16 and x.shape[0] == plan.n
        if y is None:
            y = torch.empty_like(x)
        pp = ctypes.c_void_p(pos.data_ptr()) if pos is not None else None
        check(lib().anelm_layer_decode(self.handle, plan.handle, layer, ctypes.c_void_p(x.data_ptr()), pp,
                                       ctypes.c_void_p(y.data_ptr()), _stream(x.device)), "anelm_layer_decode")
        return y

    def deltanet_decode(self, plan: Plan, layer: int, proj: torch.Tensor, out=None, out_dtype=torch.float32):
        assert proj.is_cuda and proj.is_contiguous() and proj.shape == (plan.n, self.gdn_proj_dim)
        if out is None:
            out = torch.empty((plan.n, self.gdn_out_dim), dtype=out_dtype, device=proj.device)
        check(lib().anelm_deltanet_decode(self.handle, plan.handle, layer, ctypes.c_void_p(proj.data_ptr()),
                                          _dtype_code(proj), ctypes.c_void_p(out.data_ptr()), _dtype_code(out),
                                          _stream(proj.device)), "anelm_deltanet_decode")
        return out


def gated_delta_chunked(q: torch.Tensor, k: torch.Tensor, v: torch.Tensor, log_decay: torch.Tensor,
                        beta: torch.Tensor, state: torch.Tensor, delta_mode: int = 0, y=None,
                        y_dtype=torch.float32, workspace=None) -> torch.Tensor:
    """The chunked gated delta rule on the GPU (anelm_gated_delta_chunked): q, k [B][T][Hk][128],
    v [B][T][Hv][128] (f32/f16/bf16), log_decay, beta [B][T][Hv] fp32, state [B][Hv][128][128] fp32
    updated in place.  Returns y [B][T][Hv][128]."""
    B, T, Hk, dk = q.shape
    Hv, dv = v.shape[2], v.shape[3]
    for t in (q, k, v, log_decay, beta, state):
        assert t.is_cuda and t.is_contiguous()
    assert log_decay.dtype == torch.float32 and beta.dtype == torch.float32 and state.dtype == torch.float32
    if y is None:
        y = torch.empty((B, T, Hv, dv), dtype=y_dtype, device=q.device)
    need = lib().anelm_gated_delta_chunked_workspace_bytes(B, T, Hk, Hv)
    if workspace is None:
        workspace = torch.empty(need, dtype=torch.uint8, device=q.device)
    check(lib().anelm_gated_delta_chunked(
        ctypes.c_void_p(q.data_ptr()), ctypes.c_void_p(k.data_ptr()), ctypes.c_void_p(v.data_ptr()), _dtype_code(q),
        ctypes.c_void_p(log_decay.data_ptr()), ctypes.c_void_p(beta.data_ptr()), ctypes.c_void_p(state.data_ptr()),
        B, T, Hk, Hv, dk, dv, delta_mode, ctypes.c_void_p(y.data_ptr()), _dtype_code(y),
        ctypes.c_void_p(workspace.data_ptr()), workspace.numel(), _stream(q.device)), "anelm_gated_delta_chunked")
    return y


def gemm_bf16(a: torch.Tensor, b: torch.Tensor, out_dtype=torch.bfloat16, out=None) -> torch.Tensor:
    """a [M][K] @ b[N][K]^T on the tensor cores (anelm_gemm_bf16): bf16 inputs (row-major, unit
    column stride), fp32 accumulation, result [M][N] of out_dtype (bf16 / fp16 / fp32)."""
    assert a.is_cuda and b.is_cuda and a.dtype == torch.bfloat16 and b.dtype == torch.bfloat16
    assert a.dim() == 2 and b.dim() == 2 and a.stride(1) == 1 and b.stride(1) == 1 and a.shape[1] == b.shape[1]
    M, K = a.shape
    N = b.shape[0]
    if out is None:
        out = torch.empty((M, N), dtype=out_dtype, device=a.device)
    assert out.stride(1) == 1
    check(lib().anelm_gemm_bf16(ctypes.c_void_p(a.data_ptr()), a.stride(0), ctypes.c_void_p(b.data_ptr()), b.stride(0),
                                ctypes.c_void_p(out.data_ptr()), out.stride(0), _dtype_code(out), M, N, K,
                                _stream(a.device)), "anelm_gemm_bf16")
    return out


def lm_head_topk(h: torch.Tensor, w: torch.Tensor, k: int = 32, workspace=None):
    """Top-k logits of h [n][hidden] @ w[vocab][hidden]^T without materialising the logits
    (anelm_lm_head_topk): bf16 inputs; returns (values fp32 [n][k], indices int32 [n][k]),
    sorted descending."""
    assert h.is_cuda and w.is_cuda and h.dtype == torch.bfloat16 and w.dtype == torch.bfloat16
    assert h.dim() == 2 and w.dim() == 2 and h.stride(1) == 1 and w.stride(1) == 1 and h.shape[1] == w.shape[1]
    n, hidden = h.shape
    vocab = w.shape[0]
    vals = torch.empty((n, k), dtype=torch.float32, device=h.device)
    idx = torch.empty((n, k), dtype=torch.int32, device=h.device)
    need = lib().anelm_lm_head_topk_workspace_bytes(n, vocab)
    if workspace is None:
        workspace = torch.empty(need, dtype=torch.uint8, device=h.device)
    check(lib().anelm_lm_head_topk(ctypes.c_void_p(h.data_ptr()), h.stride(0), ctypes.c_void_p(w.data_ptr()),
                                   w.stride(0), n, vocab, hidden, k, ctypes.c_void_p(vals.data_ptr()),
                                   ctypes.c_void_p(idx.data_ptr()), ctypes.c_void_p(workspace.data_ptr()),
                                   workspace.numel(), _stream(h.device)), "anelm_lm_head_topk")
    return vals, idx

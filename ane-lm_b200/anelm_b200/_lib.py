"""ctypes binding of the anelm_b200 C ABI (include/anelm_b200.h).

Loads the in-tree library anelm_b200/lib/libanelm_b200.so.  There is no CPU
fallback: if the library is missing the import fails loudly, and every compute
entry point reports ANELM_ERR_CUDA without an sm_100 device.
"""
from __future__ import annotations

import ctypes
import os
import re

HERE = os.path.dirname(os.path.abspath(__file__))
LIB_PATH = os.path.join(HERE, "lib", "libanelm_b200.so")
HEADER = os.path.join(os.path.dirname(os.path.dirname(HERE)), "include", "anelm_b200.h")

OK, ERR_INVALID_ARG, ERR_CAPACITY, ERR_CUDA, ERR_TIMEOUT, ERR_UNSUPPORTED, ERR_STATE, ERR_NOMEM = range(8)
F32, F16, BF16 = 0, 1, 2
LAYER_LINEAR_ATTN, LAYER_FULL_ATTN = 0, 1
ROPE_INTERLEAVED, ROPE_HALF = 0, 1
DELTA_CPUOPS, DELTA_HF = 0, 1
KV_RING, KV_LINEAR = 0, 1


class AnelmError(RuntimeError):
    def __init__(self, status: int, what: str, msg: str):
        super().__init__(f"{what}: status {status} ({msg})")
        self.status = status


class Config(ctypes.Structure):
    """anelm_config; field order must match include/anelm_b200.h."""

    _fields_ = [
        ("num_layers", ctypes.c_int),
        ("layer_types", ctypes.POINTER(ctypes.c_int)),
        ("full_attention_interval", ctypes.c_int),
        ("num_q_heads", ctypes.c_int), ("num_kv_heads", ctypes.c_int),
        ("head_dim", ctypes.c_int), ("rot_dim", ctypes.c_int),
        ("rope_theta", ctypes.c_float), ("rms_eps", ctypes.c_float),
        ("attn_output_gate", ctypes.c_int),
        ("lin_num_key_heads", ctypes.c_int), ("lin_num_val_heads", ctypes.c_int),
        ("lin_key_dim", ctypes.c_int), ("lin_val_dim", ctypes.c_int), ("conv_kernel", ctypes.c_int),
        ("max_seqs", ctypes.c_int), ("kv_capacity", ctypes.c_int),
        ("seq_kv_capacity", ctypes.POINTER(ctypes.c_int)),
        ("rope_table_len", ctypes.c_int),
        ("rope_mode", ctypes.c_int), ("delta_mode", ctypes.c_int), ("l2_eps", ctypes.c_float),
        ("qk_norm_in_core", ctypes.c_int), ("kv_mode", ctypes.c_int),
    ]


_vp = ctypes.c_void_p
_ip = ctypes.POINTER(ctypes.c_int)
_fp = ctypes.POINTER(ctypes.c_float)
_i = ctypes.c_int
_f = ctypes.c_float
_u16p = ctypes.c_void_p

SIGNATURES = {
    "anelm_config_default": [ctypes.POINTER(Config)],
    "anelm_create": [ctypes.POINTER(Config), _i, ctypes.POINTER(_vp)],
    "anelm_destroy": [_vp],
    "anelm_set_full_attn_weights": [_vp, _i, _vp, _vp],
    "anelm_set_deltanet_weights": [_vp, _i, _vp, _vp, _vp, _vp],
    "anelm_reset": [_vp, _i],
    "anelm_kv_export": [_vp, _i, _i, _vp, _vp, _ip, _ip],
    "anelm_kv_import": [_vp, _i, _i, _vp, _vp, _i, _i],
    "anelm_kv_write": [_vp, _i, _i, _i, _i, _vp, _vp, _vp],
    "anelm_kv_set_meta": [_vp, _i, _i, _i, _i],
    "anelm_deltanet_state_export": [_vp, _i, _i, _vp, _vp, _ip],
    "anelm_deltanet_state_import": [_vp, _i, _i, _vp, _vp, _i],
    "anelm_deltanet_state_write": [_vp, _i, _i, _vp, _vp],
    "anelm_get_device_error": [_vp, _ip],
    "anelm_full_attn_from_proj": [_vp, _i, _i, _vp, _i, _i, _vp, _i, _vp],
    "anelm_deltanet_from_proj": [_vp, _i, _i, _vp, _i, _vp, _i, _vp],
    "anelm_plan_create": [_vp, _i, _ip, ctypes.POINTER(_vp)],
    "anelm_plan_destroy": [_vp],
    "anelm_plan_info": [_vp, _ip, _ip],
    "anelm_full_attn_decode": [_vp, _vp, _i, _vp, _i, _vp, _vp, _i, _vp],
    "anelm_deltanet_decode": [_vp, _vp, _i, _vp, _i, _vp, _i, _vp],
    "anelm_set_layer_projections": [_vp, _i, _i, _vp, _vp],
    "anelm_layer_decode": [_vp, _vp, _i, _vp, _vp, _vp, _vp],
    "anelm_full_attn_prefill": [_vp, _vp, _i, _i, _vp, _i, _i, _vp, _i, _vp],
    "anelm_deltanet_prefill": [_vp, _vp, _i, _i, _vp, _i, _vp, _i, _vp],
    "anelm_gated_delta_chunked": [_vp, _vp, _vp, _i, _vp, _vp, _vp, _i, _i, _i, _i, _i, _i, _i, _vp, _i, _vp,
                                  ctypes.c_size_t, _vp],
    "anelm_py_cpu_attention": [_vp, _i, _i, _u16p, _u16p, _u16p, _i, _u16p, _vp],
    "anelm_gemm_bf16": [_vp, ctypes.c_longlong, _vp, ctypes.c_longlong, _vp, ctypes.c_longlong, _i, _i, _i, _i, _vp],
    "anelm_lm_head_topk": [_vp, ctypes.c_longlong, _vp, ctypes.c_longlong, _i, _i, _i, _i, _vp, _vp, _vp,
                           ctypes.c_size_t, _vp],
    "anelm_gqa_attention": [_vp, _vp, _vp, _vp, _i, _i, _i, _i, _i, _i, _i, _i, _vp],
    "anelm_gqa_attention_noalloc": [_vp, _vp, _vp, _vp, _i, _i, _i, _i, _i, _i, _i, _vp],
    "anelm_selftest_wait_timeout": [_vp, ctypes.c_uint, _vp],
    "anelm_full_attn_prefill_gather": [_vp, _vp, _i, _i, _vp, _i, _i, _vp, _i, _i, _i, _i, _vp],
    "anelm_ipc_handle": [_vp, _vp, ctypes.POINTER(ctypes.c_size_t)],
    "anelm_ipc_open": [_vp, ctypes.c_size_t, _i, ctypes.POINTER(ctypes.c_void_p)],
    "anelm_ipc_close": [_vp],
    "anelm_ssm_step": [_vp, _vp, _vp, _vp, _vp, _f, _f, _i, _i, _vp],
    "anelm_conv1d_update": [_vp, _vp, _ip, _vp, _vp, _i, _i, _vp],
    "anelm_rmsnorm": [_vp, _vp, _vp, _i, _f, _i, _vp],
    "anelm_rmsnorm_gated": [_vp, _vp, _vp, _vp, _i, _i, _vp],
    "anelm_apply_rope_cached": [_vp, _vp, _i, _i, _i, _i, _i, _i, _i, _f, _vp, _vp, _vp],
    "anelm_l2_normalize": [_vp, _i, _i, _vp],
    "anelm_silu_vec_inplace": [_vp, _i, _vp],
    "anelm_mul_sigmoid_inplace": [_vp, _vp, _i, _vp],
    "anelm_softmax": [_vp, _i, _i, _vp],
    "anelm_matvec": [_vp, _vp, _vp, _i, _i, _vp],
    "anelm_device_check": [_i],
}


def header_functions(path: str = HEADER) -> list[str]:
    """Names of every ANELM_API function declared in include/anelm_b200.h."""
    txt = open(path).read()
    return re.findall(r"ANELM_API\s+[\w\s\*]+?\b(anelm_\w+)\s*\(", txt)


_lib = None


def lib() -> ctypes.CDLL:
    global _lib
    if _lib is not None:
        return _lib
    if not os.path.exists(LIB_PATH):
        raise ImportError(f"{LIB_PATH} is missing: build it with `python ane-lm_b200/build.py` "
                          "(there is no CPU fallback)")
    L = ctypes.CDLL(LIB_PATH)
    for name, args in SIGNATURES.items():
        f = getattr(L, name)
        f.argtypes = args
        f.restype = ctypes.c_int
    for name in ("anelm_status_string",):
        getattr(L, name).argtypes = [_i]
        getattr(L, name).restype = ctypes.c_char_p
    L.anelm_last_error.argtypes = []
    L.anelm_last_error.restype = ctypes.c_char_p
    L.anelm_version.argtypes = []
    L.anelm_version.restype = ctypes.c_char_p
    L.anelm_gated_delta_chunked_workspace_bytes.argtypes = [_i, _i, _i, _i]
    L.anelm_gated_delta_chunked_workspace_bytes.restype = ctypes.c_size_t
    L.anelm_lm_head_topk_workspace_bytes.argtypes = [_i, _i]
    L.anelm_lm_head_topk_workspace_bytes.restype = ctypes.c_size_t
    _lib = L
    return L


def check(status: int, what: str) -> None:
    if status != OK:
        L = lib()
        raise AnelmError(status, what, (L.anelm_last_error() or b"").decode() or
                         L.anelm_status_string(status).decode())

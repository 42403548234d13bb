"""CPU-only checks of the C ABI boundary: the library loads, exports every entry
point include/anelm_b200.h declares, validates arguments before touching a GPU,
and fails loudly (no CPU fallback) when no sm_100 device is present."""
import ctypes

import pytest

import anelm_b200 as ab
from anelm_b200._lib import Config, header_functions, lib


def test_library_exports_every_header_symbol():
    L = lib()
    names = header_functions()
    assert len(names) >= 30
    missing = [n for n in names if not hasattr(L, n)]
    assert not missing, missing
    assert L.anelm_version().startswith(b"anelm_b200")


def test_config_default_matches_qwen35_args():
    c = Config()
    assert lib().anelm_config_default(ctypes.byref(c)) == 0
    # models/llm/qwen3_5.h:51-80 and qwen3_5.h:125-126
    assert (c.num_layers, c.num_q_heads, c.num_kv_heads, c.head_dim, c.rot_dim) == (24, 8, 2, 256, 64)
    assert (c.lin_num_key_heads, c.lin_num_val_heads, c.lin_key_dim, c.lin_val_dim) == (16, 16, 128, 128)
    assert c.kv_capacity == 2048 and c.rope_table_len == 4096 and c.full_attention_interval == 4
    assert abs(c.rope_theta - 1e7) < 1 and abs(c.l2_eps - 1e-12) < 1e-15


def test_argument_validation_without_gpu():
    L = lib()
    assert L.anelm_gqa_attention(None, None, None, None, 0, 1, 1, 256, 256, 0, 1, 1, None) == ab._lib.ERR_INVALID_ARG
    assert b"null" in L.anelm_last_error()
    assert L.anelm_rmsnorm(None, None, None, 0, 1e-6, 1, None) == ab._lib.ERR_INVALID_ARG
    assert L.anelm_create(None, 0, None) == ab._lib.ERR_INVALID_ARG
    assert L.anelm_plan_create(None, 1, None, None) == ab._lib.ERR_INVALID_ARG
    assert L.anelm_status_string(2) == b"capacity exceeded"


def test_no_cpu_fallback():
    torch = pytest.importorskip("torch")
    if torch.cuda.is_available():
        pytest.skip("a GPU is present")
    c = Config()
    lib().anelm_config_default(ctypes.byref(c))
    h = ctypes.c_void_p()
    rc = lib().anelm_create(ctypes.byref(c), 0, ctypes.byref(h))
    assert rc == ab._lib.ERR_CUDA and not h.value

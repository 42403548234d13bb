"""CPU-only checks of the C ABI boundary: the library loads, exports every entry
point include/anelm_b200.h declares, validates arguments before touching a GPU,
and fails loudly (no CPU fallback) when no sm_100 device is present."""
import ctypes
import os

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


def test_cpu_ops_compat_exports_and_links(tmp_path):
    """include/cpu_ops_compat/cpu_ops.h declares core/cpu_ops.h's functions (namespace ane_lm);
    the library exports each with that signature, and the oracle's layer glue, written against
    core/cpu_ops.h, compiles and links against the shim unchanged (no GPU needed)."""
    import re
    import shutil
    import subprocess

    repo = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
    hdr = open(os.path.join(repo, "include", "cpu_ops_compat", "cpu_ops.h")).read()
    names = [n for n in re.findall(r"^void\s+(\w+)\s*\(", hdr, re.M)]
    assert len(names) == 11, names
    nm = shutil.which("nm")
    if nm:
        syms = subprocess.run([nm, "-DC", ab.LIB_PATH], capture_output=True, text=True).stdout
        for n in names:
            assert re.search(rf" T ane_lm::{n}\(", syms), n
        assert "ane_lm::gqa_attention(float*, float const*, float const*, float const*, int, int, int, int, int, int, int)" in syms
    gxx = shutil.which("g++")
    if not gxx:
        pytest.skip("no g++")
    libdir = os.path.dirname(ab.LIB_PATH)
    out = tmp_path / "libshim_glue.so"
    r = subprocess.run([gxx, "-O1", "-fPIC", "-shared", "-std=c++17", f"-I{repo}/include/cpu_ops_compat",
                        f"-I{repo}/oracle", f"{repo}/oracle/ref_glue.cpp", f"-L{libdir}", "-lanelm_b200",
                        f"-Wl,-rpath,{libdir}", "-Wl,--no-undefined", "-o", str(out)], capture_output=True, text=True)
    assert r.returncode == 0, r.stderr[-3000:]

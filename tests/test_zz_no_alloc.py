"""anelm_gqa_attention_noalloc: the allocation-free gqa_attention for callers that
cannot allocate device memory where attention runs (a server whose own pool
holds all free HBM, a plugin host that owns the allocator).  It must give the
same result as anelm_gqa_attention, through the C ABI, on two calls in a row
(the second one reuses the library's fixed scratch as the first left it).

This file is named to be collected last, so a run that stops at the first
failure has already run every other test."""
import ctypes

import numpy as np
import pytest

torch = pytest.importorskip("torch")

import anelm_b200 as ab  # noqa: E402
from anelm_b200._lib import lib  # noqa: E402
from helpers import ATOL, RTOL, assert_close, f16  # noqa: E402
from oracle import pyoracle as po  # noqa: E402

pytestmark = pytest.mark.gpu


def _p(t):
    return ctypes.c_void_p(t.data_ptr())


def _pool_usage():
    """(used, reserved) bytes of the current device's default stream-ordered pool, the pool
    cudaMallocAsync draws from, plus torch's own allocator counter."""
    from cuda.bindings import runtime as rt
    err, dev = rt.cudaGetDevice()
    assert err == rt.cudaError_t.cudaSuccess
    err, pool = rt.cudaDeviceGetDefaultMemPool(dev)
    assert err == rt.cudaError_t.cudaSuccess
    vals = []
    for attr in (rt.cudaMemPoolAttr.cudaMemPoolAttrUsedMemCurrent, rt.cudaMemPoolAttr.cudaMemPoolAttrReservedMemCurrent):
        err, v = rt.cudaMemPoolGetAttribute(pool, attr)
        assert err == rt.cudaError_t.cudaSuccess
        vals.append(int(v))
    return vals[0], vals[1], torch.cuda.memory_allocated()


def _torch_attention(q, kc, vc, start, length):
    """fp32 torch restatement of gqa_attention (core/cpu_ops.cpp:148-204) over the ring's logical
    order [start, cap) then [0, ...): softmax(q K^T / sqrt(d)) V per q head."""
    cap, Hkv, d = kc.shape
    Hq = q.shape[0]
    idx = (start + torch.arange(length, device=kc.device)) % cap
    k = kc[idx].float().transpose(0, 1)                      # [Hkv][L][d]
    v = vc[idx].float().transpose(0, 1)
    qh = q[:, :d].reshape(Hkv, Hq // Hkv, d)
    p = torch.softmax(qh @ k.transpose(1, 2) / d ** 0.5, dim=-1)
    return (p @ v).reshape(Hq, d)


@pytest.mark.parametrize("Hq,Hkv,d,cap,start,length", [(8, 2, 256, 4096, 1000, 4096), (16, 4, 256, 300, 299, 300),
                                                       (4, 1, 128, 20000, 7, 19990)])
def test_noalloc_matches_allocating_entry(Hq, Hkv, d, cap, start, length):
    rng = np.random.default_rng(cap + Hq)
    kc = torch.from_numpy(f16(rng.standard_normal((cap, Hkv, d)))).half().cuda()
    vc = torch.from_numpy(f16(rng.standard_normal((cap, Hkv, d)))).half().cuda()
    L = lib()
    want = torch.empty((Hq, d), device="cuda")
    outs = []
    for call in range(2):
        q = torch.from_numpy((2 * rng.standard_normal((Hq, 2 * d))).astype(np.float32)).cuda()
        assert L.anelm_gqa_attention(_p(want), _p(q), _p(kc), _p(vc), ab.F16, Hq, Hkv, d, 2 * d, start, length, cap,
                                     None) == 0, L.anelm_last_error()
        got = torch.full((Hq, d), float("nan"), device="cuda")
        rc = L.anelm_gqa_attention_noalloc(_p(got), _p(q), _p(kc), _p(vc), Hq, Hkv, d, 2 * d, start, length, cap,
                                           None)
        assert rc == 0, L.anelm_last_error()
        torch.cuda.synchronize()
        assert_close(got.cpu().numpy(), want.cpu().numpy(), atol=ATOL, rtol=RTOL, what=f"call {call}")
        # and against the CPU oracle (gqa_attention restated from core/cpu_ops.cpp:148-204)
        ref = np.zeros((Hq, d), np.float32)
        po.fn("oracle", "gqa_attention")(po.P(ref), po.P(q.cpu().numpy()), po.P(kc.float().cpu().numpy()),
                                         po.P(vc.float().cpu().numpy()), Hq, Hkv, d, 2 * d, start, length, cap)
        assert_close(got.cpu().numpy(), ref, atol=ATOL, rtol=RTOL, what=f"call {call} vs oracle")
        outs.append(got.cpu().numpy())
    assert not np.array_equal(outs[0], outs[1])  # two different queries really ran


def test_noalloc_long_splits_when_the_scratch_caps_the_split_count():
    """512 kv heads of 256: one split's partials (2 MiB) leave room for a single split in the
    fixed scratch, so the whole 6000-token ring (wrapped at slot 1234) is one 6016-token split --
    longer than the allocating entry's 4096-token splits.  Checked against the allocating entry
    and an fp32 torch restatement, on two calls in a row."""
    Hq = Hkv = 512
    d, cap, start, length = 256, 6000, 1234, 6000
    g = torch.Generator(device="cuda")
    g.manual_seed(5)
    kc = torch.randn(cap, Hkv, d, generator=g, device="cuda").half()
    vc = torch.randn(cap, Hkv, d, generator=g, device="cuda").half()
    L = lib()
    for call in range(2):
        q = 2 * torch.randn(Hq, 2 * d, generator=g, device="cuda")
        want = torch.empty((Hq, d), device="cuda")
        assert L.anelm_gqa_attention(_p(want), _p(q), _p(kc), _p(vc), ab.F16, Hq, Hkv, d, 2 * d, start, length, cap,
                                     None) == 0, L.anelm_last_error()
        got = torch.full((Hq, d), float("nan"), device="cuda")
        assert L.anelm_gqa_attention_noalloc(_p(got), _p(q), _p(kc), _p(vc), Hq, Hkv, d, 2 * d, start, length, cap,
                                             None) == 0, L.anelm_last_error()
        torch.cuda.synchronize()
        assert_close(got.cpu().numpy(), want.cpu().numpy(), what=f"call {call} vs allocating entry")
        assert_close(got.cpu().numpy(), _torch_attention(q, kc, vc, start, length).cpu().numpy(),
                     what=f"call {call} vs fp32 torch")


def test_noalloc_allocates_nothing():
    """After a first call (which looks the scratch address up), further calls leave the
    stream-ordered pool and torch's allocator exactly where they were."""
    Hq, Hkv, d, cap = 16, 4, 256, 9000
    g = torch.Generator(device="cuda")
    g.manual_seed(6)
    kc = torch.randn(cap, Hkv, d, generator=g, device="cuda").half()
    vc = torch.randn(cap, Hkv, d, generator=g, device="cuda").half()
    q = torch.randn(Hq, 2 * d, generator=g, device="cuda")
    out = torch.empty((Hq, d), device="cuda")
    L = lib()
    args = (_p(out), _p(q), _p(kc), _p(vc), Hq, Hkv, d, 2 * d, 17, cap, cap, None)
    assert L.anelm_gqa_attention_noalloc(*args) == 0, L.anelm_last_error()
    torch.cuda.synchronize()
    before = _pool_usage()
    for _ in range(3):
        assert L.anelm_gqa_attention_noalloc(*args) == 0, L.anelm_last_error()
        assert _pool_usage() == before
    torch.cuda.synchronize()
    assert _pool_usage() == before


def test_noalloc_rejects_what_does_not_fit():
    L = lib()
    x = torch.zeros(16, device="cuda")
    # n_kv_heads * (4*d + 8) * 4 bytes of partials for one split exceed the fixed scratch
    rc = L.anelm_gqa_attention_noalloc(_p(x), _p(x), _p(x), _p(x), 1024, 1024, 256, 256, 0, 10, 10, None)
    assert rc == ab._lib.ERR_CAPACITY
    assert b"scratch" in L.anelm_last_error()
    rc = L.anelm_gqa_attention_noalloc(None, _p(x), _p(x), _p(x), 8, 2, 256, 512, 0, 10, 10, None)
    assert rc == ab._lib.ERR_INVALID_ARG

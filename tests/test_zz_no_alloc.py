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

pytestmark = pytest.mark.gpu


def _p(t):
    return ctypes.c_void_p(t.data_ptr())


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
        outs.append(got.cpu().numpy())
    assert not np.array_equal(outs[0], outs[1])  # two different queries really ran


def test_noalloc_rejects_what_does_not_fit():
    L = lib()
    x = torch.zeros(16, device="cuda")
    # n_kv_heads * (4*d + 8) * 4 bytes of partials for one split exceed the fixed scratch
    rc = L.anelm_gqa_attention_noalloc(_p(x), _p(x), _p(x), _p(x), 1024, 1024, 256, 256, 0, 10, 10, None)
    assert rc == ab._lib.ERR_CAPACITY
    assert b"scratch" in L.anelm_last_error()
    rc = L.anelm_gqa_attention_noalloc(None, _p(x), _p(x), _p(x), 8, 2, 256, 512, 0, 10, 10, None)
    assert rc == ab._lib.ERR_INVALID_ARG

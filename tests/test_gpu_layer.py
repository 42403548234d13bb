"""GPU layer steps with the projections on the device (anelm_set_layer_projections /
anelm_layer_decode): a DeltaNet layer and an attention layer of the Qwen3.5-4B shape (hidden
2560) over a plan of three sequences.  The fused call must equal, bit for bit, the composition
of the public pieces it replaces — bf16 in-projection (anelm_gemm_bf16), the core decode entry
with bf16 projection rows and output, bf16 out-projection — and leave the same KV ring and
DeltaNet state.  The pieces' numerics are checked on their own (test_gpu_gemm.py and the core
parity tests)."""
import numpy as np
import pytest

torch = pytest.importorskip("torch")

import anelm_b200 as ab  # noqa: E402
from anelm_b200.core import Context, gemm_bf16  # noqa: E402
from helpers import fa_inputs, fa_shape, gdn_inputs, gdn_shape, random_ring  # noqa: E402

pytestmark = pytest.mark.gpu

HIDDEN = 2560
HQ, HKV, D, R = 16, 4, 256, 64
HK, HV = 16, 32


def _ctx(caps):
    return Context(layer_types=[ab.LAYER_LINEAR_ATTN, ab.LAYER_FULL_ATTN], num_q_heads=HQ, num_kv_heads=HKV,
                   head_dim=D, rot_dim=R, rope_theta=1e7, lin_num_key_heads=HK, lin_num_val_heads=HV,
                   lin_key_dim=128, lin_val_dim=128, max_seqs=len(caps), seq_kv_capacity=caps)


def test_layer_decode_equals_projection_core_projection():
    rng = np.random.default_rng(21)
    gen = torch.Generator(device="cuda")
    gen.manual_seed(21)
    caps = [300, 128, 520]
    order = [2, 0, 1]
    fs, gs = fa_shape(HQ, HKV, D, R, 1e7), gdn_shape(HK, HV)
    _, qn, kn = fa_inputs(rng, fs, 1)
    _, conv_w, A, dt_bias, norm_w = gdn_inputs(rng, gs, 1)
    C = conv_w.shape[0]
    rings = [random_ring(rng, c, HKV, D, l, s) for c, (l, s) in zip(caps, [(300, 40), (17, 0), (100, 500)])]
    ssm = [(0.1 * rng.standard_normal((HV, 128, 128))).astype(np.float32) for _ in caps]
    conv = [rng.standard_normal((C, 3)).astype(np.float32) for _ in caps]
    fa_pd, gdn_pd = HQ * 2 * D + 2 * HKV * D, C + HV * 128 + 2 * HV
    w = {
        0: ((torch.randn(gdn_pd, HIDDEN, generator=gen, device="cuda") / HIDDEN ** 0.5).to(torch.bfloat16),
            (torch.randn(HIDDEN, HV * 128, generator=gen, device="cuda") / 64).to(torch.bfloat16)),
        1: ((torch.randn(fa_pd, HIDDEN, generator=gen, device="cuda") / HIDDEN ** 0.5).to(torch.bfloat16),
            (torch.randn(HIDDEN, HQ * D, generator=gen, device="cuda") / 64).to(torch.bfloat16)),
    }
    x = torch.randn(len(order), HIDDEN, generator=gen, device="cuda").to(torch.bfloat16)
    pos = torch.tensor([900, 17, 100], dtype=torch.int32, device="cuda")
    results = []
    for fused in (True, False):
        with _ctx(caps) as ctx:
            ctx.set_deltanet_weights(0, conv_w, A, dt_bias, norm_w)
            ctx.set_full_attn_weights(1, qn, kn)
            for s in range(len(caps)):
                ctx.kv_import(1, s, rings[s].k, rings[s].v, rings[s].len, rings[s].start)
                ctx.deltanet_state_import(0, s, ssm[s], conv[s], s % 3)
            plan = ctx.plan(order)
            if fused:
                for L in (0, 1):
                    ctx.set_layer_projections(L, *w[L])
                h = ctx.layer_decode(plan, 0, x)
                y = ctx.layer_decode(plan, 1, h, pos)
            else:
                p0 = gemm_bf16(x, w[0][0])
                h = gemm_bf16(ctx.deltanet_decode(plan, 0, p0, out_dtype=torch.bfloat16), w[0][1])
                p1 = gemm_bf16(h, w[1][0])
                y = gemm_bf16(ctx.full_attn_decode(plan, 1, p1, pos, out_dtype=torch.bfloat16), w[1][1])
            torch.cuda.synchronize()
            results.append((h.cpu(), y.cpu(), [ctx.kv_export(1, s) for s in range(len(caps))],
                            [ctx.deltanet_state_export(0, s) for s in range(len(caps))]))
            plan.close()
    (h1, y1, kv1, st1), (h2, y2, kv2, st2) = results
    assert torch.equal(h1, h2) and torch.equal(y1, y2)
    assert torch.isfinite(y1.float()).all() and y1.float().abs().max() > 0
    for a, b in zip(kv1, kv2):
        np.testing.assert_array_equal(a[0], b[0])
        np.testing.assert_array_equal(a[1], b[1])
        assert a[2:] == b[2:]
    for a, b in zip(st1, st2):
        np.testing.assert_array_equal(a[0], b[0])
        np.testing.assert_array_equal(a[1], b[1])
        assert a[2] == b[2]


def test_layer_decode_state_errors():
    with _ctx([64]) as ctx:
        plan = ctx.plan([0])
        x = torch.zeros(1, HIDDEN, device="cuda", dtype=torch.bfloat16)
        with pytest.raises(ab.AnelmError) as e:
            ctx.layer_decode(plan, 0, x)         # projections not set
        assert e.value.status == ab.ERR_STATE
        plan.close()

"""GPU parity of the chunkwise Gated DeltaNet prefill through the C ABI.

* The bare chunked delta rule (anelm_gated_delta_chunked) against the oracle's token-by-token
  recurrence (ssm_step, cpu_ops.cpp:131-146, or the decay-first order of
  export_hybrid_chunks.py:142-147): outputs and final state, ragged chunk counts, both orders,
  and BASELINE config 4 (Hv 32 / Hk 16, 8192 tokens) with the final state of two heads checked
  against the recurrence.
* The layer prefill (anelm_deltanet_prefill) against the oracle's per-token loop of
  forward_deltanet_from_proj (qwen3_5.cpp:849-909 called as in qwen3_5.cpp:1205-1217): outputs,
  state, conv ring and ring position, then decode continuing from the prefilled state.
Tolerance 2e-3 abs + 1e-2 rel (fp16 operands, fp32 accumulation and state); conv ring and
position bit-exact."""
import numpy as np
import pytest

torch = pytest.importorskip("torch")

import anelm_b200 as ab  # noqa: E402
from anelm_b200.core import Context, gated_delta_chunked  # noqa: E402
from helpers import assert_close, f16, gdn_inputs, gdn_shape  # noqa: E402
from oracle import pyoracle as po  # noqa: E402

pytestmark = pytest.mark.gpu


def core_inputs(rng, B, T, Hk, Hv, state_scale=0.1):
    """fp16-representable q, k (L2-normalised rows, q also scaled by 1/sqrt(128)), v N(0,1);
    log g ~ U(-0.1, 0), beta ~ U(0, 1) (BASELINE config 4 distributions)."""
    def unit(x):
        return x / np.linalg.norm(x, axis=-1, keepdims=True)
    q = f16(unit(rng.standard_normal((B, T, Hk, 128))) / np.sqrt(128.0))
    k = f16(unit(rng.standard_normal((B, T, Hk, 128))))
    v = f16(rng.standard_normal((B, T, Hv, 128)))
    lg = (-0.1 * rng.random((B, T, Hv))).astype(np.float32)
    beta = rng.random((B, T, Hv)).astype(np.float32)
    s0 = (state_scale * rng.standard_normal((B, Hv, 128, 128))).astype(np.float32)
    return q, k, v, lg, beta, s0


def run_core(q, k, v, lg, beta, s0, mode, dtype=torch.float16):
    dev = lambda a, dt=torch.float32: torch.tensor(a, device="cuda").to(dt).contiguous()  # noqa: E731
    state = dev(s0)
    y = gated_delta_chunked(dev(q, dtype), dev(k, dtype), dev(v, dtype), dev(lg), dev(beta), state, mode)
    torch.cuda.synchronize()
    return y.float().cpu().numpy(), state.cpu().numpy()


@pytest.mark.parametrize("mode", [ab.DELTA_CPUOPS, ab.DELTA_HF])
@pytest.mark.parametrize("T", [1, 63, 64, 65, 200])
def test_chunked_core_matches_recurrence(mode, T):
    rng = np.random.default_rng(100 + T + 7 * mode)
    B, Hk, Hv = 2, 2, 4
    q, k, v, lg, beta, s0 = core_inputs(rng, B, T, Hk, Hv)
    y, s = run_core(q, k, v, lg, beta, s0, mode)
    for b in range(B):
        st = s0[b].copy()
        want = po.gated_delta_tokens("oracle", q[b], k[b], v[b], lg[b], beta[b], st, mode)
        assert_close(y[b], want, what=f"y (b={b}, mode={mode}, T={T})")
        assert_close(s[b], st, what=f"final state (b={b}, mode={mode}, T={T})")


def test_chunked_core_bf16_inputs_and_strong_decay():
    """bf16 q/k/v and decays down to e^-4 per token (small g: the chunk form uses only ratios)."""
    rng = np.random.default_rng(5)
    B, T, Hk, Hv = 1, 130, 1, 2
    q, k, v, lg, beta, s0 = core_inputs(rng, B, T, Hk, Hv)
    q, k, v = (torch.tensor(a).to(torch.bfloat16).float().numpy() for a in (q, k, v))
    lg = (-4.0 * rng.random((B, T, Hv))).astype(np.float32)
    y, s = run_core(q, k, v, lg, beta, s0, ab.DELTA_CPUOPS, torch.bfloat16)
    st = s0[0].copy()
    want = po.gated_delta_tokens("oracle", q[0], k[0], v[0], lg[0], beta[0], st, 0)
    assert_close(y[0], want, what="y, strong decay")
    assert_close(s[0], st, what="state, strong decay")


def test_chunked_core_config4_final_state():
    """Hv 32 / Hk 16, 8192 tokens, B = 1, zero initial state; the final fp32
    state and the last outputs of value heads 0 and 31 against the token recurrence."""
    rng = np.random.default_rng(4)
    B, T, Hk, Hv = 1, 8192, 16, 32
    q, k, v, lg, beta, s0 = core_inputs(rng, B, T, Hk, Hv, state_scale=0.0)
    y, s = run_core(q, k, v, lg, beta, s0, ab.DELTA_CPUOPS)
    heads, kheads = [0, 31], [0, 15]
    st = np.zeros((2, 128, 128), np.float32)
    want = po.gated_delta_tokens("oracle", q[0][:, kheads], k[0][:, kheads], v[0][:, heads],
                                 lg[0][:, heads], beta[0][:, heads], st, 0)
    assert_close(s[0][heads], st, what="config-4 final state")
    assert_close(y[0][-64:, heads], want[-64:], what="config-4 last chunk outputs")
    assert_close(y[0][:64, heads], want[:64], what="config-4 first chunk outputs")


def gdn_ctx(shape, max_seqs=1, **kw):
    return Context(layer_types=[ab.LAYER_LINEAR_ATTN], lin_num_key_heads=shape.lin_num_key_heads,
                   lin_num_val_heads=shape.lin_num_val_heads, lin_key_dim=128, lin_val_dim=128,
                   max_seqs=max_seqs, kv_capacity=16, **kw)


@pytest.mark.parametrize("n", [2, 150])
def test_deltanet_prefill_matches_token_loop(n):
    """Two sequences (plan order reversed) from random states and conv rings at ring position 1;
    n = 2 keeps part of the old ring, n = 150 spans three chunks.  Then one decode token each."""
    rng = np.random.default_rng(20 + n)
    shape = gdn_shape(2, 4)
    Hv = 4
    proj, conv_w, A, dt_bias, norm_w = gdn_inputs(rng, shape, 2 * (n + 1))
    C = conv_w.shape[0]
    states = [po.DeltaState((0.1 * rng.standard_normal((Hv, 128, 128))).astype(np.float32),
                            rng.standard_normal((C, 3)).astype(np.float32), 1) for _ in range(2)]
    pre = proj[:2 * n].reshape(2, n, -1)
    nxt = proj[2 * n:].reshape(2, 1, -1)
    with gdn_ctx(shape, max_seqs=2) as ctx:
        ctx.set_deltanet_weights(0, conv_w, A, dt_bias, norm_w)
        for s in range(2):
            ctx.deltanet_state_import(0, s, states[s].ssm, states[s].conv, states[s].conv_pos)
        plan = ctx.plan([1, 0])  # row 0 is sequence 1
        p = torch.tensor(pre, device="cuda").to(torch.float16).contiguous()
        got = ctx.deltanet_prefill(plan, 0, p).cpu().numpy()
        exported = [ctx.deltanet_state_export(0, s) for s in range(2)]
        dec = ctx.deltanet_decode(plan, 0, torch.tensor(nxt[:, 0], device="cuda").to(torch.float16).contiguous())
        dec = dec.cpu().numpy()
        after = [ctx.deltanet_state_export(0, s) for s in range(2)]
        plan.close()
    for row, s in enumerate([1, 0]):
        st = states[s]
        want = po.deltanet_tokens("oracle", shape, po.make_variant(), conv_w, A, dt_bias, norm_w, st, pre[row])
        assert_close(got[row], want, what=f"prefill outputs (seq {s}, n={n})")
        ssm, conv, pos = exported[s]
        assert_close(ssm, st.ssm, what=f"prefill state (seq {s})")
        np.testing.assert_array_equal(conv, st.conv)
        assert pos == st.conv_pos
        want_dec = po.deltanet_tokens("oracle", shape, po.make_variant(), conv_w, A, dt_bias, norm_w, st, nxt[row])
        assert_close(dec[row], want_dec[0], what=f"decode after prefill (seq {s})")
        assert_close(after[s][0], st.ssm, what=f"state after decode (seq {s})")
        np.testing.assert_array_equal(after[s][1], st.conv)


def test_deltanet_prefill_hf_variant_gqa_shape():
    """Decay-first order with L2 eps 1e-6 on the 4B GQA shape (32 value / 16 key heads)."""
    rng = np.random.default_rng(31)
    shape = gdn_shape(16, 32)
    n = 70
    proj, conv_w, A, dt_bias, norm_w = gdn_inputs(rng, shape, n)
    st = po.DeltaState.zeros(shape)
    st.ssm[:] = (0.1 * rng.standard_normal(st.ssm.shape)).astype(np.float32)
    with gdn_ctx(shape, delta_mode=ab.DELTA_HF, l2_eps=1e-6) as ctx:
        ctx.set_deltanet_weights(0, conv_w, A, dt_bias, norm_w)
        ctx.deltanet_state_import(0, 0, st.ssm, st.conv, 0)
        plan = ctx.plan([0])
        got = ctx.deltanet_prefill(plan, 0, torch.tensor(proj[None], device="cuda").contiguous(),
                                   out_dtype=torch.bfloat16).float().cpu().numpy()
        ssm, conv, pos = ctx.deltanet_state_export(0, 0)
        plan.close()
    want = po.deltanet_tokens("oracle", shape, po.make_variant(delta_hf=1, l2_eps=1e-6), conv_w, A, dt_bias,
                              norm_w, st, proj)
    assert_close(got[0], want, what="HF-order prefill (bf16 out)")
    assert_close(ssm, st.ssm, what="HF-order prefill state")
    np.testing.assert_array_equal(conv, st.conv)
    assert pos == st.conv_pos


def test_chunked_core_rejects_bad_arguments():
    q = torch.zeros(1, 8, 1, 64, device="cuda", dtype=torch.float16)
    with pytest.raises(ab.AnelmError) as e:
        gated_delta_chunked(q, q, q, torch.zeros(1, 8, 1, device="cuda"), torch.zeros(1, 8, 1, device="cuda"),
                            torch.zeros(1, 1, 64, 64, device="cuda"))
    assert e.value.status == ab.ERR_UNSUPPORTED
    q = torch.zeros(1, 8, 1, 128, device="cuda", dtype=torch.float16)
    small = torch.empty(16, dtype=torch.uint8, device="cuda")
    with pytest.raises(ab.AnelmError) as e:
        gated_delta_chunked(q, q, q, torch.zeros(1, 8, 1, device="cuda"), torch.zeros(1, 8, 1, device="cuda"),
                            torch.zeros(1, 1, 128, 128, device="cuda"), workspace=small)
    assert e.value.status == ab.ERR_CAPACITY


@pytest.mark.parametrize("y_dtype", [torch.bfloat16, torch.float32])
def test_chunked_core_output_without_16_byte_alignment(y_dtype):
    """An output buffer that does not start on a 16-byte boundary takes the per-element store path
    of the recurrence kernel; its values must equal those of the aligned buffer bit for bit."""
    rng = np.random.default_rng(77)
    B, T, Hk, Hv = 1, 100, 2, 4
    q, k, v, lg, beta, s0 = core_inputs(rng, B, T, Hk, Hv)
    dev = lambda a, dt=torch.float32: torch.tensor(a, device="cuda").to(dt).contiguous()  # noqa: E731
    st_a, st_b = dev(s0), dev(s0)
    y_a = gated_delta_chunked(dev(q, torch.bfloat16), dev(k, torch.bfloat16), dev(v, torch.bfloat16), dev(lg),
                              dev(beta), st_a, ab.DELTA_CPUOPS, y_dtype=y_dtype)
    n = B * T * Hv * 128
    buf = torch.zeros(n + 1, dtype=y_dtype, device="cuda")
    y_b = buf[1:].view(B, T, Hv, 128)
    assert y_b.data_ptr() % 16 != 0
    gated_delta_chunked(dev(q, torch.bfloat16), dev(k, torch.bfloat16), dev(v, torch.bfloat16), dev(lg), dev(beta),
                        st_b, ab.DELTA_CPUOPS, y=y_b)
    torch.cuda.synchronize()
    assert torch.equal(y_a, y_b)
    assert torch.equal(st_a, st_b)
    assert buf[0].item() == 0


def test_chunked_core_fp32_inputs_through_the_pack():
    """fp32 q / k / v are not exact in fp16: the pack splits them into hi / lo planes and every product
    takes its three terms (the path 16-bit inputs skip by reading them in place)."""
    rng = np.random.default_rng(91)
    B, T, Hk, Hv = 2, 130, 2, 4
    q, k, v, lg, beta, s0 = core_inputs(rng, B, T, Hk, Hv)
    q = q + (1e-4 * rng.standard_normal(q.shape)).astype(np.float32)  # values fp16 cannot hold exactly
    y, s = run_core(q, k, v, lg, beta, s0, ab.DELTA_CPUOPS, torch.float32)
    for b in range(B):
        st = s0[b].copy()
        want = po.gated_delta_tokens("oracle", q[b], k[b], v[b], lg[b], beta[b], st, ab.DELTA_CPUOPS)
        assert_close(y[b], want, what=f"y (b={b}, fp32 inputs)")
        assert_close(s[b], st, what=f"final state (b={b}, fp32 inputs)")

"""CPU check of the chunk decomposition that the chunkwise Gated DeltaNet kernels compute
(ane-lm_b200/csrc/gdn_prefill.cu), against the oracle's token-by-token recurrence (ssm_step,
cpu_ops.cpp:131-146, or the decay-first order of export_hybrid_chunks.py:142-147).

Per 64-token chunk with state S0 at its start, lc the in-chunk cumulative log decay and
lt = lc shifted by one token (cpu_ops order) or lc itself (decay first):
  A_ti = beta_t e^{lt_t - lc_i} k_t.k_i (i < t),  T = (I + A)^-1,
  W = T diag(beta e^lt) K,  U = T diag(beta) V,  M_ti = e^{lc_t - lc_i} q_t.k_i (i <= t)
(gdn_pf_chunk_kernel), then along the chunks (gdn_pf_chain_tc_kernel)
  D = U - W S0,  Y = diag(e^lc) Q S0 + M D,  S = e^{lc_last} S0 + K^T diag(e^{lc_last - lc}) D.
Tokens past the end are zero (k, v, q, beta, log g), which leaves the state unchanged.

The restatement runs twice: in float64 (the algebra alone, tight tolerance) and with every
tensor-core operand rounded the way the kernels round it -- 16-bit inputs as one plane, computed
operands as hi / lo pairs (fp16, or bf16 where an MMA meets bf16 inputs) except W, which meets the
state by its hi plane alone, each product as hi*hi + lo*hi + hi*lo in fp32, T by an fp32 solve,
S and D in fp32 -- over BASELINE config 4's 8192 tokens, within 1e-4 abs + 1e-3 rel (the GPU
tests allow 2e-3 + 1e-2).  CPU only; the GPU tests check the
kernels themselves."""
import numpy as np
import pytest

from helpers import assert_close
from oracle import pyoracle as po

CHUNK = 64


def bf16(x):
    """Round float32 to the nearest bfloat16 (ties to even), returned as float32."""
    u = np.asarray(x, np.float32).view(np.uint32).astype(np.uint64)
    u = ((u + 0x7FFF + ((u >> 16) & 1)) >> 16) << 16
    return u.astype(np.uint32).view(np.float32)


def f16(x):
    return np.asarray(x, np.float32).astype(np.float16).astype(np.float32)


ROUND = {"f16": f16, "bf16": bf16}


def split(x, kind):
    """hi / lo pair of a computed fp32 operand: hi = round(x), lo = round(x - hi)."""
    x = np.asarray(x, np.float32)
    hi = ROUND[kind](x)
    return hi, ROUND[kind](x - hi)


def mma(a, b):
    """Product of two operands given as plane tuples ((hi,) for exact 16-bit values, (hi, lo)
    for pairs): hi*hi + lo*hi + hi*lo, the lo*lo term dropped, fp32 sums."""
    out = a[0] @ b[0]
    if len(a) > 1:
        out = out + a[1] @ b[0]
    if len(b) > 1:
        out = out + a[0] @ b[1]
    return out


def chunk_form(q, k, v, lg, beta, s0, hf, inputs=None, pairs=True):
    """One value head: q, k [T][dk] (its key head), v [T][dv], lg, beta [T], s0 [dk][dv].
    inputs None: float64 algebra; "f16" / "bf16": the kernels' operand rounding for inputs of
    that type (pairs False: computed operands as one 16-bit plane, for comparison).  Returns
    y [T][dv] and the final state."""
    T = len(q)
    n = -(-T // CHUNK) * CHUNK
    ft = np.float64 if inputs is None else np.float32

    def pad(a):
        out = np.zeros((n,) + a.shape[1:], ft)
        out[:T] = a
        return out

    q, k, v, lg, beta = (pad(a) for a in (q, k, v, lg, beta))
    S = np.array(s0, ft)
    comp = "bf16" if inputs == "bf16" else "f16"  # computed operands meeting the inputs

    def sp(x, kind):
        return split(x, kind) if pairs else split(x, kind)[:1]

    below = np.tril(np.ones((CHUNK, CHUNK), bool), -1)
    upto = np.tril(np.ones((CHUNK, CHUNK), bool))
    y = np.zeros((n, v.shape[1]), ft)
    for c0 in range(0, n, CHUNK):
        Q, K, V = q[c0:c0 + CHUNK], k[c0:c0 + CHUNK], v[c0:c0 + CHUNK]
        b = beta[c0:c0 + CHUNK]
        lc = np.cumsum(lg[c0:c0 + CHUNK]).astype(ft)
        lt = lc if hf else np.concatenate([[0.0], lc[:-1]]).astype(ft)
        # decay ratios only: every exponent used below is <= 0
        e_a = np.exp(np.minimum(lt[:, None] - lc[None, :], 0)) * below
        e_m = np.exp(np.minimum(lc[:, None] - lc[None, :], 0)) * upto
        if inputs is None:
            KK, QK = K @ K.T, Q @ K.T
        else:  # GEMM 1: exact 16-bit K and Q, one term
            KK, QK = mma((K,), (K.T,)), mma((Q,), (K.T,))
        A = (b[:, None] * e_a * KK).astype(ft)
        Tm = np.linalg.solve(np.eye(CHUNK, dtype=ft) + A, np.eye(CHUNK, dtype=ft)).astype(ft)
        Tp = Tm * (b * np.exp(lt))[None, :]
        Tpp = Tm * b[None, :]
        M = (e_m * QK).astype(ft)
        G = np.exp(lc[-1] - lc).astype(ft)
        if inputs is None:
            W, U = Tp @ K, Tpp @ V
            D = U - W @ S
            y[c0:c0 + CHUNK] = np.exp(lc)[:, None] * (Q @ S) + M @ D
            S = np.exp(lc[-1]) * S + K.T @ (G[:, None] * D)
        else:
            # GEMM 2: [T'; T''] as hi / lo pairs against exact K | V
            W, U = mma(sp(Tp, comp), (K,)), mma(sp(Tpp, comp), (V,))
            Sp = sp(S, comp)
            QS, WS = mma((Q,), Sp), mma(sp(W, comp)[:1], Sp)  # A = [Q; W] S, W by its hi plane
            D = U - WS
            MD = mma(sp(M, "f16"), sp(D, "f16"))  # B = M D stays fp16
            y[c0:c0 + CHUNK] = np.exp(lc)[:, None] * QS + MD
            S = np.float32(np.exp(lc[-1])) * S + mma((K.T,), sp(G[:, None] * D, comp))  # C = K^T Gamma D
    return y[:T], S


def inputs_cfg4(rng, T, Hk, Hv, kind):
    """BASELINE config 4 distributions: q, k L2-normalised rows (q also / sqrt(128)), v N(0, 1),
    log g ~ U(-0.1, 0), beta ~ U(0, 1), all of q / k / v representable in `kind`; state N(0, 0.1)."""
    def unit(x):
        return x / np.linalg.norm(x, axis=-1, keepdims=True)
    r = ROUND[kind]
    q = r(unit(rng.standard_normal((T, Hk, 128))) / np.sqrt(128.0))
    k = r(unit(rng.standard_normal((T, Hk, 128))))
    v = r(rng.standard_normal((T, Hv, 128)))
    lg = (-0.1 * rng.random((T, Hv))).astype(np.float32)
    beta = rng.random((T, Hv)).astype(np.float32)
    s0 = (0.1 * rng.standard_normal((Hv, 128, 128))).astype(np.float32)
    return q, k, v, lg, beta, s0


def run_chunks(q, k, v, lg, beta, s0, hf, inputs=None, pairs=True):
    Hk, Hv = q.shape[1], v.shape[1]
    ys, ss = [], []
    for h in range(Hv):
        kh = h // (Hv // Hk)  # value head h reads key head h / (Hv / Hk), qwen3_5.cpp:891
        y, s = chunk_form(q[:, kh], k[:, kh], v[:, h], lg[:, h], beta[:, h], s0[h], hf, inputs, pairs)
        ys.append(y)
        ss.append(s)
    return np.stack(ys, 1), np.stack(ss)


@pytest.mark.parametrize("hf", [0, 1])
@pytest.mark.parametrize("T", [1, 63, 64, 65, 200])
def test_chunk_algebra_equals_token_recurrence(hf, T):
    rng = np.random.default_rng(300 + T + 11 * hf)
    q, k, v, lg, beta, s0 = inputs_cfg4(rng, T, 2, 4, "f16")
    st = s0.copy()
    want = po.gated_delta_tokens("oracle", q, k, v, lg, beta, st, hf)
    y, s = run_chunks(q, k, v, lg, beta, s0, hf)
    assert_close(y, want, atol=2e-5, rtol=1e-4, what=f"y, float64 chunk form (hf={hf}, T={T})")
    assert_close(s, st, atol=2e-5, rtol=1e-4, what=f"state, float64 chunk form (hf={hf}, T={T})")


@pytest.mark.parametrize("inputs", ["f16", "bf16"])
@pytest.mark.parametrize("hf", [0, 1])
def test_kernel_operand_format_over_config4_length(hf, inputs):
    """8192 tokens (128 chunk steps) of one value head with the kernels' operand rounding: the
    hi / lo products keep outputs and state within 1e-4 + 1e-3 rel of the recurrence after 128
    chunk steps (the GPU tests allow 2e-3 + 1e-2 rel; measured ~3e-6 with fp16 inputs, ~2e-5
    with bf16), where one 16-bit plane per computed operand drifts past it (fp16: ~5e-5 in y,
    ~4e-4 in the state; bf16: ~3e-4 and ~2e-3)."""
    rng = np.random.default_rng(40 + hf + 2 * (inputs == "bf16"))
    q, k, v, lg, beta, s0 = inputs_cfg4(rng, 8192, 1, 1, inputs)
    st = s0.copy()
    want = po.gated_delta_tokens("oracle", q, k, v, lg, beta, st, hf)
    y, s = run_chunks(q, k, v, lg, beta, s0, hf, inputs)
    tight = dict(atol=1e-4, rtol=1e-3)
    assert_close(y, want, **tight, what=f"y, {inputs} operand pairs (hf={hf})")
    assert_close(s, st, **tight, what=f"state, {inputs} operand pairs (hf={hf})")
    y1, s1 = run_chunks(q, k, v, lg, beta, s0, hf, inputs, pairs=False)
    with pytest.raises(AssertionError):
        assert_close(s1, st, **tight, what="state, one plane per operand")


def test_split_products_keep_the_pair_precision():
    """A hi / lo pair carries 22 significant bits in fp16 and 16 in bf16; a three-term product
    of two pairs is that accurate relative to the float64 product, one plane alone is not."""
    rng = np.random.default_rng(7)
    a = rng.standard_normal((64, 128)).astype(np.float32)
    b = rng.standard_normal((128, 32)).astype(np.float32)
    exact = a.astype(np.float64) @ b.astype(np.float64)
    scale = np.abs(a).astype(np.float64) @ np.abs(b).astype(np.float64)

    def rel(got):
        return float(np.max(np.abs(got - exact) / scale))

    assert rel(mma(split(a, "f16"), split(b, "f16"))) < 2.0 ** -19
    assert rel(mma(split(a, "bf16"), split(b, "bf16"))) < 2.0 ** -14
    assert rel(mma((f16(a),), (f16(b),))) > 2.0 ** -14  # fp16 operands alone: ~2^-11

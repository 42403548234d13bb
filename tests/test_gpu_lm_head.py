"""GPU parity of the LM head with in-model top-k (anelm_lm_head_topk; LMHeadArgmax of
scripts/export_hybrid_chunks.py:409-421) against torch.topk over a plain PyTorch fp32 matmul of
the same bf16 operands: the values agree within fp32 accumulation-order rounding (1e-4 of the
row scale), and every returned index is a top-k index of the reference up to near-ties (its
reference logit is within that tolerance of the k-th largest).  Qwen3.5 vocabulary (248,320) at
hidden 2560 for one row (CUDA-core path) and batches (tensor-core path); a ragged vocabulary
(three rows) and k < 32."""
import pytest

torch = pytest.importorskip("torch")

from anelm_b200.core import lm_head_topk  # noqa: E402

pytestmark = pytest.mark.gpu


def _check(n, vocab, hidden, k, seed):
    g = torch.Generator(device="cuda")
    g.manual_seed(seed)
    h = torch.randn(n, hidden, generator=g, device="cuda").to(torch.bfloat16)
    w = (torch.randn(vocab, hidden, generator=g, device="cuda") / hidden ** 0.5).to(torch.bfloat16)
    vals, idx = lm_head_topk(h, w, k)
    logits = h.float() @ w.float().T
    want_v, want_i = torch.topk(logits, k, dim=-1)
    scale = logits.abs().amax(dim=-1, keepdim=True)
    tol = 1e-4 * scale
    assert ((vals - want_v).abs() <= tol).all(), float(((vals - want_v).abs() / scale).max())
    assert (vals[:, :-1] >= vals[:, 1:]).all()          # sorted descending
    got_logit = logits.gather(1, idx.long())          # the reference logit of every returned index
    assert (got_logit >= want_v[:, -1:] - tol).all()
    assert ((got_logit - vals).abs() <= tol).all()
    assert all(len(set(r.tolist())) == k for r in idx)  # no index twice


@pytest.mark.parametrize("n", [1, 4, 5, 8, 9, 16, 17, 24, 25, 33, 64, 65, 256])
def test_lm_head_top32_qwen_vocab(n):
    """One row takes the CUDA-core path (weights streamed, per-warp running top-32), 2-8 rows the
    swapped-role kernel, more rows the tensor-core tile kernel: 9-24 rows with four copies of the row
    block in the A tile (each epilogue warp takes a quarter of every tile's columns), others with one
    (256: two row tiles).  The tile kernel's lists only take logits at or above the bound built from
    every CTA's first-tile maxima."""
    _check(n, 248320, 2560, 32, seed=n)


@pytest.mark.parametrize("k", [1, 5, 32])
@pytest.mark.parametrize("n", [1, 3, 17, 40])
def test_lm_head_ragged_vocab(n, k):
    """A 1,000-row vocabulary (four 256-column tiles, the last one partial) at hidden 136 (a partial
    64-wide k-step): the GEMV, swapped and tile kernels; the tile kernel runs four CTAs here, fewer
    than the 32 groups its first-tile bound needs, so its lists take every logit."""
    _check(n, 1000, 136, k, seed=k + 10 * n)


@pytest.mark.parametrize("n", [17, 40])
def test_lm_head_ragged_vocab_with_bound(n):
    """34 vocabulary tiles (8,548 rows, the last tile 100 columns): 34 CTAs, enough for the
    first-tile bound, with a partial tile among them."""
    _check(n, 33 * 256 + 100, 136, 32, seed=500 + n)


@pytest.mark.parametrize("n", [2, 8, 16])
def test_lm_head_wide_hidden_few_rows(n):
    """2-8 rows take the swapped-role kernel only while the rows of h fit its shared memory (hidden up
    to about 3,100); at hidden 4,096 they fall back to the tensor-core tile kernel with one copy of the
    row block (16 rows: four copies) -- that path, against the same reference."""
    _check(n, 32768, 4096, 32, seed=100 + n)


@pytest.mark.parametrize("n", [16, 32, 128])
def test_lm_head_ties_exact(n):
    """Integer logits (h, W in {-1, 0, 1}, hidden 256: exact in fp32 whatever the summation order) with
    about a dozen vocabulary rows per value near the top, so the 32nd value is tied across rows that
    land in different CTAs' lists.  The tile kernel's lists and the merge order by (value descending,
    index ascending) and keep logits equal to the first-tile bound, so the result is exactly the first
    32 of that order: values and indices."""
    import numpy as np

    g = torch.Generator(device="cuda")
    g.manual_seed(7 + n)
    vocab, hidden = 248320, 256
    h = torch.randint(-1, 2, (n, hidden), generator=g, device="cuda").to(torch.bfloat16)
    w = torch.randint(-1, 2, (vocab, hidden), generator=g, device="cuda").to(torch.bfloat16)
    vals, idx = lm_head_topk(h, w, 32)
    logits = (h.float() @ w.float().T).cpu().numpy()
    cols = np.arange(vocab)
    for r in range(n):
        order = np.lexsort((cols, -logits[r]))[:32]
        assert np.array_equal(idx[r].cpu().numpy(), order), r
        assert np.array_equal(vals[r].cpu().numpy(), logits[r][order]), r
    # the boundary is tied: the 32nd value also appears beyond the first 32
    assert any((logits[r] == logits[r][np.lexsort((cols, -logits[r]))[31]]).sum() > 1 for r in range(n))

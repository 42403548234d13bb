"""GPU numerics of the tcgen05 bf16 projection GEMM (anelm_gemm_bf16) against a plain PyTorch
fp32 matmul of the same bf16 operands: the decode shapes of the Qwen3.5-4B projections around
the attention core (first_proj rows in, o_proj out), ragged M / N / K (TMA zero fill, masked
stores), and every output dtype.  Tolerance: 1e-3 relative to the row's scale (fp32 accumulation
in a different order; bf16 / fp16 outputs add their own rounding)."""
import pytest

torch = pytest.importorskip("torch")

import anelm_b200 as ab  # noqa: E402
from anelm_b200.core import gemm_bf16  # noqa: E402

pytestmark = pytest.mark.gpu


def _check(M, N, K, out_dtype, seed=0):
    g = torch.Generator(device="cuda")
    g.manual_seed(seed)
    a = torch.randn(M, K, generator=g, device="cuda").to(torch.bfloat16)
    b = (torch.randn(N, K, generator=g, device="cuda") / K ** 0.5).to(torch.bfloat16)
    got = gemm_bf16(a, b, out_dtype).float()
    want = a.float() @ b.float().T
    scale = want.abs().amax().clamp_min(1e-6)
    tol = {torch.float32: 1e-4, torch.float16: 2e-3, torch.bfloat16: 1e-2}[out_dtype]
    err = float(((got - want).abs() / scale).amax())
    assert err < tol, (M, N, K, out_dtype, err)


@pytest.mark.parametrize("M,N,K", [(256, 10240, 2560), (1, 2560, 4096), (256, 2560, 4096)])
def test_gemm_projection_shapes(M, N, K):
    """4B shapes: full-attention first_proj (16 q+gate heads + 2 x 4 kv heads of 256 = 10240 rows
    from hidden 2560), o_proj (4096 -> 2560) at batch 256 and batch 1."""
    _check(M, N, K, torch.float32)


@pytest.mark.parametrize("out_dtype", [torch.float32, torch.bfloat16])
@pytest.mark.parametrize("M,N,K", [(4096, 2560, 128), (2304, 5000, 64)])
def test_gemm_multi_wave_persistent(M, N, K, out_dtype):
    """Several waves of 256-wide tiles run persistent CTAs (two TMEM accumulators, each tile's
    epilogue beside the next tile's MMAs) over bands of 16 row tiles: two full bands (4096 rows),
    and a full band plus a partial one of 2 row tiles (2304 rows, ragged N)."""
    _check(M, N, K, out_dtype, seed=M + N)


@pytest.mark.parametrize("out_dtype", [torch.float32, torch.float16, torch.bfloat16])
@pytest.mark.parametrize("M,N,K", [(1, 12352, 2560), (4, 10240, 2560), (2, 2561, 4096), (3, 17, 8)])
def test_gemm_few_rows(M, N, K, out_dtype):
    """1-4 rows take the CUDA-core path that streams the weights (single-sequence layer steps):
    decode shapes, an odd row count N, and a K of one 16-byte chunk."""
    _check(M, N, K, out_dtype, seed=M * N)


@pytest.mark.parametrize("out_dtype", [torch.float32, torch.bfloat16])
@pytest.mark.parametrize("M,N,K", [(256, 12352, 2560), (256, 10240, 2560), (1024, 5000, 256)])
def test_gemm_narrow_tiles(M, N, K, out_dtype):
    """Shapes whose 256-wide tiles would leave SMs idle take narrower tiles: DeltaNet in-projection
    (12352 rows: 176-wide tiles, a 16-column TMEM tail and a ragged last tile), full-attention
    in-projection (144-wide), and a 1024 x 5000 case; fp32 and 16-bit (vector-store tail) outputs."""
    _check(M, N, K, out_dtype, seed=N)


@pytest.mark.parametrize("out_dtype", [torch.float32, torch.float16, torch.bfloat16])
@pytest.mark.parametrize("M,N,K", [(77, 200, 136), (130, 129, 72), (3, 64, 40)])
def test_gemm_ragged(M, N, K, out_dtype):
    _check(M, N, K, out_dtype, seed=M + N + K)


def test_gemm_rejects_unaligned_rows():
    a = torch.zeros(4, 13, device="cuda", dtype=torch.bfloat16)   # row stride 13 elements: not 16-byte
    b = torch.zeros(8, 13, device="cuda", dtype=torch.bfloat16)
    with pytest.raises(ab.AnelmError) as e:
        gemm_bf16(a, b)
    assert e.value.status == ab.ERR_UNSUPPORTED

"""The tcgen05 bf16 GEMM (bt_gemm_bf16) against a float64 product of the same bf16
operands, for every operand-major combination and ragged edges."""
import numpy as np
import pytest

pytestmark = pytest.mark.gpu

SHAPES = [(128, 128, 64), (256, 256, 256), (304, 200, 136), (128, 64, 8272), (16384, 256, 256),
          (8, 8, 8)]


@pytest.mark.parametrize("shape", SHAPES, ids=[f"{m}x{n}x{k}" for m, n, k in SHAPES])
@pytest.mark.parametrize("a_mn", [0, 1])
@pytest.mark.parametrize("b_mn", [0, 1])
def test_umma_gemm_matches_a_reference_product(shape, a_mn, b_mn):
    import torch

    from boonta_b200 import _lib

    m, n, k = shape
    g = torch.Generator(device="cuda").manual_seed(m * 7 + n * 3 + k)
    a = torch.randn(m, k, device="cuda", generator=g).to(torch.bfloat16)
    b = torch.randn(n, k, device="cuda", generator=g).to(torch.bfloat16)
    a_in = a.t().contiguous() if a_mn else a.contiguous()
    b_in = b.t().contiguous() if b_mn else b.contiguous()
    d = torch.full((m, n), float("nan"), device="cuda")
    _lib.check(_lib.lib().bt_gemm_bf16(a_in.data_ptr(), b_in.data_ptr(), d.data_ptr(), m, n, k,
                                       a_mn, b_mn, 1, None, torch.cuda.current_stream().cuda_stream))
    torch.cuda.synchronize()
    ref = (a.double() @ b.double().t()).cpu().numpy()
    out = d.cpu().numpy()
    assert np.isfinite(out).all()
    np.testing.assert_allclose(out, ref, rtol=1e-4, atol=1e-4 * np.sqrt(k))


@pytest.mark.parametrize("shape", SHAPES[:4], ids=[f"{m}x{n}x{k}" for m, n, k in SHAPES[:4]])
@pytest.mark.parametrize("a_mn", [0, 1])
@pytest.mark.parametrize("b_mn", [0, 1])
def test_split_bf16_gemm_reaches_fp32_accuracy(shape, a_mn, b_mn):
    """x = hi + lo pairs; hi*hi + hi*lo + lo*hi carries ~16 mantissa bits, so the result
    matches the float64 product of the fp32 operands to ~1e-5 relative."""
    import torch

    from boonta_b200 import _lib

    m, n, k = shape
    g = torch.Generator(device="cuda").manual_seed(m + n + k)
    a = torch.randn(m, k, device="cuda", generator=g)
    b = torch.randn(n, k, device="cuda", generator=g)

    def split(x):
        hi = x.to(torch.bfloat16)
        lo = (x - hi.float()).to(torch.bfloat16)
        return hi, lo

    a_in = a.t().contiguous() if a_mn else a
    b_in = b.t().contiguous() if b_mn else b
    (ah, al), (bh, bl) = split(a_in), split(b_in)
    d = torch.full((m, n), float("nan"), device="cuda")
    _lib.check(_lib.lib().bt_gemm_bf16x3(ah.data_ptr(), al.data_ptr(), bh.data_ptr(), bl.data_ptr(),
                                         d.data_ptr(), m, n, k, a_mn, b_mn,
                                         torch.cuda.current_stream().cuda_stream))
    torch.cuda.synchronize()
    ref = (a.double() @ b.double().t()).cpu().numpy()
    out = d.cpu().numpy()
    err = np.linalg.norm(out - ref) / np.linalg.norm(ref)
    assert err < 3e-5, err

"""Fused MLA KV decompression (ats/model/mla_triton.py) on the tensor-core GEMM.

(k, v) = (c w_uk^T, c w_uv^T) runs as one GEMM against [w_uk; w_uv] with
float32 accumulation and one rounding to bf16.  Forward and backward are
compared with float64 products of the same bf16 operands, rounded once to
bf16 (almost every element bit-equal; the rest within the bf16 tolerance
2e-2 relative / 1e-2 absolute).  The reference's own kernel test (fp32, tiny
shapes, atol 1e-5) runs as written; those shapes take torch's GEMM."""

from __future__ import annotations

import pytest
import torch

from ats_v2_b200 import _lib
from ats_v2_b200.mla_fused import _triton_matmul, fused_mla_kv_decompress
from tests.util import close, np32

pytestmark = pytest.mark.gpu


def _ref64(c, w):
    return (c.double() @ w.double().t()).float().bfloat16()


@pytest.mark.parametrize("lead,latent,out", [((2, 150), 512, 1024), ((1, 128), 128, 128), ((3, 1000), 256, 384)])
def test_bf16_decompress_on_the_tensor_cores(lead, latent, out):
    rows = lead[0] * lead[1]
    assert _lib.query("ats_gemm_supported", _lib.ATS_BF16, rows, 2 * out, latent) == 1
    g = torch.Generator(device="cuda").manual_seed(rows + latent)
    c = torch.randn(*lead, latent, device="cuda", generator=g).bfloat16().requires_grad_()
    w_uk = (0.05 * torch.randn(out, latent, device="cuda", generator=g)).bfloat16().requires_grad_()
    w_uv = (0.05 * torch.randn(out, latent, device="cuda", generator=g)).bfloat16().requires_grad_()
    before = _lib.query("ats_kernel_launches")
    k, v = fused_mla_kv_decompress(c, w_uk, w_uv)
    assert _lib.query("ats_kernel_launches") > before  # the library GEMM ran
    assert k.shape == (*lead, out) and v.shape == (*lead, out) and k.dtype == torch.bfloat16
    c2 = c.detach().reshape(-1, latent)
    close(k.reshape(-1, out), np32(_ref64(c2, w_uk.detach())), "bf16", min_exact=0.98)
    close(v.reshape(-1, out), np32(_ref64(c2, w_uv.detach())), "bf16", min_exact=0.98)
    dk = torch.randn_like(k)
    dv = torch.randn_like(v)
    torch.autograd.backward([k, v], [dk, dv])
    dk2, dv2 = dk.reshape(-1, out).double(), dv.reshape(-1, out).double()
    dc_ref = (dk2 @ w_uk.detach().double() + dv2 @ w_uv.detach().double()).float().bfloat16()
    close(c.grad.reshape(-1, latent), np32(dc_ref), "bf16", min_exact=0.95)
    close(w_uk.grad, np32((dk2.t() @ c2.double()).float().bfloat16()), "bf16", min_exact=0.95)
    close(w_uv.grad, np32((dv2.t() @ c2.double()).float().bfloat16()), "bf16", min_exact=0.95)


def test_other_shapes_and_dtypes_use_the_library_gemm():
    g = torch.Generator(device="cuda").manual_seed(3)
    c = torch.randn(2, 5, 8, device="cuda", generator=g)
    w_uk = torch.randn(16, 8, device="cuda", generator=g)
    w_uv = torch.randn(16, 8, device="cuda", generator=g)
    k, v = fused_mla_kv_decompress(c, w_uk, w_uv)
    torch.testing.assert_close(k, c @ w_uk.t(), rtol=1e-5, atol=1e-5)
    torch.testing.assert_close(v, c @ w_uv.t(), rtol=1e-5, atol=1e-5)
    assert _lib.query("ats_gemm_supported", _lib.ATS_BF16, 100, 256, 256) == 0  # fewer than 128 rows
    assert _lib.query("ats_gemm_supported", _lib.ATS_F32, 1024, 256, 256) == 0


def test_reference_kernel_test_as_written():
    """tests/test_triton.py:194-207 of the reference."""
    torch.manual_seed(0)
    c = torch.randn(2, 8, 16, device="cuda")
    w_uk = torch.randn(32, 16, device="cuda")
    torch.randn(32, 16, device="cuda")
    k_triton = _triton_matmul(c.reshape(-1, 16), w_uk.t()).reshape(2, 8, 32)
    k_pytorch = c @ w_uk.t()
    assert torch.allclose(k_triton, k_pytorch, atol=1e-5)

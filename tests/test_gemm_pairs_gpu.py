"""The expert, dense-FFN and MLA GEMMs on CTA pairs (256-row tiles, tcgen05
cta_group::2, each SM of the pair holding half of the B tile) against the same
GEMMs on single CTAs (128-row tiles): every output and gradient must be bit-
identical.  The tile shape changes only which SM computes a row; each output
element is the same K-ordered sum of the same products.

The shapes cover the pair tiles' edge cases: an odd number of 128-row blocks
(the last pair tile's second half lies past the rows and is not stored), expert
segments of odd 128-row counts in the M-grouped GEMMs, weight-gradient outputs
whose row count is an odd multiple of 128 (K-grouped), an ffn size that is an
odd multiple of 128 (256-wide tiles with a zero-filled upper half), and an
expert that receives no rows (tiles with no K blocks write zeros)."""

from __future__ import annotations

import pytest
import torch

from ats_v2_b200 import _lib
from ats_v2_b200.ep import ExpertParallelMoE
from ats_v2_b200.mla_fused import fused_mla_kv_decompress
from ats_v2_b200.moe import dense_swiglu

pytestmark = pytest.mark.gpu


def _both(run):
    with _lib.gemm_pairs(True):
        a = run()
    torch.cuda.synchronize()
    with _lib.gemm_pairs(False):
        b = run()
    torch.cuda.synchronize()
    _lib.check_device_status("the pair comparison")
    return a, b


@pytest.mark.parametrize("T,H,F", [(1100, 384, 384), (4096, 512, 1408), (128, 256, 256), (2000, 1024, 640)])
def test_dense_ffn_pairs_equal_single_ctas(T, H, F):
    g = torch.Generator(device="cuda").manual_seed(T + H + F)
    x = torch.randn(T, H, device="cuda", generator=g).bfloat16()
    wgu = (0.05 * torch.randn(2 * F, H, device="cuda", generator=g)).bfloat16()
    wd = (0.05 * torch.randn(H, F, device="cuda", generator=g)).bfloat16()
    dy = torch.randn(T, H, device="cuda", generator=g).bfloat16()

    def run():
        xa, wa, wb = (t.clone().requires_grad_() for t in (x, wgu, wd))
        out = dense_swiglu(xa, wa, wb)
        out.backward(dy)
        return out.detach(), xa.grad, wa.grad, wb.grad

    a, b = _both(run)
    for name, u, v in zip(("out", "dx", "dw_gate_up", "dw_down"), a, b):
        assert torch.equal(u, v), f"{name}: CTA pairs and single CTAs differ"


@pytest.mark.parametrize("T,H,F,E,cf", [(700, 384, 384, 8, 1.25), (3000, 256, 1408, 16, 2.0)])
def test_routed_experts_pairs_equal_single_ctas(T, H, F, E, cf):
    torch.manual_seed(T)
    with torch.device("cuda"):
        layer = ExpertParallelMoE(H, F, E, num_layers=2, top_k=2, capacity_factor=cf)
    with torch.no_grad():
        layer.gate.weight.normal_(0, 0.05)
        for ex in layer.experts:
            ex.gate_up_proj.weight.normal_(0, 0.05)
            ex.down_proj.weight.normal_(0, 0.05)
    layer.experts.to(torch.bfloat16)
    bias = torch.zeros(E, device="cuda")
    bias[3] = -1e4  # expert 3 receives no rows: its weight-gradient tiles have no K blocks
    bias[5] = 2.0   # expert 5 overflows its capacity
    g = torch.Generator(device="cuda").manual_seed(T + 1)
    x = torch.randn(1, T, H, device="cuda", generator=g).bfloat16()
    dy = torch.randn(1, T, H, device="cuda", generator=g).bfloat16()

    def run():
        for p in layer.parameters():
            p.grad = None
        xa = x.clone().requires_grad_()
        out, aux = layer(xa, logit_bias=bias)
        torch.autograd.backward([out, aux], [dy, torch.ones_like(aux)])
        grads = [xa.grad] + [p.grad.clone() for p in layer.experts.parameters()] + [layer.gate.weight.grad.clone()]
        return [out.detach()] + grads

    a, b = _both(run)
    assert len(a) == len(b)
    for i, (u, v) in enumerate(zip(a, b)):
        assert torch.equal(u, v), f"tensor {i}: CTA pairs and single CTAs differ"
    assert float(a[1 + 1 + 2 * 3].abs().max()) == 0.0  # expert 3's gate/up weight gradient: no rows, zeros


@pytest.mark.parametrize("lead,latent,out", [((2, 333), 512, 1024), ((1, 1000), 1024, 2048)])
def test_mla_decompression_pairs_equal_single_ctas(lead, latent, out):
    g = torch.Generator(device="cuda").manual_seed(latent + out)
    c = torch.randn(*lead, latent, device="cuda", generator=g).bfloat16()
    w_uk = (0.03 * torch.randn(out, latent, device="cuda", generator=g)).bfloat16()
    w_uv = (0.03 * torch.randn(out, latent, device="cuda", generator=g)).bfloat16()
    gk = torch.randn(*lead, out, device="cuda", generator=g).bfloat16()
    gv = torch.randn(*lead, out, device="cuda", generator=g).bfloat16()

    def run():
        ca, ka, va = (t.clone().requires_grad_() for t in (c, w_uk, w_uv))
        k, v = fused_mla_kv_decompress(ca, ka, va)
        torch.autograd.backward([k, v], [gk, gv])
        return k.detach(), v.detach(), ca.grad, ka.grad, va.grad

    a, b = _both(run)
    for name, u, v in zip(("k", "v", "dc", "dw_uk", "dw_uv"), a, b):
        assert torch.equal(u, v), f"{name}: CTA pairs and single CTAs differ"

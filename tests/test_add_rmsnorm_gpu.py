"""The residual add fused with the RMSNorm after it (``fused_add_rmsnorm``,
``ats_add_rmsnorm_fwd/bwd``), the post-attention step of TransformerBlock
(ats/model/transformer.py:208-212), against the oracle: s = round(x +
residual), y the RMSNorm of s, and in the backward the RMSNorm gradient
rounded, then the gradient that reaches s from the next residual add added --
the order in which autograd sums the two.  Also checked against the unfused
pair (a torch add, then the RMSNorm kernels) inside a block-shaped autograd
graph."""

from __future__ import annotations

import numpy as np
import pytest
import torch

from ats_v2_b200.norm import RMSNorm
from ats_v2_b200.norm_fused import fused_add_rmsnorm
from oracle import norm as onorm
from oracle.bf16 import round_to
from tests.util import close, close_f32_sum, dev, np32, seeded_normal

pytestmark = pytest.mark.gpu

TD = {"f32": torch.float32, "bf16": torch.bfloat16}


@pytest.mark.parametrize("rows,H", [(1, 8), (37, 1000), (256, 2048), (130, 4096), (4096, 4096)])
@pytest.mark.parametrize("xd,wd", [("bf16", "f32"), ("bf16", "bf16"), ("f32", "f32")])
def test_fused_add_rmsnorm_matches_the_oracle(rows, H, xd, wd):
    if xd == "f32" and H > 2048:
        pytest.skip("float32 rows of more than 2048 take the unfused kernels")
    seed = rows * 31 + H
    x = seeded_normal((rows, H), seed)
    res = seeded_normal((rows, H), seed + 1)
    w = seeded_normal((H,), seed + 2, 0.1, 1.0)
    dy = seeded_normal((rows, H), seed + 3)
    ds_in = seeded_normal((rows, H), seed + 4)
    x, res, dy, ds_in = (round_to(v, xd) for v in (x, res, dy, ds_in))
    w = round_to(w, wd)
    xt, rt = dev(x, TD[xd], True), dev(res, TD[xd], True)
    wt = dev(w, TD[wd], True)
    h, s = fused_add_rmsnorm(xt, rt, wt, 1e-5)
    es = round_to(x + res, xd)
    close(s, es, xd, min_exact=1.0)  # one rounding of the same sum: bit-exact
    ey, _ = onorm.rmsnorm_fwd(es, w, 1e-5, xd)
    close(h, ey, xd, min_exact=0.99 if xd == "bf16" else None)
    torch.autograd.backward([h, s], [dev(dy, TD[xd]), dev(ds_in, TD[xd])])
    edx, edw = onorm.rmsnorm_bwd(dy, es, w, 1e-5, xd, wd)
    eds = round_to(edx + ds_in, xd)
    close(xt.grad, eds, xd, atol=1e-5 if xd == "f32" else 1e-2)
    assert torch.equal(xt.grad, rt.grad)
    if wd == "f32":
        x64 = np.asarray(es, np.float64)
        r = 1.0 / np.sqrt(np.mean(x64 * x64, axis=-1, keepdims=True) + 1e-5)
        close_f32_sum(wt.grad, edw, np.sum(np.abs(np.asarray(dy, np.float64) * x64 * r), axis=0))
    else:
        close(wt.grad, edw, wd)


def test_fused_matches_the_unfused_block_step():
    """x = residual + attn_out; h = norm(x); next = x + f(h): the gradients reaching
    attn_out and residual through the fused op equal those of the unfused graph."""
    torch.manual_seed(0)
    T, H = 2048, 4096
    norm = RMSNorm(H, eps=1e-5).cuda()
    with torch.no_grad():
        norm.weight.add_(0.02 * torch.randn(H, device="cuda"))
    attn = torch.randn(T, H, device="cuda").bfloat16()
    resid = torch.randn(T, H, device="cuda").bfloat16()
    g = torch.randn(T, H, device="cuda").bfloat16()

    def run(fused):
        a, r = attn.clone().requires_grad_(), resid.clone().requires_grad_()
        norm.weight.grad = None
        if fused:
            h, x = fused_add_rmsnorm(a, r, norm.weight, norm.eps)
        else:
            x = r + a
            h = norm(x)
        out = x + h * 0.5  # the next residual add, with a stand-in FFN
        out.backward(g)
        return h.detach(), x.detach(), a.grad, r.grad, norm.weight.grad.clone()

    fh, fx, fa, fr, fw = run(True)
    uh, ux, ua, ur, uw = run(False)
    assert torch.equal(fx, ux)
    close(fh, np32(uh), "bf16", min_exact=0.99)
    close(fa, np32(ua), "bf16", min_exact=0.99)
    assert torch.equal(fa, fr)
    torch.testing.assert_close(fw, uw, rtol=1e-4, atol=1e-4 * float(uw.abs().max()))

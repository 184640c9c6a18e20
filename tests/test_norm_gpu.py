"""RMSNorm and fused RMSNorm+residual on the CUDA kernels vs the golden
vectors (reference outputs) and the numpy oracle.  Tolerances: float32 within
1e-5 relative, bfloat16 within 2e-2 relative / 1e-2 absolute."""

from __future__ import annotations

import numpy as np
import pytest
import torch

from ats_v2_b200.norm import RMSNorm, rms_norm
from ats_v2_b200.norm_fused import _cuda_rmsnorm_residual, fused_rmsnorm_residual
from oracle import norm as onorm
from oracle.bf16 import round_bf16
from tests.conftest import load_golden
from tests.util import close, close_f32_sum, dev, np32, seeded_normal

pytestmark = pytest.mark.gpu

TD = {"f32": torch.float32, "bf16": torch.bfloat16}


def _dw_abs_sum(dy, x, eps):
    """sum over rows of |dy * x * rstd| per column: the magnitude a float32 dw sum rounds at."""
    x64 = np.asarray(x, np.float64).reshape(-1, x.shape[-1])
    r = 1.0 / np.sqrt(np.mean(x64 * x64, axis=-1, keepdims=True) + eps)
    return np.sum(np.abs(np.asarray(dy, np.float64).reshape(x64.shape) * x64 * r), axis=0)


def _run(x_np, w_np, dy_np, eps, xd, wd):
    x = dev(x_np, TD[xd], requires_grad=True)
    m = RMSNorm(x_np.shape[-1], eps=eps).cuda().to(TD[wd])
    with torch.no_grad():
        m.weight.copy_(dev(w_np, TD[wd]))
    y = m(x)
    y.backward(dev(dy_np, TD[xd]))
    return y, x.grad, m.weight.grad


def test_golden_f32():
    g = load_golden("rmsnorm")
    y, dx, dw = _run(g["f32_x"], g["f32_w"], g["f32_dy"], 1e-6, "f32", "f32")
    close(y, g["f32_y"], "f32")
    close(dx, g["f32_dx"], "f32", atol=1e-5)
    close(dw, g["f32_dw"], "f32", atol=1e-5)


def test_golden_bf16_fp32_weight():
    g = load_golden("rmsnorm")
    y, dx, dw = _run(g["b_x"], g["b_w"], g["b_dy"], 1e-5, "bf16", "f32")
    assert y.dtype == torch.bfloat16 and dx.dtype == torch.bfloat16 and dw.dtype == torch.float32
    close(y, g["b_y"], "bf16", min_exact=0.99)
    close(dx, g["b_dx"], "bf16", min_exact=0.95)
    close(dw, g["b_dw"], "f32", rtol=1e-4, atol=1e-4)


def test_cpu_parity_workload_shape_f32():
    """The CPU parity workload's RMSNorm: x [4,256,512] fp32, w = 1+N(0,.02), eps 1e-6."""
    x = seeded_normal((4, 256, 512), 0)
    w = seeded_normal((512,), 1, 0.02, 1.0)
    dy = seeded_normal((4, 256, 512), 2)
    y, dx, dw = _run(x, w, dy, 1e-6, "f32", "f32")
    ey, _ = onorm.rmsnorm_fwd(x, w, 1e-6, "f32")
    edx, edw = onorm.rmsnorm_bwd(dy, x, w, 1e-6, "f32", "f32")
    close(y, ey, "f32")
    close(dx, edx, "f32", atol=1e-5)
    close_f32_sum(dw, edw, _dw_abs_sum(dy, x, 1e-6))


@pytest.mark.parametrize("rows,H", [(1, 6), (3, 16), (7, 100), (33, 1000), (130, 4096), (5, 8192), (2, 12288),
                                    (301, 2048), (777, 4096), (3, 4096)])
@pytest.mark.parametrize("xd,wd", [("f32", "f32"), ("bf16", "f32"), ("bf16", "bf16"), ("f32", "bf16")])
def test_shapes_and_dtypes(rows, H, xd, wd):
    seed = rows * 7919 + H
    x = seeded_normal((rows, H), seed)
    w = seeded_normal((H,), seed + 1, 0.1, 1.0)
    dy = seeded_normal((rows, H), seed + 2)
    if xd == "bf16":
        x, dy = round_bf16(x), round_bf16(dy)
    if wd == "bf16":
        w = round_bf16(w)
    y, dx, dw = _run(x, w, dy, 1e-5, xd, wd)
    ey, _ = onorm.rmsnorm_fwd(x, w, 1e-5, xd)
    edx, edw = onorm.rmsnorm_bwd(dy, x, w, 1e-5, xd, wd)
    close(y, ey, xd, min_exact=0.99 if xd == "bf16" else None)
    close(dx, edx, xd, atol=1e-5 if xd == "f32" else 1e-2)
    if wd == "f32":
        close_f32_sum(dw, edw, _dw_abs_sum(dy, x, 1e-5))
    else:
        close(dw, edw, wd)


def test_zero_rows_and_strided_input():
    w = torch.ones(64, device="cuda")
    x = torch.empty(0, 64, device="cuda", requires_grad=True)
    y = rms_norm(x, w.requires_grad_(), 1e-6)
    assert y.shape == (0, 64)
    y.sum().backward()
    assert torch.equal(w.grad, torch.zeros(64, device="cuda"))
    big = torch.randn(10, 96, device="cuda")
    xs = big[:, 16:80]  # row stride 96 > hidden 64
    ys = rms_norm(xs, torch.ones(64, device="cuda"), 1e-6)
    ref, _ = onorm.rmsnorm_fwd(np32(xs), np.ones(64, np.float32), 1e-6)
    close(ys, ref, "f32")


@pytest.mark.parametrize("H", [1024, 2048, 4096])
def test_dw_is_deterministic(H):
    torch.manual_seed(0)
    x = torch.randn(4096, H, device="cuda", dtype=torch.bfloat16, requires_grad=True)
    w = torch.nn.Parameter(torch.ones(H, device="cuda"))
    dy = torch.randn(4096, H, device="cuda", dtype=torch.bfloat16)
    grads = []
    for _ in range(2):
        w.grad = None
        rms_norm(x, w, 1e-5).backward(dy)
        grads.append(w.grad.clone())
    assert torch.equal(grads[0], grads[1])


def test_full_size_7b_config_sampled_rows():
    """x [4,4096,4096] bf16, w fp32, eps 1e-5: rows are independent, so 64
    sampled rows are checked against the oracle; dw against a float64 sum."""
    g = torch.Generator(device="cuda").manual_seed(0)
    x = torch.randn(4, 4096, 4096, device="cuda", generator=g).bfloat16().requires_grad_()
    w = (1 + 0.02 * torch.randn(4096, device="cuda", generator=g)).requires_grad_()
    dy = torch.randn(4, 4096, 4096, device="cuda", generator=g).bfloat16()
    y = rms_norm(x, w, 1e-5)
    y.backward(dy)
    rows = torch.randint(0, 16384, (64,), device="cuda", generator=g)
    xs, dys = np32(x.view(-1, 4096)[rows]), np32(dy.view(-1, 4096)[rows])
    ey, _ = onorm.rmsnorm_fwd(xs, np32(w), 1e-5, "bf16")
    edx, _ = onorm.rmsnorm_bwd(dys, xs, np32(w), 1e-5, "bf16", "f32")
    close(y.view(-1, 4096)[rows], ey, "bf16", min_exact=0.99)
    close(x.grad.view(-1, 4096)[rows], edx, "bf16")
    xd = x.detach().view(-1, 4096).double()
    r = torch.rsqrt(xd.pow(2).mean(-1, keepdim=True) + 1e-5)
    dw_ref = (dy.view(-1, 4096).double() * xd * r).sum(0)
    torch.testing.assert_close(w.grad.double(), dw_ref, rtol=1e-4, atol=1e-3)


# --------------------------------------------------------------- residual
def test_residual_golden_f32_reference_test_shape():
    g = load_golden("rmsnorm")
    x, res, w = (dev(g[k], requires_grad=True) for k in ("r32_x", "r32_res", "r32_w"))
    out = fused_rmsnorm_residual(x, res, w, 1e-6)
    close(out, g["r32_out"], "f32")
    out.backward(dev(g["r32_g"]))
    close(x.grad, g["r32_dx"], "f32", atol=1e-5)
    close(res.grad, g["r32_dres"], "f32")
    close(w.grad, g["r32_dw"], "f32", atol=1e-5)


def test_residual_golden_bf16():
    g = load_golden("rmsnorm")
    x, res, w = (dev(g[k], torch.bfloat16, requires_grad=True) for k in ("rb_x", "rb_res", "rb_w"))
    out = fused_rmsnorm_residual(x, res, w, 1e-6)
    assert out.dtype == torch.bfloat16
    close(out, g["rb_out"], "bf16", min_exact=0.99)
    out.backward(dev(g["rb_g"], torch.bfloat16))
    close(x.grad, g["rb_dx"], "bf16")
    close(res.grad, g["rb_dres"], "bf16", min_exact=1.0)
    close(w.grad, g["rb_dw"], "bf16")


def test_residual_reference_parity_test():
    """tests/test_triton.py:132-149 of the reference, on the CUDA kernel."""
    torch.manual_seed(0)
    x = torch.randn(4, 32, device="cuda")
    residual = torch.randn(4, 32, device="cuda")
    weight = torch.randn(32, device="cuda")
    out = _cuda_rmsnorm_residual(x, residual, weight, eps=1e-6)
    ref, _ = onorm.rmsnorm_residual_fwd(np32(x), np32(residual), np32(weight), 1e-6)
    assert torch.allclose(out, dev(ref), atol=1e-5)


@pytest.mark.parametrize("xd,wd", [("bf16", "f32"), ("f32", "bf16"), ("bf16", "bf16"), ("f32", "f32")])
def test_residual_mixed_dtypes(xd, wd):
    x = seeded_normal((9, 4096), 5)
    res = seeded_normal((9, 4096), 6)
    w = seeded_normal((4096,), 7, 0.1, 1.0)
    gout = seeded_normal((9, 4096), 8)
    if xd == "bf16":
        x, res = round_bf16(x), round_bf16(res)
    if wd == "bf16":
        w = round_bf16(w)
    od = "f32" if "f32" in (xd, wd) else "bf16"
    if od == "bf16":
        gout = round_bf16(gout)
    xt, rt, wt = dev(x, TD[xd], True), dev(res, TD[xd], True), dev(w, TD[wd], True)
    out = fused_rmsnorm_residual(xt, rt, wt, 1e-6)
    assert out.dtype == TD[od]
    eo, _ = onorm.rmsnorm_residual_fwd(x, res, w, 1e-6, xd, xd, wd)
    close(out, eo, od, min_exact=0.99 if od == "bf16" else None)
    out.backward(dev(gout, TD[od]))
    edx, edr, edw = onorm.rmsnorm_residual_bwd(gout, x, w, 1e-6, xd, xd, wd)
    close(xt.grad, edx, xd, atol=1e-5 if xd == "f32" else 1e-2)
    close(rt.grad, edr, xd)
    if wd == "f32":
        # n1 = (x*r) rounded to x's dtype: the terms of dw are gout*n1
        x64 = np.asarray(x, np.float64)
        r = 1.0 / np.sqrt(np.mean(x64 * x64, axis=-1, keepdims=True) + 1e-6)
        close_f32_sum(wt.grad, edw, np.sum(np.abs(np.asarray(gout, np.float64) * x64 * r), axis=0))
    else:
        close(wt.grad, edw, wd)

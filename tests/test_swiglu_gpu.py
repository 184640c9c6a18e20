"""Dense SwiGLU FFN (ats/model/ffn.py:37-45) on the tensor-core GEMMs.

The dense path runs the expert GEMMs once over the token rows (no routing,
gather or combine).  Its results must be bit-identical to the same FFN run as
a single routed expert with gate 1.0 -- the same GEMMs on the same rows,
where the combine multiplies by 1.0 and the un-permute sums one row -- and
its forward must match the oracle's SwiGLU (bf16 tolerance 2e-2 relative /
1e-2 absolute).  Token counts that are not multiples of 128 exercise the
clipped TMA stores and the zero rows past T."""

from __future__ import annotations

import numpy as np
import pytest
import torch

from ats_v2_b200 import _lib
from ats_v2_b200.ffn import SwiGLU
from ats_v2_b200.moe import dense_swiglu, routed_swiglu
from oracle import moe as omoe
from tests.util import close, np32

pytestmark = pytest.mark.gpu


def _weights(H, F, seed):
    g = torch.Generator(device="cuda").manual_seed(seed)
    wgu = (0.05 * torch.randn(2 * F, H, device="cuda", generator=g)).bfloat16()
    wd = (0.05 * torch.randn(H, F, device="cuda", generator=g)).bfloat16()
    return wgu, wd


@pytest.mark.parametrize("T,H,F", [(128, 128, 128), (300, 256, 384), (1024, 512, 1024), (4097, 256, 256)])
def test_dense_path_is_bit_identical_to_the_routed_single_expert(T, H, F):
    assert _lib.query("ats_swiglu_supported", _lib.ATS_BF16, T, H, F) == 1
    wgu, wd = _weights(H, F, T + H)
    g = torch.Generator(device="cuda").manual_seed(T)
    x = torch.randn(T, H, device="cuda", generator=g).bfloat16()
    dy = torch.randn(T, H, device="cuda", generator=g).bfloat16()
    res = []
    for fn in (dense_swiglu, routed_swiglu):
        xa = x.clone().requires_grad_()
        wa, wb = wgu.clone().requires_grad_(), wd.clone().requires_grad_()
        out = fn(xa, wa, wb)
        out.backward(dy)
        res.append((out.detach(), xa.grad, wa.grad, wb.grad))
    for name, a, b in zip(("out", "dx", "dw_gate_up", "dw_down"), res[0], res[1]):
        assert torch.equal(a, b), f"{name}: dense and routed paths differ"
    y_ref = omoe.expert_fwd(np32(x), np32(wgu), np32(wd), "bf16")[0]
    close(res[0][0], y_ref, "bf16")


def _swiglu_c_abi(x, wgu, wd, dy):
    """Forward and backward through the C ABI on this thread (autograd would run
    the backward on its own device thread, outside a thread's SM limit)."""
    T, H = x.shape
    F = wd.shape[1]
    st = _lib.stream_of(x)
    R = _lib.query("ats_swiglu_rows", T)
    wsb = _lib.query("ats_swiglu_workspace_bytes")
    ws = torch.empty(wsb, dtype=torch.uint8, device="cuda")
    h = torch.empty(R, 2 * F, dtype=x.dtype, device="cuda")
    a = torch.empty(R, F, dtype=x.dtype, device="cuda")
    y = torch.empty(T, H, dtype=x.dtype, device="cuda")
    _lib.call("ats_swiglu_fwd", x.data_ptr(), wgu.data_ptr(), wd.data_ptr(), h.data_ptr(), a.data_ptr(),
              y.data_ptr(), _lib.ATS_BF16, T, H, F, ws.data_ptr(), wsb, st)
    dh, dx = torch.empty_like(h), torch.empty_like(x)
    dwgu, dwd = torch.empty_like(wgu), torch.empty_like(wd)
    _lib.call("ats_swiglu_bwd", dy.data_ptr(), x.data_ptr(), h.data_ptr(), a.data_ptr(), wgu.data_ptr(),
              wd.data_ptr(), dh.data_ptr(), dx.data_ptr(), dwgu.data_ptr(), dwd.data_ptr(), _lib.ATS_BF16, T, H, F,
              ws.data_ptr(), wsb, st)
    return y, dx, dwgu, dwd


@pytest.mark.parametrize("sms", [1, 37, 147])
def test_fewer_gemm_ctas_give_the_same_bits(sms):
    """A GEMM held to fewer SMs computes the same tiles in another order
    across its CTAs: every output is bit-equal."""
    T, H, F = 1100, 256, 384
    wgu, wd = _weights(H, F, 7)
    g = torch.Generator(device="cuda").manual_seed(8)
    x = torch.randn(T, H, device="cuda", generator=g).bfloat16()
    dy = torch.randn(T, H, device="cuda", generator=g).bfloat16()
    full = _swiglu_c_abi(x, wgu, wd, dy)
    with _lib.gemm_sm_limit(sms):
        assert _lib.query("ats_gemm_sm_limit") == sms
        held = _swiglu_c_abi(x, wgu, wd, dy)
    for name, a, b in zip(("out", "dx", "dw_gate_up", "dw_down"), full, held):
        assert torch.equal(a, b), f"{name}: differs with the GEMMs on {sms} SMs"


def test_swiglu_module_forward_and_backward_against_the_oracle():
    T, H, F = 512, 256, 512
    torch.manual_seed(0)
    m = SwiGLU(H, F).cuda().bfloat16()
    x = torch.randn(2, T // 2, H, device="cuda").bfloat16().requires_grad_()
    out = m(x)
    y_ref = omoe.expert_fwd(np32(x.view(T, H)), np32(m.gate_up_proj.weight), np32(m.down_proj.weight), "bf16")[0]
    close(out.view(T, H), y_ref, "bf16")
    dy = torch.randn_like(out)
    out.backward(dy)
    # gradients against a float32 chain on the same bf16 values with the kernels' rounding points
    xs, d = x.detach().view(T, H).float(), dy.view(T, H).float()
    wgu, wd = m.gate_up_proj.weight.detach().float(), m.down_proj.weight.detach().float()
    hh = (xs @ wgu.T).bfloat16().float()
    gg, uu = hh[:, :F], hh[:, F:]
    s = torch.nn.functional.silu(gg).bfloat16().float()
    a = (s * uu).bfloat16().float()
    da = (d @ wd).bfloat16().float()
    sig = torch.sigmoid(gg)
    du = (da * s).bfloat16().float()
    ds = (da * uu).bfloat16().float()
    dg = (ds * sig * (1 + gg * (1 - sig))).bfloat16().float()
    dh = torch.cat([dg, du], dim=1)

    def rel(got, ref, what):
        scale = float(ref.abs().max())
        torch.testing.assert_close(got.float(), ref, rtol=2e-2, atol=2e-2 * scale, msg=lambda msg: f"{what}: {msg}")

    rel(x.grad.view(T, H), (dh @ wgu).bfloat16().float(), "dx")
    rel(m.down_proj.weight.grad, (d.T @ a).bfloat16().float(), "dW_down")
    rel(m.gate_up_proj.weight.grad, (dh.T @ xs).bfloat16().float(), "dW_gate_up")


def test_unsupported_shapes_take_the_routed_path():
    for T, H, F in [(100, 256, 256), (512, 200, 256), (512, 256, 200)]:
        assert _lib.query("ats_swiglu_supported", _lib.ATS_BF16, T, H, F) == 0
    assert _lib.query("ats_swiglu_supported", _lib.ATS_F32, 512, 256, 256) == 0
    wgu, wd = _weights(256, 200, 3)
    x = torch.randn(100, 256, device="cuda").bfloat16()
    y_ref = omoe.expert_fwd(np32(x), np32(wgu), np32(wd), "bf16")[0]
    close(dense_swiglu(x, wgu, wd), y_ref, "bf16")

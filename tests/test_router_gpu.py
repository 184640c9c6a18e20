"""The MoE router GEMMs on the tensor cores (bf16 tokens, float32 router weight).

The float32 operands run as three bf16 parts each; the results must be
float32 GEMMs up to summation order.  Every output is compared with a float64
reference of the same operands.  The bound for an element is 2e-6 of the
sum of the absolute products that make it up, which is about 30 float32 ulps
of that sum and covers any summation order over these depths.  A bf16-only
router would miss it by orders of magnitude.  The token gradient is checked
with the un-permute of the expert-row gradients fused in, against the
separate un-permute kernel plus the router share, both as bf16 values."""

from __future__ import annotations

import ctypes

import pytest
import torch

from ats_v2_b200 import _lib
from ats_v2_b200.moe import capacity_for, router_forward

pytestmark = pytest.mark.gpu


def _bound_close(got: torch.Tensor, ref64: torch.Tensor, absref64: torch.Tensor, what: str, rel: float = 2e-6):
    err = (got.double() - ref64).abs()
    lim = rel * absref64 + 1e-30
    bad = err > lim
    assert not bool(bad.any()), (f"{what}: {int(bad.sum())} elements over the bound; worst ratio "
                                 f"{float((err / lim).max()):.3g}")


def _inputs(T, H, E, seed, bias=False):
    g = torch.Generator(device="cuda").manual_seed(seed)
    x = torch.randn(T, H, device="cuda", generator=g).bfloat16()
    w = 0.02 * torch.randn(E, H, device="cuda", generator=g)
    b = torch.randn(E, device="cuda", generator=g) if bias else None
    return x, w, b


@pytest.mark.parametrize("T,H,E,bias", [(128, 128, 8, False), (1000, 256, 64, True), (8192, 2048, 8, False),
                                        (777, 384, 5, True), (4096, 4096, 64, False)])
def test_router_logits_are_float32_gemm(T, H, E, bias):
    assert _lib.query("ats_moe_router_supported", _lib.ATS_BF16, T, H, E) == 1
    x, w, b = _inputs(T, H, E, T + E, bias)
    logits, rws, _ = router_forward(x, w, b)
    assert rws is not None  # the tensor-core path ran
    x64, w64 = x.double(), w.double()
    ref = x64 @ w64.T
    absref = x64.abs() @ w64.abs().T
    if b is not None:
        ref = ref + b.double()
        absref = absref + b.double().abs()
    _bound_close(logits, ref, absref, "logits")
    # and as close to torch's float32 GEMM as float32 GEMMs are to each other
    t32 = torch.nn.functional.linear(x.float(), w) + (b if b is not None else 0)
    _bound_close(t32, ref, absref, "torch float32 logits (sanity)")


def _plan(x, logits, k, cf, layout=_lib.ATS_MOE_PACKED):
    T, H = x.shape
    E = logits.shape[1]
    C = capacity_for(T, k, E, cf)
    wsb = _lib.query("ats_moe_workspace_bytes", T, E, k, C, layout)
    R = _lib.query("ats_moe_max_rows", T, E, k, C, layout)
    ws = torch.empty(wsb, dtype=torch.uint8, device="cuda")
    gates = torch.empty(T, k, device="cuda")
    idx = torch.empty(T, k, dtype=torch.int64, device="cuda")
    aux = torch.empty((), device="cuda")
    st = _lib.stream_of(x)
    _lib.call("ats_moe_route_plan", logits.data_ptr(), T, E, k, C, layout, 0.01, gates.data_ptr(), idx.data_ptr(),
              aux.data_ptr(), None, None, ws.data_ptr(), wsb, st)
    return ws, wsb, C, R


@pytest.mark.parametrize("T,H,E,k,cf", [(1000, 256, 8, 2, 1.25), (4096, 2048, 64, 2, 1.25), (300, 128, 5, 3, 0.7)])
def test_router_backward_token_and_weight_gradients(T, H, E, k, cf):
    x, w, _ = _inputs(T, H, E, 3 * T + E)
    logits, rws, w32 = router_forward(x, w, None)
    g = torch.Generator(device="cuda").manual_seed(T)
    dl = torch.randn(T, E, device="cuda", generator=g) * 1e-2
    ws, wsb, C, R = _plan(x, logits, k, cf)
    dxp = torch.randn(R, H, device="cuda", generator=g).bfloat16()
    st = _lib.stream_of(x)
    dx = torch.empty(T, H, dtype=torch.bfloat16, device="cuda")
    dw = torch.empty(E, H, device="cuda")
    _lib.call("ats_moe_router_bwd", dl.data_ptr(), x.data_ptr(), w32.data_ptr(), dxp.data_ptr(), ws.data_ptr(),
              wsb, k, C, _lib.ATS_MOE_PACKED, dx.data_ptr(), dw.data_ptr(), T, H, E, rws.data_ptr(), rws.numel(),
              st)
    # weight gradient: dl^T x in float32
    x64, dl64, w64 = x.double(), dl.double(), w.double()
    _bound_close(dw, dl64.T @ x64, dl64.abs().T @ x64.abs(), "dw")
    # token gradient: bf16(sum of the token's expert rows) + bf16(dl . w), rounded once more
    share = dl64 @ w64
    moe = torch.empty(T, H, dtype=torch.bfloat16, device="cuda")
    _lib.call("ats_moe_scatter_grad", dxp.data_ptr(), moe.data_ptr(), _lib.ATS_BF16, T, H, E, k, C,
              _lib.ATS_MOE_PACKED, ws.data_ptr(), wsb, st)
    share16 = share.float().bfloat16()
    ref = (moe.double() + share16.double()).float().bfloat16()
    diff = (dx.float() - ref.float()).abs()
    # the router share is rounded from a float32 sum of another order: one bf16 ulp of the
    # share and one of the result is the slack
    tol = (ref.float().abs() + share16.float().abs()) * 2.0 ** -7 + 1e-12
    assert bool((diff <= tol).all()), f"dx: {int((diff > tol).sum())} elements beyond one bf16 ulp"
    exact = float((dx == ref).float().mean())
    assert exact > 0.98, f"dx: only {exact:.4f} of the elements equal the reference rounding"
    s = ctypes.c_int(-1)
    _lib.call("ats_moe_router_status", rws.data_ptr(), rws.numel(), T, H, E, ctypes.byref(s))
    assert s.value == 0


def test_staged_router_backward_equals_the_one_call():
    """ats_moe_router_bwd_staged: the weight-gradient stage, then (on the same
    workspace) the token-gradient stage, give exactly the one-call results --
    the form the expert-parallel backward uses to overlap the first stage with
    the output-gradient exchange."""
    T, H, E, k, cf = 2048, 1024, 64, 2, 1.25
    x, w, _ = _inputs(T, H, E, 77)
    logits, rws, w32 = router_forward(x, w, None)
    g = torch.Generator(device="cuda").manual_seed(5)
    dl = torch.randn(T, E, device="cuda", generator=g) * 1e-2
    ws, wsb, C, R = _plan(x, logits, k, cf)
    dxp = torch.randn(R, H, device="cuda", generator=g).bfloat16()
    st = _lib.stream_of(x)
    out = []
    for stages in ((_lib.ATS_ROUTER_BWD_ALL,), (_lib.ATS_ROUTER_BWD_DW, _lib.ATS_ROUTER_BWD_DX)):
        dx = torch.empty(T, H, dtype=torch.bfloat16, device="cuda")
        dw = torch.empty(E, H, device="cuda")
        for sg in stages:
            _lib.call("ats_moe_router_bwd_staged", dl.data_ptr(), x.data_ptr(), w32.data_ptr(), dxp.data_ptr(),
                      ws.data_ptr(), wsb, k, C, _lib.ATS_MOE_PACKED, dx.data_ptr(), dw.data_ptr(), T, H, E,
                      rws.data_ptr(), rws.numel(), sg, st)
        out.append((dx, dw))
    assert torch.equal(out[0][0], out[1][0]) and torch.equal(out[0][1], out[1][1])


def test_router_without_expert_rows_gives_the_router_share_only():
    T, H, E = 512, 256, 16
    x, w, _ = _inputs(T, H, E, 11)
    _, rws, w32 = router_forward(x, w, None)
    dl = torch.randn(T, E, device="cuda") * 1e-2
    dx = torch.empty(T, H, dtype=torch.bfloat16, device="cuda")
    dw = torch.empty(E, H, device="cuda")
    _lib.call("ats_moe_router_bwd", dl.data_ptr(), x.data_ptr(), w32.data_ptr(), None, None, 0, 2, 1, 0,
              dx.data_ptr(), dw.data_ptr(), T, H, E, rws.data_ptr(), rws.numel(), _lib.stream_of(x))
    share = (dl.double() @ w.double())
    ref = share.float().bfloat16()
    exact = float((dx == ref).float().mean())
    assert exact > 0.98
    assert float((dx.float() - ref.float()).abs().max()) <= float(ref.float().abs().max()) * 2 ** -7


def test_unsupported_router_shapes_use_the_library_gemm():
    for T, H, E in [(64, 256, 8), (1024, 200, 8), (1024, 256, 65)]:
        assert _lib.query("ats_moe_router_supported", _lib.ATS_BF16, T, H, E) == 0
        x, w, _ = _inputs(T, H, E, 5)
        logits, rws, _ = router_forward(x, w, None)
        assert rws is None
        torch.testing.assert_close(logits, torch.nn.functional.linear(x.float(), w), rtol=0, atol=0)
    assert _lib.query("ats_moe_router_supported", _lib.ATS_F32, 1024, 256, 8) == 0

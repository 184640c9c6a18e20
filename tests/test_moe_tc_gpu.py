"""The tcgen05 grouped GEMMs of the bf16 experts, one GEMM at a time.

The MoE stages are driven through the C ABI; after each stage the outputs of
every expert segment are compared with a float32 torch matmul of the same
permuted bf16 operands (K-major and MN-major operand layouts, M-grouped and
K-grouped GEMMs, the three epilogues).  Each GEMM is checked on its own
inputs, so an error points at one kernel.  Tolerance: 2e-2 relative with an
absolute floor of 2e-2 of the tensor's largest magnitude (bf16 outputs of
float32 accumulations summed in a different order)."""

from __future__ import annotations

import ctypes

import pytest
import torch
import torch.nn.functional as Fn

from ats_v2_b200 import _lib
from ats_v2_b200.moe import capacity_for

pytestmark = pytest.mark.gpu


def _close(got: torch.Tensor, ref: torch.Tensor, what: str) -> None:
    got, ref = got.float(), ref.float()
    scale = float(ref.abs().max()) if ref.numel() else 0.0
    torch.testing.assert_close(got, ref, rtol=2e-2, atol=max(2e-2 * scale, 1e-6), msg=lambda m: f"{what}: {m}")


def _silu_mul(g, u):
    s = Fn.silu(g.float()).bfloat16().float()
    return (s * u.float()).bfloat16()


def _swiglu_grad(g, u, da):
    g, u, da = g.float(), u.float(), da.float()
    s = Fn.silu(g).bfloat16().float()
    sig = torch.sigmoid(g)
    du = (da * s).bfloat16()
    ds = (da * u).bfloat16().float()
    dg = (ds * sig * (1 + g * (1 - sig))).bfloat16()
    return dg, du


def _run(T, H, F, E, k, cf, seed, starve=None, layout=_lib.ATS_MOE_PACKED):
    assert _lib.query("ats_moe_uses_tensor_cores", _lib.ATS_BF16, H, F) == 1
    g = torch.Generator(device="cuda").manual_seed(seed)
    x = torch.randn(T, H, device="cuda", generator=g).bfloat16()
    logits = torch.randn(T, E, device="cuda", generator=g)
    if starve is not None:
        logits[:, starve] = -1e4  # an expert nobody picks: empty segment
    wgu = (0.05 * torch.randn(E, 2 * F, H, device="cuda", generator=g)).bfloat16()
    wd = (0.05 * torch.randn(E, H, F, device="cuda", generator=g)).bfloat16()
    C = capacity_for(T, k, E, cf)
    L = layout
    wsb = _lib.query("ats_moe_workspace_bytes", T, E, k, C, L)
    R = _lib.query("ats_moe_max_rows", T, E, k, C, L)
    ws = torch.empty(wsb, dtype=torch.uint8, device="cuda")
    st = _lib.stream_of(x)
    gates = torch.empty(T, k, device="cuda")
    idx = torch.empty(T, k, dtype=torch.int64, device="cuda")
    aux = torch.empty((), device="cuda")
    _lib.call("ats_moe_route_plan", logits.data_ptr(), T, E, k, C, L, 0.01, gates.data_ptr(), idx.data_ptr(),
              aux.data_ptr(), None, None, ws.data_ptr(), wsb, st)
    seg = torch.empty(E + 1, dtype=torch.int32, device="cuda")
    kept = torch.empty(E, dtype=torch.int32, device="cuda")
    _lib.call("ats_moe_plan_export", ws.data_ptr(), wsb, T, E, k, C, L, seg.data_ptr(), None, kept.data_ptr(), st)
    xp = torch.empty(R, H, dtype=torch.bfloat16, device="cuda")
    _lib.call("ats_moe_gather", x.data_ptr(), xp.data_ptr(), _lib.ATS_BF16, T, H, E, k, C, L, ws.data_ptr(), wsb, st)
    h = torch.empty(R, 2 * F, dtype=torch.bfloat16, device="cuda")
    a = torch.empty(R, F, dtype=torch.bfloat16, device="cuda")
    y = torch.empty(R, H, dtype=torch.bfloat16, device="cuda")
    _lib.call("ats_moe_experts_fwd", xp.data_ptr(), wgu.data_ptr(), wd.data_ptr(), h.data_ptr(), a.data_ptr(),
              y.data_ptr(), _lib.ATS_BF16, T, E, k, C, L, H, F, ws.data_ptr(), wsb, st)
    dout = torch.randn(T, H, device="cuda", generator=g).bfloat16()
    dy = torch.empty(R, H, dtype=torch.bfloat16, device="cuda")
    dgr = torch.empty(R, device="cuda")
    _lib.call("ats_moe_combine_bwd", dout.data_ptr(), y.data_ptr(), dy.data_ptr(), dgr.data_ptr(), _lib.ATS_BF16,
              T, H, E, k, C, L, ws.data_ptr(), wsb, st)
    dh = torch.empty(R, 2 * F, dtype=torch.bfloat16, device="cuda")
    dxp = torch.empty(R, H, dtype=torch.bfloat16, device="cuda")
    dwgu = torch.empty(E, 2 * F, H, dtype=torch.bfloat16, device="cuda")
    dwd = torch.empty(E, H, F, dtype=torch.bfloat16, device="cuda")
    _lib.call("ats_moe_experts_bwd", dy.data_ptr(), xp.data_ptr(), h.data_ptr(), a.data_ptr(), wgu.data_ptr(),
              wd.data_ptr(), dh.data_ptr(), dxp.data_ptr(), dwgu.data_ptr(), dwd.data_ptr(), _lib.ATS_BF16, T, E,
              k, C, L, H, F, ws.data_ptr(), wsb, st)
    status = ctypes.c_int(-1)
    _lib.call("ats_moe_status", ws.data_ptr(), wsb, T, E, k, C, L, ctypes.byref(status))
    assert status.value == 0
    seg, kept = seg.tolist(), kept.tolist()
    for e in range(E):
        # the rows the GEMMs compute: kept rows rounded up to 128 (zero padding)
        r0, r1 = seg[e], seg[e] + (kept[e] + 127) // 128 * 128
        if layout == _lib.ATS_MOE_PACKED:
            assert r1 == seg[e + 1]
        else:
            assert seg[e] == e * ((C + 127) // 128 * 128)
        if starve == e:
            assert r1 == r0
        xs, hs, as_, dys, dhs = xp[r0:r1], h[r0:r1], a[r0:r1], dy[r0:r1], dh[r0:r1]
        # forward GEMM 1 (K-major A and B, gate/up halves) + SwiGLU epilogue
        _close(hs, (xs.float() @ wgu[e].float().T).bfloat16(), f"h[e={e}]")
        _close(as_, _silu_mul(hs[:, :F], hs[:, F:]), f"a[e={e}]")
        # forward GEMM 2
        _close(y[r0:r1], (as_.float() @ wd[e].float().T).bfloat16(), f"y[e={e}]")
        # dgrad GEMM 1 (N-major B) + SwiGLU backward epilogue
        da = (dys.float() @ wd[e].float()).bfloat16()
        rdg, rdu = _swiglu_grad(hs[:, :F], hs[:, F:], da)
        _close(dhs[:, :F], rdg, f"dg[e={e}]")
        _close(dhs[:, F:], rdu, f"du[e={e}]")
        # dgrad GEMM 2 (N-major B)
        _close(dxp[r0:r1], (dhs.float() @ wgu[e].float()).bfloat16(), f"dxp[e={e}]")
        # weight-gradient GEMMs (M-major A, N-major B, K = segment rows)
        _close(dwd[e], (dys.float().T @ as_.float()).bfloat16(), f"dWd[e={e}]")
        _close(dwgu[e], (dhs.float().T @ xs.float()).bfloat16(), f"dWgu[e={e}]")


@pytest.mark.parametrize("T,H,F,E,k,cf", [
    (512, 256, 384, 4, 2, 1.25),    # N tiles of 128 on the ffn dim (384 = 3 x 128)
    (1024, 512, 1024, 8, 2, 4.0),   # N tiles of 256 everywhere
    (300, 128, 128, 3, 1, 1.0),     # smallest tiles, ragged segments
])
def test_each_grouped_gemm_matches_torch(T, H, F, E, k, cf):
    _run(T, H, F, E, k, cf, seed=T + H + F)


def test_empty_expert_segment_gives_zero_weight_gradient():
    _run(512, 256, 256, 4, 2, 4.0, seed=7, starve=2)


@pytest.mark.parametrize("T,H,F,E,k,cf", [(1000, 256, 256, 8, 2, 1.25), (600, 128, 384, 4, 3, 0.7)])
def test_each_grouped_gemm_on_capacity_slots(T, H, F, E, k, cf):
    _run(T, H, F, E, k, cf, seed=T + F, layout=_lib.ATS_MOE_SLOTS)

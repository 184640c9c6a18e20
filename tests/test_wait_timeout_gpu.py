"""The ATS_ETIMEOUT path of the bounded device waits.

Every mbarrier wait in the tensor-core GEMM and the RMSNorm ring kernels
gives up after a budget of SM cycles: the role that gave up records a code,
raises the CTA's abort flag, the other roles stop, the copies and MMAs
already issued are drained (those waits keep the full budget) and TMEM is
freed.  These tests shorten the main-loop budget to one cycle
(``ats_set_wait_budget``), so the first wait that does not complete at once
gives up, and check that the call reports ATS_ETIMEOUT through its own status
word and through ``ats_device_status``, that reading clears the status, and
that a call made after the budget is restored is correct again.  No wait is
made to hang: each one ends by its budget, and the GPU stays usable.
"""

from __future__ import annotations

import ctypes

import pytest
import torch

from ats_v2_b200 import _lib
from tests.util import close, np32

pytestmark = pytest.mark.gpu


@pytest.fixture
def short_waits():
    torch.cuda.synchronize()
    _lib.check_device_status("before the timeout test")
    _lib.call("ats_set_wait_budget", 1)
    try:
        yield
    finally:
        torch.cuda.synchronize()
        _lib.call("ats_set_wait_budget", 0)


def _status(name, *args):
    code = ctypes.c_int(0)
    st = _lib.query(name, *args, ctypes.byref(code))
    return st, code.value


def _swiglu(x, wgu, wd, ws):
    T, H = x.shape
    F = wd.shape[1]
    R = _lib.query("ats_swiglu_rows", T)
    h = torch.empty(R, 2 * F, dtype=x.dtype, device="cuda")
    a = torch.empty(R, F, dtype=x.dtype, device="cuda")
    y = torch.empty(T, H, dtype=x.dtype, device="cuda")
    _lib.call("ats_swiglu_fwd", x.data_ptr(), wgu.data_ptr(), wd.data_ptr(), h.data_ptr(), a.data_ptr(),
              y.data_ptr(), _lib.ATS_BF16, T, H, F, ws.data_ptr(), ws.numel(), _lib.stream_of(x))
    return y


def _swiglu_ref(x, wgu, wd):
    hh = (x.float() @ wgu.float().t()).bfloat16()
    g, u = hh.chunk(2, dim=-1)
    a = (torch.nn.functional.silu(g.float()).bfloat16().float() * u.float()).bfloat16()
    return (a.float() @ wd.float().t()).bfloat16()


def test_gemm_wait_that_runs_out_reports_timeout_and_the_next_call_is_correct(short_waits):
    T, H, F = 512, 256, 384
    g = torch.Generator(device="cuda").manual_seed(0)
    x = torch.randn(T, H, device="cuda", generator=g).bfloat16()
    wgu = (0.05 * torch.randn(2 * F, H, device="cuda", generator=g)).bfloat16()
    wd = (0.05 * torch.randn(H, F, device="cuda", generator=g)).bfloat16()
    ws = torch.empty(_lib.query("ats_swiglu_workspace_bytes"), dtype=torch.uint8, device="cuda")
    _swiglu(x, wgu, wd, ws)
    torch.cuda.synchronize()
    st, code = _status("ats_swiglu_status", ws.data_ptr(), ws.numel())
    assert st == _lib.ATS_ETIMEOUT and code != 0
    st, code2 = _status("ats_device_status")
    assert st == _lib.ATS_ETIMEOUT and code2 != 0
    assert _status("ats_device_status") == (_lib.ATS_OK, 0)  # reading cleared it
    # the budget back at its default: the same call completes and is right
    _lib.call("ats_set_wait_budget", 0)
    y = _swiglu(x, wgu, wd, ws)
    torch.cuda.synchronize()
    assert _status("ats_swiglu_status", ws.data_ptr(), ws.numel()) == (_lib.ATS_OK, 0)
    assert _status("ats_device_status") == (_lib.ATS_OK, 0)
    close(y, np32(_swiglu_ref(x, wgu, wd)), "bf16")


def test_rmsnorm_ring_wait_that_runs_out_reports_timeout_and_the_next_call_is_correct(short_waits):
    rows, H = 4096, 2048  # bf16 rows of 4 KB take the ring kernels
    g = torch.Generator(device="cuda").manual_seed(1)
    x = torch.randn(rows, H, device="cuda", generator=g).bfloat16()
    dy = torch.randn(rows, H, device="cuda", generator=g).bfloat16()
    w = 1 + 0.02 * torch.randn(H, device="cuda", generator=g)
    n = _lib.query("ats_rmsnorm_bwd_workspace_bytes", rows, H)
    ws = torch.empty(n, dtype=torch.uint8, device="cuda")

    def bwd():
        dx = torch.empty_like(x)
        dw = torch.empty(H, device="cuda")
        _lib.call("ats_rmsnorm_bwd", dy.data_ptr(), x.data_ptr(), _lib.ATS_BF16, w.data_ptr(), _lib.ATS_F32,
                  dx.data_ptr(), dw.data_ptr(), ws.data_ptr(), n, rows, H, 1e-5, _lib.stream_of(x))
        return dx, dw

    bwd()
    torch.cuda.synchronize()
    st, code = _status("ats_rmsnorm_status")
    assert st == _lib.ATS_ETIMEOUT and code != 0
    assert _status("ats_rmsnorm_status") == (_lib.ATS_OK, 0)  # reading cleared it
    # the library-wide word saw it too
    bwd()
    torch.cuda.synchronize()
    with pytest.raises(_lib.AtsError) as ei:
        _lib.check_device_status("rmsnorm backward")
    assert ei.value.status == _lib.ATS_ETIMEOUT
    _lib.call("ats_set_wait_budget", 0)
    dx, dw = bwd()
    torch.cuda.synchronize()
    assert _status("ats_rmsnorm_status") == (_lib.ATS_OK, 0)
    xf, dyf = x.double(), dy.double()
    r = torch.rsqrt(xf.square().mean(-1, keepdim=True) + 1e-5)
    gw = dyf * w.double()
    ref_dx = r * gw - xf * r.pow(3) * (gw * xf).mean(-1, keepdim=True)
    ref_dw = (dyf * xf * r).sum(0)
    close(dx, np32(ref_dx), "bf16")
    close(dw, np32(ref_dw), "f32", rtol=1e-4, atol=1e-3)

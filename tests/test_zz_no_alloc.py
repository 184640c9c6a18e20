"""The allocation-free RMSNorm backward, ``ats_rmsnorm_bwd_noalloc``.

Some callers cannot allocate device memory around a call: a host runtime
that drives this library through a bare C FFI and has no caching allocator
(a cudaMalloc per call would stall the device), or a process held to a fixed,
pre-reserved memory budget.  For them the entry point keeps its scratch (the
per-block weight-gradient partial sums) in a fixed device array of the
library.  These tests call it through the C ABI and check it against the
workspace entry point, ``ats_rmsnorm_bwd``, on two calls in a row -- the
second with different sizes and data, so contents left in the shared array by
the first call must not leak into the second.  This file is collected last.
"""

from __future__ import annotations

import pytest
import torch

from ats_v2_b200 import _lib
from tests.util import close, np32

pytestmark = pytest.mark.gpu


def _inputs(rows, hidden, seed, xdt, wdt):
    g = torch.Generator(device="cuda").manual_seed(seed)
    x = torch.randn(rows, hidden, device="cuda", generator=g).to(xdt)
    dy = torch.randn(rows, hidden, device="cuda", generator=g).to(xdt)
    w = (1 + 0.1 * torch.randn(hidden, device="cuda", generator=g)).to(wdt)
    return x, dy, w


def _with_workspace(x, dy, w, eps):
    rows, hidden = x.shape
    dx = torch.empty_like(x)
    dw = torch.empty(hidden, dtype=w.dtype, device="cuda")
    n = _lib.query("ats_rmsnorm_bwd_workspace_bytes", rows, hidden)
    ws = torch.empty(n, dtype=torch.uint8, device="cuda")
    _lib.call("ats_rmsnorm_bwd", dy.data_ptr(), x.data_ptr(), _lib.dtype_code(x.dtype), w.data_ptr(),
              _lib.dtype_code(w.dtype), dx.data_ptr(), dw.data_ptr(), ws.data_ptr(), n, rows, hidden, eps,
              _lib.stream_of(x))
    return dx, dw


def _without_workspace(x, dy, w, eps):
    rows, hidden = x.shape
    dx = torch.empty_like(x)
    dw = torch.empty(hidden, dtype=w.dtype, device="cuda")
    _lib.call("ats_rmsnorm_bwd_noalloc", dy.data_ptr(), x.data_ptr(), _lib.dtype_code(x.dtype), w.data_ptr(),
              _lib.dtype_code(w.dtype), dx.data_ptr(), dw.data_ptr(), rows, hidden, eps, _lib.stream_of(x))
    return dx, dw


@pytest.mark.parametrize("xdt,wdt", [(torch.bfloat16, torch.float32), (torch.float32, torch.float32)])
def test_noalloc_matches_workspace_entry_point_on_two_calls(xdt, wdt):
    dn = "bf16" if xdt == torch.bfloat16 else "f32"
    # first call: a large case that fills many partial rows of the shared array;
    # second call: smaller rows and hidden with other data
    for rows, hidden, seed in ((8192, 4096, 0), (300, 1024, 1)):
        x, dy, w = _inputs(rows, hidden, seed, xdt, wdt)
        ref_dx, ref_dw = _with_workspace(x, dy, w, 1e-5)
        dx, dw = _without_workspace(x, dy, w, 1e-5)
        torch.cuda.synchronize()
        close(dx, np32(ref_dx), dn)
        close(dw, np32(ref_dw), "f32", rtol=1e-5, atol=1e-5)
        assert torch.equal(dx, ref_dx) and torch.equal(dw, ref_dw)  # same kernels, same order


def test_noalloc_rejects_hidden_above_its_limit():
    x, dy, w = _inputs(4, 8200, 2, torch.bfloat16, torch.float32)
    dx = torch.empty_like(x)
    dw = torch.empty(8200, device="cuda")
    with pytest.raises(_lib.AtsError) as ei:
        _lib.call("ats_rmsnorm_bwd_noalloc", dy.data_ptr(), x.data_ptr(), _lib.ATS_BF16, w.data_ptr(),
                  _lib.ATS_F32, dx.data_ptr(), dw.data_ptr(), 4, 8200, 1e-5, _lib.stream_of(x))
    assert ei.value.status == _lib.ATS_EUNSUPPORTED
    assert "8192" in str(ei.value)

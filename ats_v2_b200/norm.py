"""RMSNorm on the sm_100a kernels -- mirror of ats/model/norm.py.

``RMSNorm(hidden_size, eps=1e-6)`` keeps the reference module's constructor,
``weight`` parameter (ones, [hidden]) and ValueError messages
(norm.py:11-29).  Its forward computes what F.rms_norm computes
(norm.py:30-31): float32 arithmetic, one rounding to x's dtype.  Forward and
backward are single-pass CUDA kernels (``ats_rmsnorm_fwd`` / ``ats_rmsnorm_bwd``)
for CUDA tensors.  CPU tensors take the reference's own computation,
``F.rms_norm`` (norm.py:30-31), so the reference's CPU tests and CPU-built
models run unchanged; a CUDA tensor never does.
"""

from __future__ import annotations

import torch
import torch.nn.functional as F
from torch import nn

from ats_v2_b200 import _lib


def _rows(x: torch.Tensor, hidden: int) -> torch.Tensor:
    x2 = x.reshape(-1, hidden)
    if x2.stride(-1) != 1:
        x2 = x2.contiguous()
    return x2


class _RMSNormFn(torch.autograd.Function):
    @staticmethod
    def forward(ctx, x: torch.Tensor, weight: torch.Tensor, eps: float):
        H = x.shape[-1]
        x2 = _rows(x, H)
        w = weight.contiguous()
        y = torch.empty((x2.shape[0], H), dtype=x.dtype, device=x.device)
        _lib.call("ats_rmsnorm_fwd", x2.data_ptr(), x2.stride(0), _lib.dtype_code(x.dtype), w.data_ptr(),
                  _lib.dtype_code(w.dtype), y.data_ptr(), H, None, x2.shape[0], H, float(eps),
                  _lib.stream_of(x))
        ctx.save_for_backward(x2, w)
        ctx.eps = eps
        ctx.x_shape = x.shape
        return y.view(x.shape)

    @staticmethod
    def backward(ctx, dy: torch.Tensor):
        x2, w = ctx.saved_tensors
        rows, H = x2.shape
        x2 = x2.contiguous()
        dy2 = dy.reshape(rows, H).contiguous()
        if dy2.dtype != x2.dtype:
            dy2 = dy2.to(x2.dtype)
        dx = torch.empty_like(x2)
        dw = torch.empty(H, dtype=w.dtype, device=w.device)
        ws_bytes = _lib.query("ats_rmsnorm_bwd_workspace_bytes", rows, H)
        ws = torch.empty(ws_bytes, dtype=torch.uint8, device=x2.device)
        _lib.call("ats_rmsnorm_bwd", dy2.data_ptr(), x2.data_ptr(), _lib.dtype_code(x2.dtype), w.data_ptr(),
                  _lib.dtype_code(w.dtype), dx.data_ptr(), dw.data_ptr(), ws.data_ptr(), ws_bytes, rows, H,
                  float(ctx.eps), _lib.stream_of(x2))
        return dx.view(ctx.x_shape), dw, None


def rms_norm(x: torch.Tensor, weight: torch.Tensor, eps: float) -> torch.Tensor:
    """Functional RMSNorm over the last dim: the CUDA kernels for CUDA tensors,
    the reference's F.rms_norm for CPU tensors."""
    if weight.shape != (x.shape[-1],):
        raise ValueError(f"rms_norm: weight shape {tuple(weight.shape)} must be ({x.shape[-1]},).")
    if _lib.on_cpu("rms_norm", x, weight):
        return F.rms_norm(x, (x.shape[-1],), weight, eps)
    return _RMSNormFn.apply(x, weight, eps)


class RMSNorm(nn.Module):
    """Drop-in for ats.model.norm.RMSNorm (norm.py:11-37) on the CUDA kernels."""

    def __init__(self, hidden_size: int, eps: float = 1e-6) -> None:
        super().__init__()
        if hidden_size <= 0:
            raise ValueError(f"RMSNorm hidden_size must be positive, got {hidden_size}.")
        self.hidden_size = hidden_size
        self.eps = eps
        self.weight = nn.Parameter(torch.ones(hidden_size))

    def forward(self, x: torch.Tensor) -> torch.Tensor:
        if x.shape[-1] != self.hidden_size:
            raise ValueError(
                f"RMSNorm expected last dimension {self.hidden_size}, got {x.shape[-1]} "
                f"(full shape {tuple(x.shape)}). Fix: check that the layer feeding this "
                f"RMSNorm produces hidden_size={self.hidden_size}."
            )
        return rms_norm(x, self.weight, self.eps)

    def extra_repr(self) -> str:
        return f"{self.hidden_size}, eps={self.eps}"

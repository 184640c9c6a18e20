"""Fused RMSNorm + residual on the sm_100a kernels -- mirror of
ats/model/norm_triton.py.

``fused_rmsnorm_residual(x, residual, weight, eps=1e-6)`` validates like the
reference (norm_triton.py:111-120) and computes the reference's PyTorch
formula (norm_triton.py:88-98), ``residual + (x*rsqrt(mean(x^2)+eps)).to(x.dtype)
* weight``, with torch's type promotion at each step, in one CUDA pass.
Unlike the reference's Triton kernel it is differentiable (x, residual and
weight).  ``_cuda_rmsnorm_residual`` is the kernel call without validation.

The reference's tests import three more names from this module
(tests/test_triton.py:19-25,142-149), kept here with the same meaning:
``HAS_TRITON`` says whether the fused GPU kernel is available (here: whether
the CUDA library is built; no Triton is involved), ``_triton_rmsnorm_residual``
is the fused kernel call, and ``_pytorch_rmsnorm_residual`` is the plain torch
formula those tests compare the kernel against.  ``fused_rmsnorm_residual``
runs that formula for CPU tensors, as the reference does
(norm_triton.py:121-123); CUDA tensors always take the kernel.
"""

from __future__ import annotations

import torch

from ats_v2_b200 import _lib

HAS_TRITON = _lib.LIB_PATH.exists()  # the reference's flag name: fused GPU kernel available


def _out_dtype(x: torch.Tensor, w: torch.Tensor) -> torch.dtype:
    return torch.promote_types(x.dtype, w.dtype)


class _RMSNormResidualFn(torch.autograd.Function):
    @staticmethod
    def forward(ctx, x, residual, weight, eps):
        H = x.shape[-1]
        x2 = x.reshape(-1, H).contiguous()
        r2 = residual.reshape(-1, H).contiguous()
        w = weight.contiguous()
        out = torch.empty(x2.shape, dtype=_out_dtype(x, weight), device=x.device)
        _lib.call("ats_rmsnorm_residual_fwd", x2.data_ptr(), r2.data_ptr(), _lib.dtype_code(x.dtype),
                  w.data_ptr(), _lib.dtype_code(w.dtype), out.data_ptr(), x2.shape[0], H, float(eps),
                  _lib.stream_of(x))
        ctx.save_for_backward(x2, w)
        ctx.eps = eps
        ctx.shape = x.shape
        return out.view(x.shape)

    @staticmethod
    def backward(ctx, dout):
        x2, w = ctx.saved_tensors
        rows, H = x2.shape
        d2 = dout.reshape(rows, H).to(_out_dtype(x2, w)).contiguous()
        dx = torch.empty_like(x2)
        dres = torch.empty_like(x2)
        dw = torch.empty(H, dtype=w.dtype, device=w.device)
        ws_bytes = _lib.query("ats_rmsnorm_bwd_workspace_bytes", rows, H)
        ws = torch.empty(ws_bytes, dtype=torch.uint8, device=x2.device)
        _lib.call("ats_rmsnorm_residual_bwd", d2.data_ptr(), x2.data_ptr(), _lib.dtype_code(x2.dtype),
                  w.data_ptr(), _lib.dtype_code(w.dtype), dx.data_ptr(), dres.data_ptr(), dw.data_ptr(),
                  ws.data_ptr(), ws_bytes, rows, H, float(ctx.eps), _lib.stream_of(x2))
        return dx.view(ctx.shape), dres.view(ctx.shape), dw, None


def _cuda_rmsnorm_residual(x: torch.Tensor, residual: torch.Tensor, weight: torch.Tensor,
                           eps: float) -> torch.Tensor:
    _lib.require_cuda("fused_rmsnorm_residual", x, residual, weight)
    if residual.dtype != x.dtype:
        raise TypeError(f"fused_rmsnorm_residual: residual dtype {residual.dtype} must equal x dtype {x.dtype}")
    return _RMSNormResidualFn.apply(x, residual, weight, eps)


# fused-kernel name of the reference module (tests/test_triton.py:142-149)
_triton_rmsnorm_residual = _cuda_rmsnorm_residual


def _pytorch_rmsnorm_residual(x: torch.Tensor, residual: torch.Tensor, weight: torch.Tensor,
                              eps: float) -> torch.Tensor:
    """The torch formula of norm_triton.py:88-98, the comparison of the reference's kernel test."""
    xf = x.to(torch.float32)
    inv = torch.rsqrt(xf.pow(2).mean(dim=-1, keepdim=True) + eps)
    return residual + (xf * inv).to(x.dtype) * weight


def fused_rmsnorm_residual(x: torch.Tensor, residual: torch.Tensor, weight: torch.Tensor,
                           eps: float = 1e-6) -> torch.Tensor:
    """``residual + rms_norm(x) * weight``: one memory pass on CUDA; the torch formula on CPU."""
    if x.shape != residual.shape:
        raise ValueError(
            f"fused_rmsnorm_residual: x shape {tuple(x.shape)} must match "
            f"residual shape {tuple(residual.shape)}."
        )
    if weight.shape[-1] != x.shape[-1]:
        raise ValueError(
            f"fused_rmsnorm_residual: weight last dim {weight.shape[-1]} must match "
            f"x last dim {x.shape[-1]}."
        )
    if _lib.on_cpu("fused_rmsnorm_residual", x, residual, weight):
        return _pytorch_rmsnorm_residual(x, residual, weight, eps)
    return _cuda_rmsnorm_residual(x, residual, weight, eps)


class _AddRMSNormFn(torch.autograd.Function):
    @staticmethod
    def forward(ctx, x, residual, weight, eps):
        H = x.shape[-1]
        a = x.reshape(-1, H).contiguous()
        b = residual.reshape(-1, H).contiguous()
        w = weight.contiguous()
        s = torch.empty_like(a)
        y = torch.empty_like(a)
        _lib.call("ats_add_rmsnorm_fwd", a.data_ptr(), b.data_ptr(), _lib.dtype_code(a.dtype), w.data_ptr(),
                  _lib.dtype_code(w.dtype), s.data_ptr(), y.data_ptr(), a.shape[0], H, float(eps),
                  _lib.stream_of(a))
        ctx.save_for_backward(s, w)
        ctx.eps = eps
        ctx.shape = x.shape
        return y.view(x.shape), s.view(x.shape)

    @staticmethod
    def backward(ctx, dy, ds_in):
        s, w = ctx.saved_tensors
        rows, H = s.shape
        dy2 = (dy if dy is not None else torch.zeros_like(s)).reshape(rows, H).to(s.dtype).contiguous()
        di = ds_in.reshape(rows, H).to(s.dtype).contiguous() if ds_in is not None else None
        ds = torch.empty_like(s)
        dw = torch.empty(H, dtype=w.dtype, device=w.device)
        wsb = _lib.query("ats_add_rmsnorm_bwd_workspace_bytes", rows, H)
        ws = torch.empty(wsb, dtype=torch.uint8, device=s.device)
        _lib.call("ats_add_rmsnorm_bwd", dy2.data_ptr(), s.data_ptr(), _lib.ptr(di), _lib.dtype_code(s.dtype),
                  w.data_ptr(), _lib.dtype_code(w.dtype), ds.data_ptr(), dw.data_ptr(), ws.data_ptr(), wsb, rows, H,
                  float(ctx.eps), _lib.stream_of(s))
        ds = ds.view(ctx.shape)
        return ds, ds, dw, None


def add_rmsnorm_supported(x: torch.Tensor, weight: torch.Tensor) -> bool:
    """Whether the fused kernel covers this shape (16-byte rows of at most 512 chunks)."""
    H = x.shape[-1]
    n = 16 // x.element_size()
    return x.dtype in (torch.float32, torch.bfloat16) and weight.dtype in (torch.float32, torch.bfloat16) \
        and H % n == 0 and H // n <= 512


def fused_add_rmsnorm(x: torch.Tensor, residual: torch.Tensor, weight: torch.Tensor,
                      eps: float = 1e-6) -> tuple[torch.Tensor, torch.Tensor]:
    """``s = residual + x; (rms_norm(s) * weight, s)`` -- the post-attention residual add
    and RMSNorm of TransformerBlock.forward (ats/model/transformer.py:208-212), whose
    ``s`` is the block's next residual.  CUDA tensors: one kernel each way (the
    backward adds the gradient that reaches ``s`` from the next residual add, as
    autograd would).  CPU tensors: the reference's two torch operations."""
    if x.shape != residual.shape:
        raise ValueError(f"fused_add_rmsnorm: x shape {tuple(x.shape)} must match residual shape "
                         f"{tuple(residual.shape)}.")
    if weight.shape != (x.shape[-1],):
        raise ValueError(f"fused_add_rmsnorm: weight shape {tuple(weight.shape)} must be ({x.shape[-1]},).")
    if _lib.on_cpu("fused_add_rmsnorm", x, residual, weight):
        s = residual + x
        return torch.nn.functional.rms_norm(s, (s.shape[-1],), weight, eps), s
    if residual.dtype != x.dtype:
        raise TypeError(f"fused_add_rmsnorm: residual dtype {residual.dtype} must equal x dtype {x.dtype}")
    if not add_rmsnorm_supported(x, weight):
        from ats_v2_b200.norm import rms_norm

        s = residual + x
        return rms_norm(s, weight, eps), s
    return _AddRMSNormFn.apply(x, residual, weight, eps)

"""Oracle for RMSNorm and the fused RMSNorm+residual entry point (test-only).

Reference:
  * ``ats/model/norm.py:23-31``  RMSNorm.forward -> F.rms_norm(x, (H,), w, eps).
    With a float32 weight and a bfloat16 input, torch 2.11 takes its composite
    path: every step is computed in float32 and the result is rounded once to
    the input dtype.  The oracle does exactly that.
  * ``ats/model/norm.py:33-37``  the manual fallback (same reduction and eps
    placement), used only when F.rms_norm is missing.
  * ``ats/model/norm_triton.py:88-98``  _pytorch_rmsnorm_residual:
    ``residual + (x32 * rsqrt(mean(x32^2) + eps)).to(x.dtype) * weight``.
  * backward: torch autograd of the expressions above (no custom backward
    exists in the reference); the gradients below are the analytic
    derivatives, evaluated in float32 and rounded to each tensor's dtype.
"""

from __future__ import annotations

import numpy as np

from oracle.bf16 import promote, round_to


def _rstd(x32: np.ndarray, eps: float) -> np.ndarray:
    """1/sqrt(mean(x^2) + eps) per row, float32 (norm.py:35-36)."""
    var = np.mean(np.square(x32, dtype=np.float32), axis=-1, keepdims=True, dtype=np.float32)
    return (np.float32(1.0) / np.sqrt(var + np.float32(eps))).astype(np.float32)


def rmsnorm_fwd(x, w, eps: float, x_dtype: str = "f32"):
    """y = round_{x_dtype}(x * rstd * w), all in float32 (norm.py:30-31).

    Returns (y, rstd[..., 1])."""
    x32 = np.asarray(x, dtype=np.float32)
    w32 = np.asarray(w, dtype=np.float32)
    r = _rstd(x32, eps)
    y = round_to((x32 * r) * w32, x_dtype)
    return y, r


def rmsnorm_bwd(dy, x, w, eps: float, x_dtype: str = "f32", w_dtype: str = "f32"):
    """Gradients of rmsnorm_fwd.

    dx_i = r*dy_i*w_i - x_i * r^3/H * sum_j(dy_j*w_j*x_j)  (rounded to x dtype)
    dw_j = sum_rows dy_j * x_j * r                          (rounded to w dtype)
    """
    x32 = np.asarray(x, dtype=np.float32)
    dy32 = np.asarray(dy, dtype=np.float32)
    w32 = np.asarray(w, dtype=np.float32)
    H = x32.shape[-1]
    r = _rstd(x32, eps)
    g = dy32 * w32
    c = np.sum(g * x32, axis=-1, keepdims=True, dtype=np.float32)
    dx = r * g - x32 * (r * r * r) * (c / np.float32(H))
    xhat = x32 * r
    dw = np.sum((dy32 * xhat).reshape(-1, H), axis=0, dtype=np.float64).astype(np.float32)
    return round_to(dx, x_dtype), round_to(dw, w_dtype)


def rmsnorm_residual_fwd(x, residual, w, eps: float,
                         x_dtype: str = "f32", r_dtype: str = "f32", w_dtype: str = "f32"):
    """residual + (x*rstd).to(x.dtype) * w  (norm_triton.py:88-98).

    Torch type promotion decides each intermediate's dtype:
      n1 = round_{x}(x*r); n2 = round_{promote(x,w)}(n1*w);
      out = round_{promote(x,w,res)}(res + n2)."""
    x32 = np.asarray(x, dtype=np.float32)
    r = _rstd(x32, eps)
    n1 = round_to(x32 * r, x_dtype)
    p1 = promote(x_dtype, w_dtype)
    n2 = round_to(n1 * np.asarray(w, dtype=np.float32), p1)
    p2 = promote(p1, r_dtype)
    out = round_to(np.asarray(residual, dtype=np.float32) + n2, p2)
    return out, r


def rmsnorm_residual_bwd(dout, x, w, eps: float,
                         x_dtype: str = "f32", r_dtype: str = "f32", w_dtype: str = "f32"):
    """Gradients of rmsnorm_residual_fwd: (dx, dresidual, dw).

    dresidual = dout cast to the residual dtype; dw = sum_rows dout*n1;
    the normalisation's gradient takes dn1 = dout*w (through the .to(x.dtype)
    cast, whose backward is a cast back to float32)."""
    x32 = np.asarray(x, dtype=np.float32)
    d32 = np.asarray(dout, dtype=np.float32)
    w32 = np.asarray(w, dtype=np.float32)
    H = x32.shape[-1]
    r = _rstd(x32, eps)
    n1 = round_to(x32 * r, x_dtype)
    p1 = promote(x_dtype, w_dtype)
    dn2 = round_to(d32, p1)
    # autograd casts the product's gradient to n1's dtype before the cast back
    dn1 = round_to(dn2 * w32, x_dtype)
    c = np.sum(dn1 * x32, axis=-1, keepdims=True, dtype=np.float32)
    dx = r * dn1 - x32 * (r * r * r) * (c / np.float32(H))
    dw = np.sum((dn2 * n1).reshape(-1, H), axis=0, dtype=np.float64).astype(np.float32)
    return round_to(dx, x_dtype), round_to(d32, r_dtype), round_to(dw, w_dtype)

"""Fused MLA KV decompression -- mirror of ats/model/mla_triton.py.

``fused_mla_kv_decompress(c, w_uk, w_uv)`` validates like
mla_triton.py:131-142 and computes (k, v) = (c w_uk^T, c w_uv^T) as one
matmul of the latent rows against the stacked weight [w_uk; w_uv]
(mla_triton.py:144-148), then splits the result.  bf16 shapes the tensor-core
tiling covers (at least 128 rows; latent and output sizes multiples of 128)
run on the library's tcgen05 GEMM (``ats_gemm_fwd/bwd``: float32
accumulation, one rounding to bf16, as the reference's kernel accumulates in
float32 and casts once); other shapes and dtypes use torch's GPU GEMM.  The
product is differentiable.

As in the reference module, ``HAS_TRITON`` says whether the fused GPU kernel
is available (here: whether the CUDA library is built; no Triton is
involved) and ``_triton_matmul(a, b)`` is the kernel call for a [M, K] and
b [K, N] (mla_triton.py:78-104), the name the reference's kernel test imports
(tests/test_triton.py:194-207).  As in the reference (mla_triton.py:144-148),
CPU tensors take two plain torch matmuls.
"""

from __future__ import annotations

import torch

from ats_v2_b200 import _lib

HAS_TRITON = _lib.LIB_PATH.exists()  # the reference's flag name: fused GPU kernel available


class _MatmulNT(torch.autograd.Function):
    """a [M, K] @ w[N, K]^T on the tensor-core GEMM (bf16, shapes ats_gemm_supported covers)."""

    @staticmethod
    def forward(ctx, a, w):
        M, K = a.shape
        N = w.shape[0]
        st = _lib.stream_of(a)
        wsb = _lib.query("ats_gemm_workspace_bytes")
        ws = torch.empty(wsb, dtype=torch.uint8, device=a.device)
        out = torch.empty((M, N), dtype=a.dtype, device=a.device)
        _lib.call("ats_gemm_fwd", a.data_ptr(), w.data_ptr(), out.data_ptr(), _lib.ATS_BF16, M, N, K, ws.data_ptr(),
                  wsb, st)
        ctx.save_for_backward(a, w)
        return out

    @staticmethod
    def backward(ctx, dout):
        a, w = ctx.saved_tensors
        M, K = a.shape
        N = w.shape[0]
        dout = dout.to(a.dtype).contiguous()
        da = torch.empty_like(a) if ctx.needs_input_grad[0] else None
        dw = torch.empty_like(w) if ctx.needs_input_grad[1] else None
        if da is None and dw is None:
            return None, None
        st = _lib.stream_of(a)
        wsb = _lib.query("ats_gemm_workspace_bytes")
        ws = torch.empty(wsb, dtype=torch.uint8, device=a.device)
        _lib.call("ats_gemm_bwd", dout.data_ptr(), a.data_ptr(), w.data_ptr(), _lib.ptr(da), _lib.ptr(dw),
                  _lib.ATS_BF16, M, N, K, ws.data_ptr(), wsb, st)
        return da, dw


def _matmul_nt(a: torch.Tensor, w: torch.Tensor) -> torch.Tensor:
    """a [M, K] @ w [N, K]^T in a's dtype (float32 accumulation), on CUDA."""
    _lib.require_cuda("fused_mla_kv_decompress", a, w)
    M, K = a.shape
    N = w.shape[0]
    if (a.dtype == torch.bfloat16 and w.dtype == torch.bfloat16
            and _lib.query("ats_gemm_supported", _lib.ATS_BF16, M, N, K) == 1):
        return _MatmulNT.apply(a.contiguous(), w.contiguous())
    return (a @ w.t()).to(a.dtype)


def _triton_matmul(a: torch.Tensor, b: torch.Tensor) -> torch.Tensor:
    """a: [M, K], b: [K, N] -> [M, N] in a's dtype, accumulated in float32 (mla_triton.py:78-104)."""
    M, K = a.shape
    K2, N = b.shape
    if K != K2:
        raise ValueError(f"_triton_matmul: inner dims must match, got {K} and {K2}.")
    return _matmul_nt(a, b.t())


def fused_mla_kv_decompress(
    c: torch.Tensor,
    w_uk: torch.Tensor,
    w_uv: torch.Tensor,
) -> tuple[torch.Tensor, torch.Tensor]:
    """(k, v) = (c @ w_uk.T, c @ w_uv.T) from the shared latent c [..., latent_dim];
    w_uk, w_uv [out_dim, latent_dim] (nn.Linear layout).  One GEMM against the
    stacked weight, split in two."""
    if c.shape[-1] != w_uk.shape[-1] or c.shape[-1] != w_uv.shape[-1]:
        raise ValueError(
            f"fused_mla_kv_decompress: c's last dim ({c.shape[-1]}) must match "
            f"w_uk/w_uv's last dim ({w_uk.shape[-1]}, {w_uv.shape[-1]})."
        )
    if w_uk.shape[0] != w_uv.shape[0]:
        raise ValueError(
            f"fused_mla_kv_decompress: w_uk and w_uv must have the same output dim, "
            f"got {w_uk.shape[0]} and {w_uv.shape[0]}."
        )
    orig_shape = c.shape
    latent_dim = orig_shape[-1]
    out_dim = w_uk.shape[0]
    c_flat = c.reshape(-1, latent_dim)
    if _lib.on_cpu("fused_mla_kv_decompress", c, w_uk, w_uv):
        k_flat, v_flat = c_flat @ w_uk.t(), c_flat @ w_uv.t()
        return k_flat.reshape(*orig_shape[:-1], out_dim), v_flat.reshape(*orig_shape[:-1], out_dim)
    combined = _matmul_nt(c_flat, torch.cat([w_uk, w_uv], dim=0))  # [rows, 2*out_dim]
    k_flat, v_flat = combined.split(out_dim, dim=-1)
    return k_flat.reshape(*orig_shape[:-1], out_dim), v_flat.reshape(*orig_shape[:-1], out_dim)

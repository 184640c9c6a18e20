"""Single-tensor fused RoPE -- mirror of ats/model/rope_triton.py.

``fused_apply_rope(x, cos, sin)`` validates like rope_triton.py:115-125 and
applies the rotate-half rotation of rope.py:83-86 to one [B,H,S,D] tensor in
one CUDA pass, reading x through its strides (the reference's Triton wrapper
copied x to contiguous first, rope_triton.py:83).  It is differentiable.
``_cuda_apply_rope`` is the kernel call without validation.

As in the reference module, ``HAS_TRITON`` says whether the fused GPU kernel
is available (here: whether the CUDA library is built; no Triton is
involved), ``_triton_apply_rope`` is the fused kernel call and
``_pytorch_apply_rope`` the plain torch formula the reference's tests compare
it against (tests/test_triton.py:152-167).  ``fused_apply_rope`` runs that
formula for CPU tensors, as the reference does (rope_triton.py:126-128); CUDA
tensors always take the kernel.
"""

from __future__ import annotations

import torch

from ats_v2_b200 import _lib
from ats_v2_b200.rope import _launch, _prepare, _RopeFn, rotate_half

HAS_TRITON = _lib.LIB_PATH.exists()  # the reference's flag name: fused GPU kernel available


def _cuda_apply_rope(x: torch.Tensor, cos: torch.Tensor, sin: torch.Tensor) -> torch.Tensor:
    x, _, cos, sin, cs = _prepare(x, None, cos, sin, "fused_apply_rope")
    return _RopeFn.apply(x, None, cos, sin, cs)[0]


# fused-kernel name of the reference module (tests/test_triton.py:152-167)
_triton_apply_rope = _cuda_apply_rope


def _pytorch_apply_rope(x: torch.Tensor, cos: torch.Tensor, sin: torch.Tensor) -> torch.Tensor:
    """The torch formula of rope_triton.py:100-105, the comparison of the reference's kernel test."""
    c, s = cos[None, None], sin[None, None]
    return x * c + rotate_half(x) * s


def fused_apply_rope(x: torch.Tensor, cos: torch.Tensor, sin: torch.Tensor) -> torch.Tensor:
    """RoPE on x [batch, heads, seq_len, head_dim] with cos/sin [seq_len, head_dim]."""
    if x.dim() != 4:
        raise ValueError(
            f"fused_apply_rope expected x of shape [batch, heads, seq_len, head_dim], "
            f"got {tuple(x.shape)}."
        )
    if x.shape[-1] != cos.shape[-1]:
        raise ValueError(
            f"fused_apply_rope: x head_dim ({x.shape[-1]}) must match cos/sin dim "
            f"({cos.shape[-1]})."
        )
    if _lib.on_cpu("fused_apply_rope", x, cos, sin):
        return _pytorch_apply_rope(x, cos, sin)
    return _cuda_apply_rope(x, cos, sin)


class _QKProjRopeFn(torch.autograd.Function):
    """[q | k] = rope(x W_q^T | x W_k^T) on the tensor-core GEMM with the rotation in its epilogue (forward);
    the rotation's adjoint on the RoPE kernel, then the GEMM backward of each projection."""

    @staticmethod
    def forward(ctx, x2, w_q, w_k, cos, sin, seq):
        T, H = x2.shape
        Nq, Nk = w_q.shape[0], w_k.shape[0]
        out = torch.empty((T, Nq + Nk), dtype=x2.dtype, device=x2.device)
        wsb = _lib.query("ats_gemm_workspace_bytes")
        ws = torch.empty(wsb, dtype=torch.uint8, device=x2.device)
        st = _lib.stream_of(x2)
        for w, col0, N in ((w_q, 0, Nq), (w_k, Nq, Nk)):
            _lib.call("ats_gemm_rope_fwd", x2.data_ptr(), w.data_ptr(), out[:, col0:].data_ptr(), Nq + Nk,
                      _lib.ATS_BF16, T, N, H, cos.data_ptr(), sin.data_ptr(), seq, ws.data_ptr(), wsb, st)
        ctx.save_for_backward(x2, w_q, w_k, cos, sin)
        ctx.seq = seq
        return out

    @staticmethod
    def backward(ctx, dout):
        x2, w_q, w_k, cos, sin = ctx.saved_tensors
        T, H = x2.shape
        Nq, Nk = w_q.shape[0], w_k.shape[0]
        S, D = ctx.seq, 128
        B = T // S
        dout = dout.contiguous()
        dq = torch.empty((T, Nq), dtype=x2.dtype, device=x2.device)
        dk = torch.empty((T, Nk), dtype=x2.dtype, device=x2.device)

        def heads(t, n):  # [T, n*D] rows of [B, S] as the [B, heads, S, D] view
            return t.view(B, S, n // D, D).transpose(1, 2)

        # the rotation's adjoint, read from the [q | k] gradient through its strides
        gq = dout[:, :Nq].view(B, S, Nq // D, D).transpose(1, 2)
        gk = dout[:, Nq:].view(B, S, Nk // D, D).transpose(1, 2)
        _launch(gq, heads(dq, Nq), gk, heads(dk, Nk), cos, sin, D, True)
        wsb = _lib.query("ats_gemm_workspace_bytes")
        ws = torch.empty(wsb, dtype=torch.uint8, device=x2.device)
        st = _lib.stream_of(x2)
        dx = torch.empty_like(x2)
        dxk = torch.empty_like(x2)
        dwq = torch.empty_like(w_q)
        dwk = torch.empty_like(w_k)
        _lib.call("ats_gemm_bwd", dq.data_ptr(), x2.data_ptr(), w_q.data_ptr(), dx.data_ptr(), dwq.data_ptr(),
                  _lib.ATS_BF16, T, Nq, H, ws.data_ptr(), wsb, st)
        _lib.call("ats_gemm_bwd", dk.data_ptr(), x2.data_ptr(), w_k.data_ptr(), dxk.data_ptr(), dwk.data_ptr(),
                  _lib.ATS_BF16, T, Nk, H, ws.data_ptr(), wsb, st)
        return dx.add_(dxk), dwq, dwk, None, None, None


def fused_qk_proj_rope(x: torch.Tensor, w_q: torch.Tensor, w_k: torch.Tensor, cos: torch.Tensor,
                       sin: torch.Tensor) -> tuple[torch.Tensor, torch.Tensor]:
    """The q/k projections of attention with the rotary embedding (ats/model/attention.py:179-199):
    ``q = (x W_q^T)`` viewed ``[B, heads, S, 128]``, ``k`` likewise, both rotated with cos/sin
    ``[S, 128]`` (the RotaryEmbedding cache, cast to x's dtype).  bf16 CUDA tensors whose shapes
    the tensor-core tiling covers run one GEMM per projection with the rotation in its epilogue
    (no pass over the projected rows between the GEMM and the rotation); other CUDA shapes run the
    projection and the RoPE kernel one after the other; CPU tensors take the reference's torch
    operations.  Returns (q, k) as ``[B, heads, S, 128]`` views of one ``[B, S, (Hq+Hk)*128]``
    buffer."""
    if x.dim() != 3:
        raise ValueError(f"fused_qk_proj_rope expected x of shape [batch, seq_len, hidden], got {tuple(x.shape)}.")
    B, S, H = x.shape
    D = cos.shape[-1]
    if w_q.shape[-1] != H or w_k.shape[-1] != H or w_q.shape[0] % D or w_k.shape[0] % D:
        raise ValueError(f"fused_qk_proj_rope: weights {tuple(w_q.shape)}, {tuple(w_k.shape)} must be "
                         f"[heads*{D}, {H}].")
    if cos.shape != (S, D) or sin.shape != (S, D):
        raise ValueError(f"fused_qk_proj_rope: cos/sin must be [{S}, {D}], got {tuple(cos.shape)}, {tuple(sin.shape)}")
    Hq, Hk = w_q.shape[0] // D, w_k.shape[0] // D
    if _lib.on_cpu("fused_qk_proj_rope", x, w_q, w_k, cos, sin):
        from ats_v2_b200.rope import apply_rotary_pos_emb

        q = (x @ w_q.t()).view(B, S, Hq, D).transpose(1, 2)
        k = (x @ w_k.t()).view(B, S, Hk, D).transpose(1, 2)
        return apply_rotary_pos_emb(q, k, cos, sin)
    T = B * S
    ok = (D == 128 and x.dtype == w_q.dtype == w_k.dtype == cos.dtype == sin.dtype == torch.bfloat16
          and _lib.query("ats_gemm_supported", _lib.ATS_BF16, T, w_q.shape[0], H) == 1
          and _lib.query("ats_gemm_supported", _lib.ATS_BF16, T, w_k.shape[0], H) == 1)
    if not ok:
        from ats_v2_b200.mla_fused import _matmul_nt
        from ats_v2_b200.rope import apply_rotary_pos_emb

        x2 = x.reshape(T, H)
        q = _matmul_nt(x2, w_q).view(B, S, Hq, D).transpose(1, 2)
        k = _matmul_nt(x2, w_k).view(B, S, Hk, D).transpose(1, 2)
        return apply_rotary_pos_emb(q, k, cos, sin)
    out = _QKProjRopeFn.apply(x.reshape(T, H).contiguous(), w_q.contiguous(), w_k.contiguous(), cos.contiguous(),
                              sin.contiguous(), S)
    qk = out.view(B, S, Hq + Hk, D)
    return qk[:, :, :Hq].transpose(1, 2), qk[:, :, Hq:].transpose(1, 2)

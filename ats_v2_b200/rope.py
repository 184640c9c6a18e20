"""Rotary position embedding on the sm_100a kernels -- mirror of
ats/model/rope.py.

* ``RotaryEmbedding(dim, max_seq_len=4096, theta=10000.)`` builds the same
  float32 ``inv_freq`` and cos/sin cache as rope.py:17-43 (same torch
  expressions, so the tables are identical), grows it by doubling
  (rope.py:50-59), and returns tables cast to the requested device/dtype
  (rope.py:60-61).  The cast tables are cached per (device, dtype) instead of
  being re-cast on every call.
* ``apply_rotary_pos_emb(q, k, cos, sin)`` (rope.py:71-87) rotates q and k
  in ONE kernel launch (``ats_rope_apply``) that reads the strided [B,H,S,D]
  views in place (the attention layout hands in transposed BSHD memory) and
  writes outputs with the inputs' strides; its backward is the adjoint
  rotation, again one launch.
* ``rotate_half`` is kept for API compatibility (rope.py:65-68).
"""

from __future__ import annotations

import torch
from torch import nn

from ats_v2_b200 import _lib


class RotaryEmbedding(nn.Module):
    """Drop-in for ats.model.rope.RotaryEmbedding."""

    def __init__(self, dim: int, max_seq_len: int = 4096, theta: float = 10000.0) -> None:
        super().__init__()
        if dim % 2 != 0:
            raise ValueError(
                f"RotaryEmbedding dim must be even, got {dim}. "
                f"Fix: head_dim (hidden_size // num_heads) must be even."
            )
        self.dim = dim
        self.theta = theta
        inv_freq = 1.0 / (theta ** (torch.arange(0, dim, 2, dtype=torch.float32) / dim))
        self.inv_freq: torch.Tensor
        self.register_buffer("inv_freq", inv_freq, persistent=False)
        self._cached_seq_len = 0
        self._cast: dict = {}
        self._build_cache(max_seq_len)

    def _build_cache(self, seq_len: int) -> None:
        t = torch.arange(seq_len, dtype=torch.float32, device=self.inv_freq.device)
        freqs = torch.outer(t, self.inv_freq)
        emb = torch.cat([freqs, freqs], dim=-1)
        self.register_buffer("_cached_cos", emb.cos(), persistent=False)
        self.register_buffer("_cached_sin", emb.sin(), persistent=False)
        self._cached_seq_len = seq_len
        self._cast = {}

    def _apply(self, fn, recurse=True):  # .to()/.cuda() move the buffers: drop cast copies
        self._cast = {}
        return super()._apply(fn, recurse)

    def forward(self, seq_len: int, device: torch.device, dtype: torch.dtype):
        if seq_len <= 0:
            raise ValueError(f"RotaryEmbedding requires seq_len > 0, got {seq_len}.")
        if seq_len > self._cached_seq_len:
            new_len = max(seq_len, self._cached_seq_len * 2 if self._cached_seq_len > 0 else seq_len)
            self._build_cache(new_len)
        key = (torch.device(device), dtype)
        full = self._cast.get(key)
        if full is None:
            full = (self._cached_cos.to(device=device, dtype=dtype),
                    self._cached_sin.to(device=device, dtype=dtype))
            self._cast[key] = full
        return full[0][:seq_len], full[1][:seq_len]


def rotate_half(x: torch.Tensor) -> torch.Tensor:
    """cat(-x2, x1) over the last dim (rope.py:65-68); not used by the kernels."""
    half = x.shape[-1] // 2
    return torch.cat((-x[..., half:], x[..., :half]), dim=-1)


def _last_dim_contig(t: torch.Tensor) -> torch.Tensor:
    return t if t.stride(-1) == 1 else t.contiguous()


def _table(t: torch.Tensor, D: int, S: int, name: str) -> tuple[torch.Tensor, int]:
    if t.dim() != 2 or t.shape[-1] != D or t.shape[0] not in (S, 1):
        raise ValueError(f"{name}: cos/sin must be [seq_len={S} (or 1), {D}], got {tuple(t.shape)}")
    t = _last_dim_contig(t)
    return t, (0 if t.shape[0] == 1 else t.stride(0))


def _launch(q_in, q_out, k_in, k_out, cos, sin, cs_stride, backward: bool) -> None:
    B, Hq, S, D = q_in.shape
    Hk = k_in.shape[1] if k_in is not None else 0
    qs = _lib.strides3(q_in.stride(0), q_in.stride(1), q_in.stride(2))
    qo = _lib.strides3(q_out.stride(0), q_out.stride(1), q_out.stride(2))
    ks = _lib.strides3(k_in.stride(0), k_in.stride(1), k_in.stride(2)) if k_in is not None else None
    ko = _lib.strides3(k_out.stride(0), k_out.stride(1), k_out.stride(2)) if k_in is not None else None
    _lib.call("ats_rope_apply", q_in.data_ptr(), q_out.data_ptr(), Hq, qs, qo,
              _lib.ptr(k_in), _lib.ptr(k_out), Hk, ks, ko, cos.data_ptr(), sin.data_ptr(), cs_stride,
              B, S, D, _lib.dtype_code(q_in.dtype), 1 if backward else 0, _lib.stream_of(q_in))


class _RopeFn(torch.autograd.Function):
    @staticmethod
    def forward(ctx, q, k, cos, sin, cs_stride):
        ctx.set_materialize_grads(False)  # an unused output's gradient arrives as None, not zeros
        q_out = torch.empty_like(q)
        k_out = torch.empty_like(k) if k is not None else None
        _launch(q, q_out, k, k_out, cos, sin, cs_stride, False)
        ctx.save_for_backward(cos, sin)
        ctx.cs_stride = cs_stride
        ctx.has_k = k is not None
        return q_out, k_out

    @staticmethod
    def backward(ctx, dq_out, dk_out):
        cos, sin = ctx.saved_tensors
        if dq_out is None and (dk_out is None or not ctx.has_k):
            return None, None, None, None, None
        if dq_out is None:  # only k was used downstream: run its adjoint alone
            dk_out = _last_dim_contig(dk_out)
            dk = torch.empty_like(dk_out)
            _launch(dk_out, dk, None, None, cos, sin, ctx.cs_stride, True)
            return None, dk, None, None, None
        dq_out = _last_dim_contig(dq_out)
        dq = torch.empty_like(dq_out)
        dk = None
        if ctx.has_k and dk_out is not None:
            dk_out = _last_dim_contig(dk_out)
            dk = torch.empty_like(dk_out)
        _launch(dq_out, dq, dk_out if dk is not None else None, dk, cos, sin, ctx.cs_stride, True)
        return dq, dk, None, None, None


def _prepare(q: torch.Tensor, k: torch.Tensor | None, cos: torch.Tensor, sin: torch.Tensor, name: str):
    _lib.require_cuda(name, q, k, cos, sin)
    if cos.requires_grad or sin.requires_grad:
        raise NotImplementedError(f"{name}: gradients w.r.t. cos/sin are not supported")
    out_dtype = torch.promote_types(q.dtype, cos.dtype)
    if k is not None:
        if k.dtype != q.dtype:
            raise TypeError(f"{name}: q and k must share a dtype ({q.dtype} vs {k.dtype})")
        if k.dim() != 4 or k.shape[0] != q.shape[0] or k.shape[2] != q.shape[2] or k.shape[3] != q.shape[3]:
            raise ValueError(f"{name}: k shape {tuple(k.shape)} incompatible with q {tuple(q.shape)}")
    # torch promotes x*cos to the wider dtype; upcasting the narrower operand is exact
    q = _last_dim_contig(q.to(out_dtype))
    k = _last_dim_contig(k.to(out_dtype)) if k is not None else None
    cos, cs_stride = _table(cos.to(out_dtype), q.shape[-1], q.shape[2], name)
    sin, ss_stride = _table(sin.to(out_dtype), q.shape[-1], q.shape[2], name)
    if cs_stride != ss_stride:  # one table broadcast, the other not: materialise both
        S, D = q.shape[2], q.shape[3]
        cos = cos.expand(S, D).contiguous()
        sin = sin.expand(S, D).contiguous()
        cs_stride = D
    return q, k, cos, sin, cs_stride


def apply_rotary_pos_emb(q: torch.Tensor, k: torch.Tensor, cos: torch.Tensor,
                         sin: torch.Tensor) -> tuple[torch.Tensor, torch.Tensor]:
    """q, k: [batch, heads, seq_len, head_dim] (any b/h/s strides); cos, sin: [seq_len, head_dim].
    One CUDA launch rotates q and k; CPU tensors take the reference's torch formula."""
    if q.shape[-1] != cos.shape[-1]:
        raise ValueError(
            f"apply_rotary_pos_emb: q head_dim ({q.shape[-1]}) does not match "
            f"cos/sin dim ({cos.shape[-1]})."
        )
    if _lib.on_cpu("apply_rotary_pos_emb", q, k, cos, sin):
        # CPU tensors: the reference's torch formula (rope.py:83-86)
        c, s = cos[None, None], sin[None, None]
        return q * c + rotate_half(q) * s, (k * c + rotate_half(k) * s if k is not None else None)
    if q.dim() != 4:
        raise ValueError(f"apply_rotary_pos_emb: q must be [batch, heads, seq_len, head_dim], got {tuple(q.shape)}")
    q, k, cos, sin, cs = _prepare(q, k, cos, sin, "apply_rotary_pos_emb")
    return _RopeFn.apply(q, k, cos, sin, cs)

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
from ats_v2_b200.rope import _prepare, _RopeFn, rotate_half

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

"""The q/k projections with the rotary embedding in the GEMM's epilogue
(``fused_qk_proj_rope``, ``ats_gemm_rope_fwd``; ats/model/attention.py:179-199).

The fused forward must equal, bit for bit, the projection on the same
tensor-core GEMM followed by the RoPE kernel (the same accumulation, then the
same bf16 roundings of rope.py:83-86), and match the oracle's rotation of the
float64 product rounded to bf16.  The backward (the rotation's adjoint, then
each projection's GEMM backward) must equal the unfused graph's gradients."""

from __future__ import annotations

import numpy as np
import pytest
import torch

from ats_v2_b200.mla_fused import _matmul_nt
from ats_v2_b200.rope import RotaryEmbedding, apply_rotary_pos_emb
from ats_v2_b200.rope_fused import fused_qk_proj_rope
from oracle import rope as orope
from oracle.bf16 import round_bf16
from tests.util import close, np32

pytestmark = pytest.mark.gpu


def _unfused(x, wq, wk, cos, sin):
    B, S, H = x.shape
    x2 = x.reshape(B * S, H)
    q = _matmul_nt(x2, wq).view(B, S, -1, 128).transpose(1, 2)
    k = _matmul_nt(x2, wk).view(B, S, -1, 128).transpose(1, 2)
    return apply_rotary_pos_emb(q, k, cos, sin)


@pytest.mark.parametrize("B,S,H,Hq,Hk", [(2, 256, 512, 4, 2), (1, 384, 1024, 8, 8), (4, 128, 256, 2, 1)])
def test_fused_projection_rope_equals_the_unfused_pair(B, S, H, Hq, Hk):
    g = torch.Generator(device="cuda").manual_seed(B * 1000 + S + H)
    x = torch.randn(B, S, H, device="cuda", generator=g).bfloat16()
    wq = (0.05 * torch.randn(Hq * 128, H, device="cuda", generator=g)).bfloat16()
    wk = (0.05 * torch.randn(Hk * 128, H, device="cuda", generator=g)).bfloat16()
    cos, sin = RotaryEmbedding(128, S, 500000.0).cuda()(S, x.device, torch.bfloat16)
    xa, wqa, wka = (t.clone().requires_grad_() for t in (x, wq, wk))
    xb, wqb, wkb = (t.clone().requires_grad_() for t in (x, wq, wk))
    qa, ka = fused_qk_proj_rope(xa, wqa, wka, cos, sin)
    qb, kb = _unfused(xb, wqb, wkb, cos, sin)
    assert qa.shape == (B, Hq, S, 128) and ka.shape == (B, Hk, S, 128)
    assert torch.equal(qa, qb) and torch.equal(ka, kb)
    # the oracle: float64 products rounded once to bf16, then the reference's bf16 rotation
    q64 = round_bf16((np32(x).astype(np.float64) @ np32(wq).astype(np.float64).T).astype(np.float32))
    qo = orope.rope_fwd(q64.reshape(B, S, Hq, 128).transpose(0, 2, 1, 3), np32(cos), np32(sin), "bf16")
    close(qa, qo, "bf16", min_exact=0.98)
    gq = torch.randn(qa.shape, device="cuda", generator=g).bfloat16()
    gk = torch.randn(ka.shape, device="cuda", generator=g).bfloat16()
    torch.autograd.backward([qa, ka], [gq, gk])
    torch.autograd.backward([qb, kb], [gq, gk])
    assert torch.equal(xa.grad, xb.grad)
    assert torch.equal(wqa.grad, wqb.grad) and torch.equal(wka.grad, wkb.grad)


"""Rotary embedding on the CUDA kernel vs the golden vectors and the oracle.

The kernel rounds after every multiply and add exactly as the reference's
torch ops do, so besides the north-star tolerance (float32 1e-5 relative,
bfloat16 2e-2 / 1e-2) the tests require (near-)bit-identical results."""

from __future__ import annotations

import numpy as np
import pytest
import torch

from ats_v2_b200.rope import RotaryEmbedding, apply_rotary_pos_emb
from ats_v2_b200.rope_fused import _cuda_apply_rope, fused_apply_rope
from oracle import rope as orope
from oracle.bf16 import round_bf16
from tests.conftest import load_golden
from tests.util import close, dev, np32, seeded_normal

pytestmark = pytest.mark.gpu


def _bshd_views(q_np, k_np, dtype):
    """BSHD memory handed in as [B,H,S,D] views, as attention.py:179-193 does."""
    q = dev(q_np, dtype).transpose(1, 2).requires_grad_()
    k = dev(k_np, dtype).transpose(1, 2).requires_grad_()
    return q, k


@pytest.mark.parametrize("tag,dtype,dn", [("f", torch.float32, "f32"), ("b", torch.bfloat16, "bf16")])
def test_golden(tag, dtype, dn):
    g = load_golden("rope")
    q, k = _bshd_views(g[f"{tag}_q"], g[f"{tag}_k"], dtype)
    cos, sin = dev(g[f"{tag}_cos"], dtype), dev(g[f"{tag}_sin"], dtype)
    qo, ko = apply_rotary_pos_emb(q, k, cos, sin)
    assert qo.stride() == q.stride() and ko.stride() == k.stride()  # written in the input layout
    close(qo, g[f"{tag}_qo"], dn, min_exact=0.999)
    close(ko, g[f"{tag}_ko"], dn, min_exact=0.999)
    torch.autograd.backward([qo, ko], [dev(g[f"{tag}_gq"], dtype), dev(g[f"{tag}_gk"], dtype)])
    close(q.grad, g[f"{tag}_dq"], dn, min_exact=0.999)
    close(k.grad, g[f"{tag}_dk"], dn, min_exact=0.999)


def test_single_tensor_entry_golden():
    g = load_golden("rope")
    y = fused_apply_rope(dev(g["t_x"]), dev(g["t_cos"]), dev(g["t_sin"]))
    close(y, g["t_y"], "f32", min_exact=0.999)


def test_reference_parity_test():
    """tests/test_triton.py:152-167 of the reference, on the CUDA kernel."""
    torch.manual_seed(0)
    head_dim = 16
    q = torch.randn(2, 4, 8, head_dim, device="cuda")
    rope = RotaryEmbedding(head_dim, max_seq_len=16, theta=10000.0)
    cos, sin = rope(seq_len=8, device=torch.device("cuda"), dtype=torch.float32)
    out = _cuda_apply_rope(q, cos, sin)
    ref = orope.rope_fwd(np32(q), np32(cos), np32(sin))
    assert torch.allclose(out, dev(ref), atol=1e-5)


def test_cpu_parity_workload_shape_f32():
    """q,k [4,256,8,64] fp32 (BSHD), positions 0..255, theta 1e4."""
    qn, kn = seeded_normal((4, 256, 8, 64), 10), seeded_normal((4, 256, 8, 64), 11)
    q, k = _bshd_views(qn, kn, torch.float32)
    cos, sin = RotaryEmbedding(64, 256, 10000.0).cuda()(256, torch.device("cuda"), torch.float32)
    qo, ko = apply_rotary_pos_emb(q, k, cos, sin)
    c, s = np32(cos), np32(sin)
    close(qo, orope.rope_fwd(qn.transpose(0, 2, 1, 3), c, s), "f32", min_exact=0.999)
    close(ko, orope.rope_fwd(kn.transpose(0, 2, 1, 3), c, s), "f32", min_exact=0.999)
    gq, gk = seeded_normal(qo.shape, 12), seeded_normal(ko.shape, 13)
    torch.autograd.backward([qo, ko], [dev(gq), dev(gk)])
    close(q.grad, orope.rope_bwd(gq, c, s), "f32", min_exact=0.999)
    close(k.grad, orope.rope_bwd(gk, c, s), "f32", min_exact=0.999)


@pytest.mark.parametrize("D", [2, 6, 8, 16, 64, 96, 128, 256])
@pytest.mark.parametrize("dn", ["f32", "bf16"])
def test_head_dims_layouts_and_q_only(D, dn):
    dtype = torch.float32 if dn == "f32" else torch.bfloat16
    B, Hq, Hk, S = 2, 3, 1, 5
    qn = seeded_normal((B, Hq, S, D), D)
    kn = seeded_normal((B, Hk, S, D), D + 1)
    if dn == "bf16":
        qn, kn = round_bf16(qn), round_bf16(kn)
    cos, sin = RotaryEmbedding(D, 8, 500000.0).cuda()(S, torch.device("cuda"), dtype)
    c, s = np32(cos), np32(sin)
    q = dev(qn, dtype)  # contiguous BHSD this time
    k = dev(kn, dtype)
    qo, ko = apply_rotary_pos_emb(q, k, cos, sin)
    close(qo, orope.rope_fwd(qn, c, s, dn), dn, min_exact=0.999)
    close(ko, orope.rope_fwd(kn, c, s, dn), dn, min_exact=0.999)
    y = fused_apply_rope(q, cos, sin)
    close(y, orope.rope_fwd(qn, c, s, dn), dn, min_exact=0.999)


def test_broadcast_single_row_and_promoted_dtype():
    qn = round_bf16(seeded_normal((1, 2, 4, 8), 3))
    cos = torch.tensor([[0.5] * 8], device="cuda")
    sin = torch.tensor([[0.25] * 8], device="cuda")
    y = fused_apply_rope(dev(qn, torch.bfloat16), cos, sin)  # bf16 x * f32 table -> f32, as torch promotes
    assert y.dtype == torch.float32
    close(y, orope.rope_fwd(qn, np.full((4, 8), 0.5, np.float32), np.full((4, 8), 0.25, np.float32)), "f32")


def test_only_k_used_downstream():
    qn, kn = seeded_normal((1, 2, 4, 8), 4), seeded_normal((1, 1, 4, 8), 5)
    q, k = dev(qn, requires_grad=True), dev(kn, requires_grad=True)
    cos, sin = RotaryEmbedding(8, 8).cuda()(4, torch.device("cuda"), torch.float32)
    _, ko = apply_rotary_pos_emb(q, k, cos, sin)
    gk = seeded_normal(ko.shape, 6)
    ko.backward(dev(gk))
    assert q.grad is None
    close(k.grad, orope.rope_bwd(gk, np32(cos), np32(sin)), "f32")


def test_full_size_7b_config_sampled_positions():
    """q [4,4096,32,128], k [4,4096,8,128] bf16 (BSHD), theta 5e5: 48 sampled
    (batch, position) pairs checked on all heads against the oracle."""
    gen = torch.Generator(device="cuda").manual_seed(0)
    qm = torch.randn(4, 4096, 32, 128, device="cuda", generator=gen).bfloat16()
    km = torch.randn(4, 4096, 8, 128, device="cuda", generator=gen).bfloat16()
    q, k = qm.transpose(1, 2).requires_grad_(), km.transpose(1, 2).requires_grad_()
    cos, sin = RotaryEmbedding(128, 4096, 500000.0).cuda()(4096, torch.device("cuda"), torch.bfloat16)
    qo, ko = apply_rotary_pos_emb(q, k, cos, sin)
    gq = torch.randn(qo.shape, device="cuda", generator=gen).bfloat16()
    gk = torch.randn(ko.shape, device="cuda", generator=gen).bfloat16()
    torch.autograd.backward([qo, ko], [gq, gk])
    bs = torch.randint(0, 4, (48,), generator=torch.Generator().manual_seed(1))
    ss = torch.randint(0, 4096, (48,), generator=torch.Generator().manual_seed(2))
    c, s = np32(cos), np32(sin)
    for b, p in zip(bs.tolist(), ss.tolist()):
        cp, sp = c[p:p + 1], s[p:p + 1]
        for x, xo, gx, dx in ((q, qo, gq, q.grad), (k, ko, gk, k.grad)):
            xin = np32(x[b:b + 1, :, p:p + 1])
            close(xo[b:b + 1, :, p:p + 1], orope.rope_fwd(xin, cp, sp, "bf16"), "bf16", min_exact=0.999)
            gin = np32(gx[b:b + 1, :, p:p + 1])
            close(dx[b:b + 1, :, p:p + 1], orope.rope_bwd(gin, cp, sp, "bf16"), "bf16", min_exact=0.999)

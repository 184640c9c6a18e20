"""The names the reference's kernel tests import from its ``*_triton`` modules.

The reference's tests/test_triton.py imports ``HAS_TRITON``, the public fused
functions and the private ``_triton_*`` / ``_pytorch_*`` pairs from
ats/model/{norm,rope,moe}_triton.py (tests/test_triton.py:19-25,142-187).
The mirror modules keep every one of those names.  On CPU this checks that
they exist, that the plain torch formulas agree with the oracle (so the GPU
comparison below is against the right thing), and that the kernel calls
refuse CPU tensors.  On GPU the
reference's three kernel-vs-formula comparisons run as that file writes them
(same shapes, seeds and 1e-5 tolerances)."""

from __future__ import annotations

import numpy as np
import pytest
import torch

from ats_v2_b200 import mla_fused, moe_fused, norm_fused, rope_fused
from ats_v2_b200.rope import RotaryEmbedding
from oracle import moe as omoe
from oracle import norm as onorm
from oracle import rope as orope


def test_reference_test_names_exist():
    for mod, names in ((norm_fused, ("HAS_TRITON", "fused_rmsnorm_residual", "_triton_rmsnorm_residual",
                                     "_pytorch_rmsnorm_residual")),
                       (rope_fused, ("HAS_TRITON", "fused_apply_rope", "_triton_apply_rope", "_pytorch_apply_rope")),
                       (moe_fused, ("HAS_TRITON", "fused_moe_routing", "fused_moe_dispatch", "_triton_moe_routing",
                                    "_pytorch_moe_routing")),
                       (mla_fused, ("HAS_TRITON", "fused_mla_kv_decompress", "_triton_matmul"))):
        for n in names:
            assert hasattr(mod, n), f"{mod.__name__}.{n}"
        assert isinstance(mod.HAS_TRITON, bool)


def test_torch_formulas_match_the_oracle():
    g = torch.Generator().manual_seed(0)
    x = torch.randn(2, 5, 16, generator=g)
    res = torch.randn(2, 5, 16, generator=g)
    w = torch.randn(16, generator=g)
    got = norm_fused._pytorch_rmsnorm_residual(x, res, w, 1e-6)
    ref = onorm.rmsnorm_residual_fwd(x.numpy(), res.numpy(), w.numpy(), 1e-6)[0]
    np.testing.assert_allclose(got.numpy(), ref, rtol=1e-5, atol=1e-6)

    logits = torch.randn(32, 8, generator=g)
    p, i = moe_fused._pytorch_moe_routing(logits, 2)
    rp, ri = omoe.route(logits.numpy(), 2)[:2]
    assert np.array_equal(i.numpy(), ri)
    np.testing.assert_allclose(p.numpy(), rp, rtol=1e-5, atol=1e-7)

    q = torch.randn(1, 2, 6, 8, generator=g)
    cos, sin = (torch.from_numpy(np.ascontiguousarray(t)) for t in orope.cos_sin_cache(6, 8, 10000.0))
    got = rope_fused._pytorch_apply_rope(q, cos, sin)
    ref = orope.rope_fwd(q.numpy(), cos.numpy(), sin.numpy())
    np.testing.assert_allclose(got.numpy(), ref, rtol=1e-5, atol=1e-6)


def test_kernel_calls_refuse_cpu_tensors():
    """The ``_triton_*`` kernel calls take CUDA tensors only (the public
    functions route CPU tensors to the torch formulas, as the reference does)."""
    x = torch.randn(2, 5, 16)
    with pytest.raises(RuntimeError):
        norm_fused._triton_rmsnorm_residual(x, x.clone(), torch.ones(16), 1e-6)
    with pytest.raises(RuntimeError):
        rope_fused._triton_apply_rope(torch.randn(1, 2, 6, 8), torch.ones(6, 8), torch.zeros(6, 8))
    with pytest.raises(RuntimeError):
        moe_fused._triton_moe_routing(torch.randn(4, 8), 2)
    with pytest.raises(RuntimeError):
        mla_fused._triton_matmul(torch.randn(10, 8), torch.randn(8, 16))


def test_mla_dim_mismatch_raises_before_any_device_work():
    """tests/test_triton.py:121-126 of the reference."""
    c = torch.randn(2, 5, 8)
    with pytest.raises(ValueError):
        mla_fused.fused_mla_kv_decompress(c, torch.randn(16, 8), torch.randn(16, 4))
    with pytest.raises(ValueError):
        mla_fused.fused_mla_kv_decompress(c, torch.randn(16, 8), torch.randn(12, 8))
    with pytest.raises(ValueError):
        mla_fused._triton_matmul(torch.randn(4, 8), torch.randn(6, 3))


@pytest.mark.gpu
def test_rmsnorm_residual_kernel_matches_torch_formula():
    torch.manual_seed(0)
    x = torch.randn(4, 32, device="cuda")
    residual = torch.randn(4, 32, device="cuda")
    weight = torch.randn(32, device="cuda")
    out = norm_fused._triton_rmsnorm_residual(x, residual, weight, eps=1e-6)
    ref = norm_fused._pytorch_rmsnorm_residual(x, residual, weight, eps=1e-6)
    assert torch.allclose(out, ref, atol=1e-5)


@pytest.mark.gpu
def test_rope_kernel_matches_torch_formula():
    torch.manual_seed(0)
    q = torch.randn(2, 4, 8, 16, device="cuda")
    rope = RotaryEmbedding(16, max_seq_len=16, theta=10000.0)
    cos, sin = rope(seq_len=8, device=torch.device("cuda"), dtype=torch.float32)
    out = rope_fused._triton_apply_rope(q, cos, sin)
    ref = rope_fused._pytorch_apply_rope(q, cos, sin)
    assert torch.allclose(out, ref, atol=1e-5)


@pytest.mark.gpu
def test_routing_kernel_matches_torch_formula():
    torch.manual_seed(0)
    gate_logits = torch.randn(32, 8, device="cuda")
    p, i = moe_fused._triton_moe_routing(gate_logits, top_k=2)
    rp, ri = moe_fused._pytorch_moe_routing(gate_logits, top_k=2)
    assert torch.equal(i.sort(dim=-1).values, ri.sort(dim=-1).values)
    assert torch.allclose(p.sort(dim=-1).values, rp.sort(dim=-1).values, atol=1e-5)
    # stronger than the reference's check: same order, not only the same set
    assert torch.equal(i, ri)

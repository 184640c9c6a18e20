"""Host-side logic of the reference-mirroring modules (CPU only): argument
validation with the reference's ValueErrors, CPU tensors on the reference's
formulas while the kernel calls refuse them, RoPE cache construction, capacity, stacked expert storage, the lazy
utilisation dict, and module construction (state-dict names, init)."""

from __future__ import annotations

import numpy as np
import pytest
import torch

from ats_v2_b200 import moe as bmoe
from ats_v2_b200.moe_fused import fused_moe_dispatch, fused_moe_routing
from ats_v2_b200.norm import RMSNorm
from ats_v2_b200.norm_fused import fused_rmsnorm_residual
from ats_v2_b200.rope import RotaryEmbedding, apply_rotary_pos_emb
from ats_v2_b200.rope_fused import fused_apply_rope
from oracle import rope as orope
from tests.conftest import load_golden


def test_rmsnorm_module_validation_matches_reference():
    with pytest.raises(ValueError):
        RMSNorm(0)
    norm = RMSNorm(hidden_size=6)
    assert torch.equal(norm.weight.data, torch.ones(6))
    with pytest.raises(ValueError):
        norm(torch.randn(2, 5))


def test_cpu_tensors_take_the_reference_formulas_and_kernel_calls_refuse_them():
    """CPU tensors run the reference's torch formulas (its CPU behaviour); the
    kernel entry points the reference's GPU tests call (``_triton_*``) still
    take CUDA tensors only, as the reference's Triton kernels do."""
    from ats_v2_b200.moe_fused import _triton_moe_routing
    from ats_v2_b200.norm_fused import _pytorch_rmsnorm_residual, _triton_rmsnorm_residual
    from ats_v2_b200.rope_fused import _pytorch_apply_rope, _triton_apply_rope

    x, r, w = torch.randn(2, 8), torch.randn(2, 8), torch.randn(8)
    assert torch.equal(fused_rmsnorm_residual(x, r, w), _pytorch_rmsnorm_residual(x, r, w, 1e-6))
    assert torch.equal(RMSNorm(8)(x), torch.nn.functional.rms_norm(x, (8,), torch.ones(8), 1e-6))
    cos, sin = RotaryEmbedding(8, 16)(4, torch.device("cpu"), torch.float32)
    q = torch.randn(1, 2, 4, 8)
    assert torch.equal(fused_apply_rope(q, cos, sin), _pytorch_apply_rope(q, cos, sin))
    with pytest.raises(RuntimeError, match="CUDA tensors only"):
        _triton_rmsnorm_residual(x, r, w, 1e-6)
    with pytest.raises(RuntimeError, match="CUDA tensors only"):
        _triton_apply_rope(q, cos, sin)
    with pytest.raises(RuntimeError, match="CUDA tensors only"):
        _triton_moe_routing(torch.randn(5, 4), 2)
    layer = bmoe.MoELayer(hidden_size=16, intermediate_size=32, num_experts=4, num_layers=2, top_k=2)
    out, aux = layer(torch.randn(1, 3, 16))
    assert out.shape == (1, 3, 16) and aux.dim() == 0


def test_fused_entry_points_validate_like_reference():
    with pytest.raises(ValueError):
        fused_rmsnorm_residual(torch.randn(2, 5, 16), torch.randn(2, 5, 8), torch.randn(16))
    with pytest.raises(ValueError):
        fused_rmsnorm_residual(torch.randn(2, 5, 16), torch.randn(2, 5, 16), torch.randn(8))
    with pytest.raises(ValueError):
        fused_apply_rope(torch.randn(2, 6, 8), torch.randn(6, 8), torch.randn(6, 8))
    with pytest.raises(ValueError):
        fused_apply_rope(torch.randn(1, 2, 6, 8), torch.randn(6, 4), torch.randn(6, 4))
    with pytest.raises(ValueError):
        apply_rotary_pos_emb(torch.randn(1, 2, 6, 8), torch.randn(1, 2, 6, 8), torch.randn(6, 4), torch.randn(6, 4))
    with pytest.raises(ValueError):
        fused_moe_routing(torch.randn(5, 4, 1), 2)
    with pytest.raises(ValueError):
        fused_moe_routing(torch.randn(5, 4), 0)
    with pytest.raises(ValueError):
        fused_moe_dispatch(torch.randn(6, 4), torch.randn(5, 16), top_k=2, capacity_factor=1.25)
    with pytest.raises(ValueError):
        fused_moe_dispatch(torch.randn(6, 4), torch.randn(6, 16), top_k=2, capacity_factor=0.0)
    with pytest.raises(ValueError):
        RotaryEmbedding(7)


def test_rope_cache_matches_reference_tables_and_doubles():
    g = load_golden("rope")
    r = RotaryEmbedding(128, max_seq_len=4096, theta=500000.0)
    assert np.array_equal(r.inv_freq.numpy(), g["inv_freq_128_5e5"])
    cos, sin = r(4096, torch.device("cpu"), torch.float32)
    rows = g["rows_128_5e5"]
    # same torch expressions as the reference: identical tables
    assert np.array_equal(cos.numpy()[rows], g["cos_128_5e5_rows"])
    assert np.array_equal(sin.numpy()[rows], g["sin_128_5e5_rows"])
    oc, _ = orope.cos_sin_cache(4096, 128, 500000.0)
    np.testing.assert_allclose(cos.numpy(), oc, rtol=0, atol=1e-6)
    r2 = RotaryEmbedding(8, max_seq_len=16, theta=10000.0)
    r2(20, torch.device("cpu"), torch.float32)
    assert r2._cached_seq_len == int(g["grow_16_to_20"][0]) == 32
    with pytest.raises(ValueError):
        r2(0, torch.device("cpu"), torch.float32)
    # cast tables are cached per (device, dtype) and sliced to seq_len
    c1, _ = r2(5, torch.device("cpu"), torch.bfloat16)
    c2, _ = r2(7, torch.device("cpu"), torch.bfloat16)
    assert c1.shape == (5, 8) and c2.shape == (7, 8) and c1.dtype == torch.bfloat16
    assert c1.data_ptr() == c2.data_ptr()


def test_capacity_matches_reference_formula():
    assert bmoe.capacity_for(32768, 2, 64, 1.25) == 1280
    assert bmoe.capacity_for(8192, 2, 8, 4.0) == 8192
    assert bmoe.capacity_for(3, 1, 64, 0.5) == 1


def test_stacked_expert_storage_is_shared_and_repaired():
    ps = [torch.nn.Parameter(torch.randn(6, 4)) for _ in range(3)]
    st = bmoe.stacked(ps)
    assert st.shape == (3, 6, 4)
    for e, p in enumerate(ps):
        assert p.data.data_ptr() == st[e].data_ptr()
        assert torch.equal(p.data, st[e])
    st2 = bmoe.stacked(ps)  # already stacked: a view, no copy
    assert st2.data_ptr() == st.data_ptr()
    with torch.no_grad():
        ps[1].add_(1.0)  # optimizer-style in-place update is seen through the stack
    assert torch.equal(st2[1], ps[1].data)
    ps[2].data = torch.randn(6, 4)  # e.g. after .to(): re-stacked once
    st3 = bmoe.stacked(ps)
    assert st3.data_ptr() != st.data_ptr()
    assert all(p.data.data_ptr() == st3[e].data_ptr() for e, p in enumerate(ps))


def test_lazy_utilization_behaves_like_a_dict():
    u = bmoe.LazyUtilization(torch.tensor([0.25, 0.75]))
    assert sum(u.values()) == pytest.approx(1.0)
    assert u[1] == 0.75 and len(u) == 2 and dict(u) == {0: 0.25, 1: 0.75}
    assert isinstance(u, dict)


def test_moe_layer_construction_mirrors_reference():
    torch.manual_seed(0)
    num_layers = 32
    layer = bmoe.MoELayer(hidden_size=64, intermediate_size=128, num_experts=4, num_layers=num_layers, top_k=2)
    assert layer.uses_deepspeed is False
    keys = set(layer.state_dict().keys())
    assert "moe.gate.weight" in keys
    assert "moe.experts.3.gate_up_proj.weight" in keys and "moe.experts.0.down_proj.weight" in keys
    assert layer.moe.experts[0].gate_up_proj.weight.shape == (256, 64)
    assert layer.moe.experts[0].down_proj.weight.shape == (64, 128)
    expected = bmoe.residual_output_std(num_layers)
    for ex in layer.moe.experts:
        assert ex.down_proj.weight.std().item() == pytest.approx(expected, rel=0.2)
        assert getattr(ex.down_proj.weight, "_ats_residual_init", False)
    q = bmoe.MoELayer(16, 32, 2, 2, top_k=1, quantization="int8")  # constructs, as the reference's does
    assert q.moe.experts[0].down_proj.quantization == "int8"

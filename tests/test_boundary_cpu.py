"""The drop-in boundary on CPU tensors and the MoELayer constructor.

CPU tensors take the reference's torch formulas (as the reference's own
modules do without a GPU kernel); they must agree with the oracle, which is
pinned to the reference's outputs.  ``MoELayer`` must construct int8
experts (QuantizedLinear projections) and, with ``ep_size`` > 1 in a
multi-process group, hold only its share of the experts.
"""

from __future__ import annotations

import os
import socket

import numpy as np
import pytest
import torch

from ats_v2_b200.moe import MoELayer
from ats_v2_b200.moe_fused import fused_moe_dispatch, fused_moe_routing
from ats_v2_b200.norm import RMSNorm
from ats_v2_b200.norm_fused import fused_rmsnorm_residual
from ats_v2_b200.quantization import QuantizedLinear
from ats_v2_b200.rope import RotaryEmbedding, apply_rotary_pos_emb
from ats_v2_b200.rope_fused import fused_apply_rope
from oracle import moe as omoe
from oracle import norm as onorm
from oracle import rope as orope
from tests.conftest import load_golden


def test_rmsnorm_cpu_matches_golden():
    g = load_golden("rmsnorm")
    m = RMSNorm(g["f32_x"].shape[-1], eps=1e-6)
    with torch.no_grad():
        m.weight.copy_(torch.from_numpy(g["f32_w"]))
    x = torch.from_numpy(g["f32_x"]).requires_grad_()
    y = m(x)
    y.backward(torch.from_numpy(g["f32_dy"]))
    np.testing.assert_allclose(y.detach().numpy(), g["f32_y"], rtol=1e-5, atol=1e-6)
    np.testing.assert_allclose(x.grad.numpy(), g["f32_dx"], rtol=1e-5, atol=1e-5)


def test_fused_entry_points_cpu_match_the_oracle():
    rng = np.random.default_rng(0)
    x, r = rng.standard_normal((2, 5, 16)).astype(np.float32), rng.standard_normal((2, 5, 16)).astype(np.float32)
    w = rng.standard_normal(16).astype(np.float32)
    out = fused_rmsnorm_residual(torch.from_numpy(x), torch.from_numpy(r), torch.from_numpy(w), 1e-6)
    ref, _ = onorm.rmsnorm_residual_fwd(x, r, w, 1e-6)
    np.testing.assert_allclose(out.numpy(), ref, rtol=1e-5, atol=1e-6)
    q = torch.randn(1, 2, 6, 8)
    cos, sin = RotaryEmbedding(8, 16)(6, torch.device("cpu"), torch.float32)
    np.testing.assert_allclose(fused_apply_rope(q, cos, sin).numpy(),
                               orope.rope_fwd(q.numpy(), cos.numpy(), sin.numpy()), rtol=1e-5, atol=1e-6)
    k = torch.randn(1, 2, 6, 8)
    qr, kr = apply_rotary_pos_emb(q, k, cos, sin)
    np.testing.assert_allclose(kr.numpy(), orope.rope_fwd(k.numpy(), cos.numpy(), sin.numpy()), rtol=1e-5,
                               atol=1e-6)
    logits = torch.randn(7, 6)
    probs, idx = fused_moe_routing(logits, 2)
    eg, ei = omoe.route(logits.numpy(), 2)[:2]
    assert np.array_equal(idx.numpy(), ei)
    np.testing.assert_allclose(probs.numpy(), eg, rtol=1e-5, atol=1e-6)
    with pytest.raises(ValueError):
        fused_moe_dispatch(logits, torch.randn(6, 4), 2, 1.25)


def test_moe_layer_cpu_matches_golden_layer():
    g = load_golden("moe_f32_drop")
    T, H = g["x"].shape
    _, F, E, k = (int(v) for v in g["cfg"])
    cf, lbw = (float(v) for v in g["cf_lbw"])
    layer = MoELayer(H, F, E, num_layers=2, top_k=k, capacity_factor=cf, load_balancing_weight=lbw)
    with torch.no_grad():
        layer.moe.gate.weight.copy_(torch.from_numpy(g["wg"]))
        for e, ex in enumerate(layer.moe.experts):
            ex.gate_up_proj.weight.copy_(torch.from_numpy(g["wgu"][e]))
            ex.down_proj.weight.copy_(torch.from_numpy(g["wd"][e]))
    out, aux = layer(torch.from_numpy(g["x"]).view(1, T, H))
    np.testing.assert_allclose(out.detach().numpy().reshape(T, H), g["out"], rtol=1e-5, atol=1e-6)
    assert aux.item() == pytest.approx(float(g["aux"][0]), rel=1e-5)
    assert sum(layer.last_expert_utilization.values()) == pytest.approx(1.0, abs=1e-5)


def test_int8_experts_construct_and_run_on_cpu():
    layer = MoELayer(16, 32, 2, num_layers=2, top_k=1, quantization="int8")
    ex = layer.moe.experts[0]
    assert isinstance(ex.down_proj, QuantizedLinear) and isinstance(ex.gate_up_proj, QuantizedLinear)
    assert set(ex.state_dict()) >= {"gate_up_proj.weight", "down_proj.weight"}
    out, aux = layer(torch.randn(2, 3, 16))
    assert out.shape == (2, 3, 16) and torch.isfinite(out).all()
    plain = MoELayer(16, 32, 2, num_layers=2, top_k=1)
    plain.load_state_dict({k: v for k, v in layer.state_dict().items() if "fake_quant" not in k})
    x = torch.randn(1, 4, 16)
    assert not torch.allclose(plain(x)[0], layer(x)[0], atol=1e-6)  # fake quantisation changes numerics


def test_ep_size_without_a_process_group_keeps_every_expert(monkeypatch):
    monkeypatch.delenv("WORLD_SIZE", raising=False)
    layer = MoELayer(16, 32, 4, num_layers=2, ep_size=4)
    assert len(layer.moe.experts) == 4 and layer.ep_size == 4


def _free_port():
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _ep_worker(rank, world, port, q):
    try:
        import torch.distributed as dist

        os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
        dist.init_process_group("gloo", rank=rank, world_size=world)
        layer = MoELayer(16, 32, 8, num_layers=2, ep_size=world)
        from ats_v2_b200.ep import ExpertParallelMoE

        assert isinstance(layer.moe, ExpertParallelMoE) and layer.moe.exchange == "device"
        assert len(layer.moe.experts) == 8 // world and layer.moe.gate.weight.shape == (8, 16)
        layer.moe._bind()
        assert layer.moe.rank == rank and layer.moe.world == world
        dist.destroy_process_group()
    except Exception as exc:  # reported to the parent
        q.put((rank, repr(exc)))
        raise


def test_ep_size_in_a_process_group_shards_the_experts():
    import torch.multiprocessing as mp

    ctx = mp.get_context("spawn")
    q = ctx.SimpleQueue()
    mp.start_processes(_ep_worker, args=(2, _free_port(), q), nprocs=2, join=True, start_method="spawn")
    assert q.empty()


def test_fused_add_rmsnorm_cpu_is_the_block_step():
    from ats_v2_b200.norm_fused import fused_add_rmsnorm

    x, r, w = torch.randn(3, 5, 16), torch.randn(3, 5, 16), 1 + 0.1 * torch.randn(16)
    h, s = fused_add_rmsnorm(x, r, w, 1e-6)
    assert torch.equal(s, r + x)
    assert torch.equal(h, torch.nn.functional.rms_norm(r + x, (16,), w, 1e-6))
    with pytest.raises(ValueError):
        fused_add_rmsnorm(x, r[:, :4], w)


def test_fused_qk_proj_rope_cpu_is_the_reference_attention_step():
    from ats_v2_b200.rope_fused import fused_qk_proj_rope

    x = torch.randn(2, 8, 32)
    wq, wk = torch.randn(2 * 16, 32), torch.randn(16, 32)
    cos, sin = RotaryEmbedding(16, 8)(8, torch.device("cpu"), torch.float32)
    q, k = fused_qk_proj_rope(x, wq, wk, cos, sin)
    rq = (x @ wq.t()).view(2, 8, 2, 16).transpose(1, 2)
    rk = (x @ wk.t()).view(2, 8, 1, 16).transpose(1, 2)
    eq, ek = apply_rotary_pos_emb(rq, rk, cos, sin)
    assert torch.equal(q, eq) and torch.equal(k, ek)

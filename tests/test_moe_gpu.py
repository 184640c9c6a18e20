"""MoE router, permutation and layer on the CUDA kernels vs the golden
vectors and the oracle.

Router indices and the permutation are required bit-exact.  Routing is
compared on the same float32 logits (the ones the GPU computed), since a
last-ulp difference between a CPU and a GPU matmul can legitimately flip a
near-tie.  Layer outputs and gradients: float32 experts within 1e-4 relative
(grouped GEMMs accumulate in a different order than numpy), bfloat16 within
2e-2 relative / 1e-2 absolute."""

from __future__ import annotations

import numpy as np
import pytest
import torch

from ats_v2_b200 import moe as bmoe
from ats_v2_b200.moe_fused import _cuda_moe_routing, fused_moe_dispatch, fused_moe_routing
from oracle import moe as omoe
from oracle.bf16 import round_bf16
from tests.conftest import load_golden
from tests.util import close, dev, np32, seeded_normal

pytestmark = pytest.mark.gpu

ROUTING_CASES = ["r5x4", "r32x8", "r64x8k1", "r64x16k4", "r512x64z", "r200x256k8"]


@pytest.mark.parametrize("case", ROUTING_CASES)
def test_routing_golden_bit_exact(case):
    g = load_golden("routing")
    k = int(g[case + "_k"][0])
    probs, idx = fused_moe_routing(dev(g[case + "_logits"]), k)
    assert idx.dtype == torch.int64 and probs.dtype == torch.float32
    assert np.array_equal(idx.cpu().numpy(), g[case + "_idx"])
    close(probs, g[case + "_probs"], "f32", rtol=1e-6, atol=1e-7)


def test_routing_reference_parity_test():
    """tests/test_triton.py:170-187 of the reference, on the CUDA kernel."""
    torch.manual_seed(0)
    gate_logits = torch.randn(32, 8, device="cuda")
    p, i = _cuda_moe_routing(gate_logits, top_k=2)
    ep, ei, _ = omoe.route(np32(gate_logits), 2)
    assert torch.equal(i.sort(dim=-1).values.cpu(), torch.from_numpy(ei).sort(dim=-1).values)
    assert torch.allclose(p.sort(dim=-1).values.cpu(), torch.from_numpy(ep).sort(dim=-1).values, atol=1e-5)


def test_routing_ties_take_lower_index():
    logits = torch.zeros(4, 8, device="cuda")
    logits[1, 5] = 1.0
    logits[2, 3] = logits[2, 6] = 2.0
    p, i = fused_moe_routing(logits, 3)
    assert i.tolist() == [[0, 1, 2], [5, 0, 1], [3, 6, 0], [0, 1, 2]]
    ep, ei, _ = omoe.route(np32(logits), 3)
    assert np.array_equal(i.cpu().numpy(), ei)
    close(p, ep, "f32", rtol=1e-6)


@pytest.mark.parametrize("T,E,k", [(1, 1, 1), (1000, 64, 2), (4097, 8, 2), (300, 33, 5), (64, 1024, 16)])
def test_routing_random_bit_exact(T, E, k):
    lg = seeded_normal((T, E), T + E + k, 2.0)
    p, i = fused_moe_dispatch(dev(lg), torch.empty(T, 4, device="cuda"), k, 1.25)
    ep, ei, _ = omoe.route(lg, k)
    assert np.array_equal(i.cpu().numpy(), ei)
    close(p, ep, "f32", rtol=1e-6, atol=1e-7)


def _layer_from(g, dtype):
    H, F, E, k = (int(v) for v in g["cfg"])
    cf, lbw = (float(v) for v in g["cf_lbw"])
    layer = bmoe.MoELayer(H, F, E, num_layers=2, top_k=k, capacity_factor=cf, load_balancing_weight=lbw).cuda()
    with torch.no_grad():
        layer.moe.gate.weight.copy_(dev(g["wg"]))
        for e, ex in enumerate(layer.moe.experts):
            ex.gate_up_proj.weight.data = dev(g["wgu"][e], dtype)
            ex.down_proj.weight.data = dev(g["wd"][e], dtype)
    return layer, (H, F, E, k, cf, lbw)


@pytest.mark.parametrize("case,dn", [("moe_f32_drop", "f32"), ("moe_f32_nodrop", "f32"),
                                     ("moe_bf16", "bf16"), ("moe_bf16_drop", "bf16")])
def test_layer_golden(case, dn):
    g = load_golden(case)
    dtype = torch.float32 if dn == "f32" else torch.bfloat16
    layer, (H, F, E, k, cf, lbw) = _layer_from(g, dtype)
    T = g["x"].shape[0]
    x = dev(g["x"], dtype).view(1, T, H).requires_grad_()
    out, aux = layer(x)
    assert out.shape == (1, T, H) and out.dtype == dtype and aux.dim() == 0
    # routing on the GPU's own logits must equal the oracle's on those logits
    logits = layer.moe.router_logits(x.detach().view(T, H))
    _, gidx = fused_moe_routing(logits, k)
    _, oidx, _ = omoe.route(np32(logits), k)
    assert np.array_equal(gidx.cpu().numpy(), oidx)
    tol = dict(rtol=1e-4, atol=1e-6) if dn == "f32" else {}
    close(out.view(T, H), g["out"], dn, **tol)
    assert aux.item() == pytest.approx(float(g["aux"][0]), rel=1e-5)
    util = layer.last_expert_utilization
    assert np.allclose([util[i] for i in range(E)], g["util"], rtol=1e-6, atol=1e-7)
    assert sum(util.values()) == pytest.approx(1.0, abs=1e-5)
    (out.float() * dev(g["g"]).view(1, T, H)).sum().add(aux).backward()
    gtol = dict(rtol=1e-4, atol=1e-6) if dn == "f32" else {}
    close(x.grad.view(T, H), g["dx"], dn, **gtol)
    scale = float(np.abs(g["dwg"]).max())
    r = 1e-3 if dn == "f32" else 2e-2
    close(layer.moe.gate.weight.grad, g["dwg"], "f32", rtol=r, atol=r * scale)
    for e, ex in enumerate(layer.moe.experts):
        for got, ref in ((ex.gate_up_proj.weight.grad, g["dwgu"][e]), (ex.down_proj.weight.grad, g["dwd"][e])):
            wt = dict(rtol=1e-4, atol=1e-4 * float(np.abs(ref).max())) if dn == "f32" else {}
            close(got, ref, dn, **wt)


def _oracle_layer_check(T, H, F, E, k, cf, lbw, dn, seed, sample_tokens=None):
    dtype = torch.float32 if dn == "f32" else torch.bfloat16
    torch.manual_seed(seed)
    layer = bmoe.MoELayer(H, F, E, num_layers=2, top_k=k, capacity_factor=cf, load_balancing_weight=lbw)
    with torch.no_grad():
        layer.moe.gate.weight.normal_(0, 0.02)
        for ex in layer.moe.experts:
            ex.gate_up_proj.weight.normal_(0, 0.02)
            ex.down_proj.weight.normal_(0, 0.02)
    layer = layer.cuda().to(dtype)
    layer.moe.gate.float()
    x = torch.randn(1, T, H, device="cuda").to(dtype).requires_grad_()
    out, aux = layer(x)
    gout = torch.randn(1, T, H, device="cuda").to(dtype)
    (out.float() * gout.float()).sum().add(aux).backward()
    xs, logits = np32(x.view(T, H)), np32(layer.moe.router_logits(x.detach().view(T, H)))
    wgu = np.stack([np32(ex.gate_up_proj.weight) for ex in layer.moe.experts])
    wd = np.stack([np32(ex.down_proj.weight) for ex in layer.moe.experts])
    fwd = omoe.moe_forward(xs, logits, wgu, wd, k, cf, lbw, dn)
    tol = dict(rtol=1e-4, atol=1e-6) if dn == "f32" else {}
    close(out.view(T, H), fwd["out"], dn, **tol)
    assert aux.item() == pytest.approx(fwd["aux"], rel=1e-5)
    b = omoe.moe_layer_backward_full(np32(gout.view(T, H)), fwd, xs, np32(layer.moe.gate.weight), wgu, wd,
                                     lbw, dn)
    close(x.grad.view(T, H), b["dx"], dn, **tol)
    # the router-weight gradient sums T products of d(logits) that inherit the
    # experts' rounding; its error is judged against the tensor's own scale
    scale = float(np.abs(b["dwg"]).max())
    r = 1e-3 if dn == "f32" else 2e-2
    close(layer.moe.gate.weight.grad, b["dwg"], "f32", rtol=r, atol=r * scale)
    # weight gradients sum hundreds of products: float32 results are judged
    # against each tensor's scale (1e-4 of its largest magnitude)
    for e, ex in enumerate(layer.moe.experts):
        for got, ref in ((ex.gate_up_proj.weight.grad, b["dwgu"][e]), (ex.down_proj.weight.grad, b["dwd"][e])):
            wt = dict(rtol=1e-4, atol=1e-4 * float(np.abs(ref).max())) if dn == "f32" else {}
            close(got, ref, dn, **wt)
    return fwd


def test_cpu_parity_workload_moe_f32():
    """The CPU parity workload's MoE: 1024 tokens, hidden 512, ffn 1024, 4 experts top-2, cf 1.25."""
    _oracle_layer_check(1024, 512, 1024, 4, 2, 1.25, 0.01, "f32", 0)


@pytest.mark.parametrize("T,H,F,E,k,cf", [(512, 256, 512, 8, 2, 4.0), (700, 128, 192, 16, 3, 0.5),
                                          (1, 64, 64, 4, 2, 1.25), (300, 64, 128, 1, 1, 1.0)])
def test_layer_bf16_vs_oracle(T, H, F, E, k, cf):
    _oracle_layer_check(T, H, F, E, k, cf, 0.01, "bf16", T + E)


def test_permutation_is_stable_and_capacity_bounded():
    """Per expert: ascending token order, first `capacity` kept (moe.py:109-116)."""
    T, E, k, cf = 2000, 8, 2, 0.6
    lg = seeded_normal((T, E), 3, 1.5)
    lg[:, 2] += 1.0  # make expert 2 overflow its capacity
    C = bmoe.capacity_for(T, k, E, cf)
    layer = bmoe.MoELayer(32, 32, E, 2, top_k=k, capacity_factor=cf).cuda()
    x = torch.randn(T, 32, device="cuda")
    wgu, wd = layer.moe._weights()
    out, aux, util, counts, idx = bmoe.moe_apply(x, dev(lg), wgu, wd, k, C, 0.01)
    _, oidx, _ = omoe.route(lg, k)
    kept, ocounts = omoe.permutation(oidx, E, C)
    assert np.array_equal(idx.cpu().numpy(), oidx)
    assert np.array_equal(counts.cpu().numpy(), ocounts)
    assert ocounts[2] > C
    # a dropped (token, expert) pair contributes nothing: token rows recomputed from kept lists
    ws_tokens = set()
    for e in range(E):
        ws_tokens |= set(kept[e].tolist())
    dropped_everywhere = [t for t in range(T) if t not in ws_tokens]
    if dropped_everywhere:
        assert torch.count_nonzero(out[dropped_everywhere]) == 0


def test_full_size_single_gpu_config_sampled_tokens():
    """tokens 8192, hidden 2048, 8 experts top-2, ffn 5632, no drop (cf = E/k).

    Nothing is dropped, so every token's output and input gradient depend on
    that token alone (the aux loss is left out of the backward): 32 sampled
    tokens are checked against the oracle run on them.  The weight gradients of
    one expert sum over all of its ~2048 rows: the oracle recomputes that
    expert on exactly those rows, with float64 sums for the two weight
    gradients, and both must match at the bf16 tolerance."""
    T, H, F, E, k = 8192, 2048, 5632, 8, 2
    torch.manual_seed(0)
    layer = bmoe.MoELayer(H, F, E, num_layers=2, top_k=k, capacity_factor=E / k).cuda()
    with torch.no_grad():
        layer.moe.gate.weight.normal_(0, 0.02)
        for ex in layer.moe.experts:
            ex.gate_up_proj.weight.normal_(0, 0.02)
            ex.down_proj.weight.normal_(0, 0.02)
    layer.moe.experts.to(torch.bfloat16)
    x = torch.randn(1, T, H, device="cuda").bfloat16().requires_grad_()
    gout = torch.randn(1, T, H, device="cuda").bfloat16()
    out, aux = layer(x)
    out.backward(gout)
    logits = layer.moe.router_logits(x.detach().view(T, H))
    gates, idx = fused_moe_routing(logits, k)
    wg = np32(layer.moe.gate.weight)
    wgu = np.stack([np32(ex.gate_up_proj.weight) for ex in layer.moe.experts])
    wd = np.stack([np32(ex.down_proj.weight) for ex in layer.moe.experts])
    xs_all, gs_all, lg_all = np32(x.view(T, H)), np32(gout.view(T, H)), np32(logits)
    # sampled tokens: output and input gradient (router share included), no aux loss
    toks = torch.randint(0, T, (32,), generator=torch.Generator().manual_seed(3)).tolist()
    fwd = omoe.moe_forward(xs_all[toks], lg_all[toks], wgu, wd, k, E / k, 0.0, "bf16")
    assert fwd["cap"] >= len(toks)  # nothing dropped in the sample either
    close(out.view(T, H)[toks], fwd["out"], "bf16")
    b = omoe.moe_layer_backward_full(gs_all[toks], fwd, xs_all[toks], wg, wgu, wd, 0.0, "bf16")
    close(x.grad.view(T, H)[toks], b["dx"], "bf16")
    # one expert's weight gradients over all of its rows
    e = 3
    ids, gts = idx.cpu().numpy(), np32(gates)
    rows = np.nonzero((ids == e).any(axis=1))[0]
    assert rows.size > 1000
    wgt = np.array([gts[t][list(ids[t]).index(e)] for t in rows], np.float32)
    y, g, u, s_, a = omoe.expert_fwd(xs_all[rows], wgu[e], wd[e], "bf16")
    dy = round_bf16(gs_all[rows] * wgt[:, None])
    _, dwgu_e, dwd_e = omoe.expert_bwd(dy, xs_all[rows], wgu[e], wd[e], g, u, s_, a, "bf16", acc=np.float64)
    # each summand (dy*a, dh*x) is a product of bf16 values that the two sides may round a half ulp apart (the
    # kernel's SwiGLU derivative uses the SFU exponential): over ~2048 rows those differences add up to a
    # fixed fraction of the gradient's typical size, whatever the element's own size -- hence the bf16
    # tolerance applied to the tensor's scale (2e-2 of its rms) beside the 2e-2 relative bound
    for got, ref in ((layer.moe.experts[e].down_proj.weight.grad, dwd_e),
                     (layer.moe.experts[e].gate_up_proj.weight.grad, dwgu_e)):
        close(got, ref, "bf16", atol=2e-2 * float(np.sqrt(np.mean(np.square(ref, dtype=np.float64)))))
    for ex in layer.moe.experts:
        assert torch.isfinite(ex.gate_up_proj.weight.grad.float()).all()
        assert torch.isfinite(ex.down_proj.weight.grad.float()).all()
"""Expert-parallel MoE on the GPU.

Single rank: the expert-parallel layer, with either exchange (packed rows or
capacity slots), must equal the single-GPU layer for the same weights (the
rows of a segment are the same and in the same order; only their place in the
buffer differs).  Two ranks (runs when two GPUs are visible): every rank's output
and input gradient equal the oracle run on that rank's own tokens with all
experts' weights, and every local expert's weight gradient equals the sum
over both ranks' tokens -- DeepSpeed's local-capacity semantics.  The
exchange in overlapped parts (with the GEMMs held to fewer SMs), the
peer-memory exchange (copy-engine copies into IPC-mapped peer buffers) and the
device-driven exchange (kernels that store rows into, and load them from, the
IPC-mapped buffers, with the split sizes never on the host) must give
bit-equal results to the NCCL exchange in one piece."""

from __future__ import annotations

import os
import socket
import traceback
from datetime import timedelta

import numpy as np
import pytest
import torch

from ats_v2_b200 import moe as bmoe
from ats_v2_b200.ep import ExpertParallelMoE
from tests.util import close, np32

pytestmark = pytest.mark.gpu


def _init_weights(mod_gate, experts, seed):
    g = torch.Generator().manual_seed(seed)
    with torch.no_grad():
        mod_gate.weight.copy_(0.02 * torch.randn(mod_gate.weight.shape, generator=g))
        for ex in experts:
            ex.gate_up_proj.weight.copy_(0.02 * torch.randn(ex.gate_up_proj.weight.shape, generator=g))
            ex.down_proj.weight.copy_(0.02 * torch.randn(ex.down_proj.weight.shape, generator=g))


@pytest.mark.parametrize("exchange", ["packed", "slots", "peer", "device"])
@pytest.mark.parametrize("T,H,F,E,k,cf", [(1024, 256, 384, 8, 2, 1.25), (700, 128, 128, 4, 2, 0.6)])
def test_single_rank_expert_parallel_layer_equals_the_layer(T, H, F, E, k, cf, exchange):
    torch.manual_seed(0)
    ep = ExpertParallelMoE(H, F, E, num_layers=2, top_k=k, capacity_factor=cf, exchange=exchange)
    ref = bmoe.MoELayer(H, F, E, num_layers=2, top_k=k, capacity_factor=cf)
    _init_weights(ep.gate, ep.experts, 1)
    _init_weights(ref.moe.gate, ref.moe.experts, 1)
    ep, ref = ep.cuda(), ref.cuda()
    ep.experts.to(torch.bfloat16)
    ref.moe.experts.to(torch.bfloat16)
    x = torch.randn(1, T, H, device="cuda").bfloat16()
    g = torch.randn(1, T, H, device="cuda").bfloat16()
    xa, xb = x.clone().requires_grad_(), x.clone().requires_grad_()
    oa, aa = ep(xa)
    ob, ab = ref(xb)
    torch.autograd.backward([oa, aa], [g, torch.ones_like(aa)])
    torch.autograd.backward([ob, ab], [g, torch.ones_like(ab)])
    close(oa, np32(ob), "bf16", min_exact=0.999)
    assert aa.item() == pytest.approx(ab.item(), rel=1e-6)
    close(xa.grad, np32(xb.grad), "bf16", min_exact=0.999)
    close(ep.gate.weight.grad, np32(ref.moe.gate.weight.grad), "f32", rtol=1e-5, atol=1e-7)
    for e in range(E):
        close(ep.experts[e].gate_up_proj.weight.grad, np32(ref.moe.experts[e].gate_up_proj.weight.grad), "bf16",
              min_exact=0.999)
        close(ep.experts[e].down_proj.weight.grad, np32(ref.moe.experts[e].down_proj.weight.grad), "bf16",
              min_exact=0.999)


def test_rebalanced_layer_computes_the_same_function():
    """Relabelling the experts (rebalance) moves gate rows and weights with
    them.  With top-2 routing the output is bit-equal and every expert's
    weight gradient is the old one under the permutation.  The router reduces
    over the experts in label order (the softmax sums, its backward, and the
    K dimension of the router's share of the input gradient), so the input
    gradient matches at bf16 tolerance with almost every element bit-equal
    and the gate gradient at float32 tolerance."""
    T, H, F, E, k = 1024, 256, 384, 8, 2
    torch.manual_seed(0)
    ep = ExpertParallelMoE(H, F, E, num_layers=2, top_k=k, capacity_factor=1.25)
    _init_weights(ep.gate, ep.experts, 3)
    ep = ep.cuda()
    ep.experts.to(torch.bfloat16)
    bias = torch.linspace(-1.0, 1.0, E, device="cuda")
    x = torch.randn(1, T, H, device="cuda").bfloat16()
    g = torch.randn(1, T, H, device="cuda").bfloat16()

    def run(b):
        xa = x.clone().requires_grad_()
        for p in ep.parameters():
            p.grad = None
        out, aux = ep(xa, logit_bias=b)
        torch.autograd.backward([out, aux], [g, torch.ones_like(aux)])
        return (out.detach(), xa.grad, aux.detach(), ep.gate.weight.grad.clone(),
                [e.gate_up_proj.weight.grad.clone() for e in ep.experts],
                [e.down_proj.weight.grad.clone() for e in ep.experts])

    before = run(bias)
    perm = ep.rebalance(perm=torch.randperm(E, generator=torch.Generator().manual_seed(4)))
    assert sorted(perm.tolist()) == list(range(E)) and perm.tolist() != list(range(E))
    after = run(bias[perm.cuda()])
    assert torch.equal(before[0], after[0])
    close(after[1], np32(before[1]), "bf16", min_exact=0.99)
    assert after[2].item() == pytest.approx(before[2].item(), rel=1e-6)
    # the router's softmax and its backward reduce over the experts in label order (float32)
    ref = before[3][perm.cuda()]
    torch.testing.assert_close(after[3], ref, rtol=1e-5, atol=1e-5 * float(ref.abs().max()))
    for j in range(E):
        assert torch.equal(after[4][j], before[4][perm[j]])
        assert torch.equal(after[5][j], before[5][perm[j]])


def _free_port() -> int:
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _two_rank_worker(rank, world, port, errq, exchange, parts):
    from oracle import moe as omoe
    try:
        os.environ["MASTER_ADDR"] = "127.0.0.1"
        os.environ["MASTER_PORT"] = str(port)
        os.environ.setdefault("NCCL_NVLS_ENABLE", "0")
        torch.cuda.set_device(rank)
        torch.distributed.init_process_group("nccl", rank=rank, world_size=world, timeout=timedelta(seconds=60),
                                             device_id=torch.device("cuda", rank))
        T, H, F, E, k, cf = 512, 128, 256, 8, 2, 1.25
        El = E // world
        full_gate = torch.nn.Linear(H, E, bias=False)
        full_experts = torch.nn.ModuleList([bmoe.SwiGLU(H, F) for _ in range(E)])
        _init_weights(full_gate, full_experts, 5)  # identical on both ranks
        def layer(p, mode=exchange):
            m = ExpertParallelMoE(H, F, E, num_layers=2, top_k=k, capacity_factor=cf, exchange=mode,
                                  overlap_parts=p, comm_sms=20)
            with torch.no_grad():
                m.gate.weight.copy_(full_gate.weight)
                for i in range(El):
                    m.experts[i].gate_up_proj.weight.copy_(full_experts[rank * El + i].gate_up_proj.weight)
                    m.experts[i].down_proj.weight.copy_(full_experts[rank * El + i].down_proj.weight)
            m = m.cuda()
            m.experts.to(torch.bfloat16)
            return m

        ep = layer(parts)
        gx = torch.Generator(device="cuda").manual_seed(100 + rank)
        x = torch.randn(1, T, H, device="cuda", generator=gx).bfloat16().requires_grad_()
        gout = torch.randn(1, T, H, device="cuda", generator=gx).bfloat16()
        out, aux = ep(x)
        torch.autograd.backward([out, aux], [gout, torch.ones_like(aux)])
        torch.cuda.synchronize()
        if parts > 1 or exchange in ("peer", "device"):
            # the overlapped and the peer-memory exchanges move the same rows to the same GEMMs:
            # bit-equal to the NCCL exchange in one piece
            one = layer(1, "packed" if exchange in ("peer", "device") else exchange)
            x1 = x.detach().clone().requires_grad_()
            out1, aux1 = one(x1)
            torch.autograd.backward([out1, aux1], [gout, torch.ones_like(aux1)])
            torch.cuda.synchronize()
            assert torch.equal(out, out1) and torch.equal(aux, aux1) and torch.equal(x.grad, x1.grad)
            for i in range(El):
                assert torch.equal(ep.experts[i].gate_up_proj.weight.grad, one.experts[i].gate_up_proj.weight.grad)
                assert torch.equal(ep.experts[i].down_proj.weight.grad, one.experts[i].down_proj.weight.grad)
            assert torch.equal(ep.gate.weight.grad, one.gate.weight.grad)
        if exchange in ("peer", "device"):
            # buffer sets are reused: a forward without backward, then a second step, give the same bits
            with torch.no_grad():
                out_ng, _ = ep(x.detach())
            assert torch.equal(out_ng, out.detach())
            first = (out.detach().clone(), x.grad.clone(), ep.experts[0].down_proj.weight.grad.clone())
            for prm in ep.parameters():
                prm.grad = None
            x2 = x.detach().clone().requires_grad_()
            out2, aux2 = ep(x2)
            torch.autograd.backward([out2, aux2], [gout, torch.ones_like(aux2)])
            torch.cuda.synchronize()
            assert torch.equal(out2, first[0]) and torch.equal(x2.grad, first[1])
            assert torch.equal(ep.experts[0].down_proj.weight.grad, first[2])
            assert len(ep._peer.sets) == 1 and not ep._peer.sets[0].busy
            ep.release_peer_buffers()
            assert not ep._peer.sets
        # oracle on this rank's tokens with all experts' (bf16) weights
        xs = np32(x.view(T, H))
        logits = np32(ep.router_logits(x.detach().view(T, H)))
        wgu = np.stack([np32(e.gate_up_proj.weight.bfloat16()) for e in full_experts])
        wd = np.stack([np32(e.down_proj.weight.bfloat16()) for e in full_experts])
        fwd = omoe.moe_forward(xs, logits, wgu, wd, k, cf, 0.01, "bf16")
        close(out.view(T, H), fwd["out"], "bf16")
        b = omoe.moe_layer_backward_full(np32(gout.view(T, H)), fwd, xs, np32(ep.gate.weight), wgu, wd, 0.01,
                                         "bf16")
        close(x.grad.view(T, H), b["dx"], "bf16")
        # expert weight gradients: sum of both ranks' contributions
        dwgu = torch.from_numpy(b["dwgu"]).cuda()
        dwd = torch.from_numpy(b["dwd"]).cuda()
        torch.distributed.all_reduce(dwgu)
        torch.distributed.all_reduce(dwd)
        for i in range(El):
            e = rank * El + i
            close(ep.experts[i].gate_up_proj.weight.grad, np32(dwgu[e]), "bf16", atol=2e-2)
            close(ep.experts[i].down_proj.weight.grad, np32(dwd[e]), "bf16", atol=2e-2)
        torch.distributed.barrier()
        torch.distributed.destroy_process_group()
    except Exception:
        errq.put((rank, traceback.format_exc()))
        raise


@pytest.mark.skipif(torch.cuda.device_count() < 2, reason="needs two GPUs")
@pytest.mark.parametrize("exchange,parts", [("packed", 1), ("slots", 1), ("packed", 2), ("slots", 4), ("peer", 1),
                                            ("peer", 2), ("device", 1), ("device", 2)])
def test_two_ranks_match_the_oracle_on_local_tokens(exchange, parts):
    import torch.multiprocessing as mp
    ctx = mp.get_context("spawn")
    errq = ctx.SimpleQueue()
    mp.start_processes(_two_rank_worker, args=(2, _free_port(), errq, exchange, parts), nprocs=2, join=True,
                       start_method="spawn")
    assert errq.empty()

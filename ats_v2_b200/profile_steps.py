"""Run a few forward+backward steps of one hot-path layer, for a profiler to capture.

    python -m ats_v2_b200.profile_steps moe      [--steps 3]   # MoE layer: 8192 tokens, hidden 2048, 8 experts
    python -m ats_v2_b200.profile_steps moe_ep16k [--steps 3]  # expert-parallel layer at one GPU, reduced
    python -m ats_v2_b200.profile_steps ffn      [--steps 3]   # dense SwiGLU FFN: 16384 tokens, 4096 x 11008

Each step runs the layer's forward and backward on seeded synthetic inputs; nothing is timed.  The shapes are
the benchmark's, except ``moe_ep16k``: 16384 tokens, hidden 4096, 32 experts top-2, ffn 1408, capacity factor
1.25 and the Zipf(1.1) router-logit bias -- the same capacity (1280) and about the same rows per expert as
the benchmark's 32768 tokens and 64 experts, in few enough GB that a full counter capture stays small.
"""

from __future__ import annotations

import argparse

import torch


def _zipf_bias(E: int) -> torch.Tensor:
    p = torch.arange(1, E + 1, dtype=torch.float64) ** -1.1
    b = torch.log((p / p.sum())[torch.randperm(E, generator=torch.Generator().manual_seed(1))])
    return (b - b.mean()).float()


def _moe():
    from ats_v2_b200.moe import MoELayer

    T, H, F, E = 8192, 2048, 5632, 8
    layer = MoELayer(H, F, E, num_layers=2, top_k=2, capacity_factor=E / 2).cuda()
    with torch.no_grad():
        for ex in layer.moe.experts:
            ex.gate_up_proj.weight.normal_(0, 0.02)
            ex.down_proj.weight.normal_(0, 0.02)
    layer.moe.experts.to(torch.bfloat16)
    x = torch.randn(1, T, H, device="cuda").bfloat16().requires_grad_()
    dy = torch.randn(1, T, H, device="cuda").bfloat16()

    def step():
        out, aux = layer(x)
        torch.autograd.backward([out, aux], [dy, torch.ones_like(aux)])

    return step


def _moe_ep16k():
    from ats_v2_b200.ep import ExpertParallelMoE

    T, H, F, E = 16384, 4096, 1408, 32
    with torch.device("cuda"):
        layer = ExpertParallelMoE(H, F, E, num_layers=2, top_k=2, capacity_factor=1.25)
    with torch.no_grad():
        layer.gate.weight.normal_(0, 0.02)
        for ex in layer.experts:
            ex.gate_up_proj.weight.normal_(0, 0.02)
            ex.down_proj.weight.normal_(0, 0.02)
    layer.experts.to(torch.bfloat16)
    bias = _zipf_bias(E).cuda()
    x = torch.randn(1, T, H, device="cuda").bfloat16().requires_grad_()
    dy = torch.randn(1, T, H, device="cuda").bfloat16()

    def step():
        out, aux = layer(x, logit_bias=bias)
        torch.autograd.backward([out, aux], [dy, torch.ones_like(aux)])

    return step


def _ffn():
    from ats_v2_b200.ffn import SwiGLU

    T, H, F = 16384, 4096, 11008
    with torch.device("cuda"):
        m = SwiGLU(H, F)
    with torch.no_grad():
        m.gate_up_proj.weight.normal_(0, 0.02)
        m.down_proj.weight.normal_(0, 0.02)
    m.bfloat16()
    x = torch.randn(T, H, device="cuda").bfloat16().requires_grad_()
    dy = torch.randn(T, H, device="cuda").bfloat16()

    def step():
        m(x).backward(dy)

    return step


LAYERS = {"moe": _moe, "moe_ep16k": _moe_ep16k, "ffn": _ffn}


def main() -> None:
    ap = argparse.ArgumentParser(description=__doc__.splitlines()[0])
    ap.add_argument("layer", choices=sorted(LAYERS))
    ap.add_argument("--steps", type=int, default=3)
    a = ap.parse_args()
    torch.manual_seed(0)
    step = LAYERS[a.layer]()
    for _ in range(a.steps):
        step()
    torch.cuda.synchronize()
    print(f"{a.layer}: {a.steps} steps")


if __name__ == "__main__":
    main()

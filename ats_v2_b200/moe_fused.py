"""Fused MoE routing on the sm_100a router kernel -- mirror of
ats/model/moe_triton.py.

``fused_moe_routing(gate_logits, top_k)`` and ``fused_moe_dispatch(gate_logits,
hidden_states, top_k, capacity_factor)`` keep the reference signatures and
ValueErrors (moe_triton.py:130-170) and return ``(top_k_probs float32,
top_k_idx int64)``: float32 softmax over experts, top-k in descending order
(exact ties go to the lower expert index), probabilities renormalised to sum
to one -- the math of _pytorch_moe_routing (moe_triton.py:121-127) -- in one
warp-per-token kernel (``ats_moe_topk``).  Logits of any float dtype are
routed in float32.  top_k may be up to 16 (the reference Triton kernel
stopped at 8).  ``_cuda_moe_routing`` is the kernel call without validation.

As in the reference module, ``HAS_TRITON`` says whether the fused GPU kernel
is available (here: whether the CUDA library is built; no Triton is
involved), ``_triton_moe_routing`` is the fused kernel call and
``_pytorch_moe_routing`` the plain torch formula the reference's tests compare
it against (tests/test_triton.py:170-187).  ``fused_moe_routing`` runs that
formula for CPU tensors, as the reference does (moe_triton.py:144-146); CUDA
tensors always take the kernel.
"""

from __future__ import annotations

import torch

from ats_v2_b200 import _lib

HAS_TRITON = _lib.LIB_PATH.exists()  # the reference's flag name: fused GPU kernel available
MAX_TOP_K = 16
MAX_EXPERTS = 1024


def _topk(logits: torch.Tensor, top_k: int, want_probs: bool = False):
    T, E = logits.shape
    if top_k > min(E, MAX_TOP_K) or E > MAX_EXPERTS:
        raise ValueError(f"router kernel supports top_k <= min(num_experts, {MAX_TOP_K}) and "
                         f"num_experts <= {MAX_EXPERTS}; got top_k={top_k}, num_experts={E}")
    lg = logits.float().contiguous()
    gates = torch.empty((T, top_k), dtype=torch.float32, device=lg.device)
    idx = torch.empty((T, top_k), dtype=torch.int64, device=lg.device)
    probs = torch.empty((T, E), dtype=torch.float32, device=lg.device) if want_probs else None
    _lib.call("ats_moe_topk", lg.data_ptr(), T, E, top_k, gates.data_ptr(), idx.data_ptr(), _lib.ptr(probs),
              _lib.stream_of(lg))
    return (gates, idx, probs) if want_probs else (gates, idx)


def _cuda_moe_routing(gate_logits: torch.Tensor, top_k: int):
    _lib.require_cuda("fused_moe_routing", gate_logits)
    return _topk(gate_logits, top_k)


# fused-kernel name of the reference module (tests/test_triton.py:170-187)
_triton_moe_routing = _cuda_moe_routing


def _pytorch_moe_routing(gate_logits: torch.Tensor, top_k: int):
    """The torch formula of moe_triton.py:121-127, the comparison of the reference's kernel test."""
    probs = torch.softmax(gate_logits, dim=-1)
    vals, idx = torch.topk(probs, top_k, dim=-1)
    return vals / vals.sum(dim=-1, keepdim=True), idx


def fused_moe_routing(gate_logits: torch.Tensor, top_k: int):
    """(top_k_probs, top_k_idx) for gate_logits [num_tokens, num_experts]."""
    if gate_logits.dim() != 2:
        raise ValueError(
            f"fused_moe_routing expected gate_logits of shape [num_tokens, num_experts], "
            f"got {tuple(gate_logits.shape)}."
        )
    if top_k < 1:
        raise ValueError(f"fused_moe_routing requires top_k >= 1, got {top_k}.")
    if _lib.on_cpu("fused_moe_routing", gate_logits):
        return _pytorch_moe_routing(gate_logits, top_k)
    return _cuda_moe_routing(gate_logits, top_k)


def fused_moe_dispatch(gate_logits: torch.Tensor, hidden_states: torch.Tensor, top_k: int,
                       capacity_factor: float):
    """Validation of moe_triton.py:149-170 followed by fused_moe_routing."""
    if hidden_states.shape[0] != gate_logits.shape[0]:
        raise ValueError(
            f"fused_moe_dispatch: hidden_states has {hidden_states.shape[0]} tokens but "
            f"gate_logits has {gate_logits.shape[0]}; they must match."
        )
    if capacity_factor <= 0:
        raise ValueError(f"fused_moe_dispatch requires capacity_factor > 0, got {capacity_factor}.")
    return fused_moe_routing(gate_logits, top_k)

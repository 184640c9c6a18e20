"""SwiGLU expert module -- mirror of ats/model/ffn.py:13-45.

Keeps the reference's parameter names and shapes (``gate_up_proj`` [2F, H],
``down_proj`` [H, F], no bias) so state dicts interchange.  Inside the MoE
layer the experts never run one by one: their weights are kept as views of
one stacked [E, ...] tensor and the grouped kernels read them from there.
A standalone ``SwiGLU.forward`` on CUDA tensors runs the same grouped kernels
as one expert over the token rows; CPU tensors take the reference's formula
``down(silu(gate) * up)`` through the two Linear modules (ffn.py:37-45).

The projections come from ``SwiGLU.linear_factory(in, out, quantization,
bias)``, by default this package's ``make_linear`` (a plain ``nn.Linear``,
or an int8 fake-quantised ``QuantizedLinear``).  A host framework with its
own factory (the reference's ``ats.model.quantization.make_linear``) installs
it on the class, so its quantized experts are its own Linear type.
Quantized projections run their own forward on CPU tensors; the CUDA kernels
take plain bf16/fp32 weights only, and refuse quantized ones.
"""

from __future__ import annotations

import torch
import torch.nn.functional as F
from torch import nn

from ats_v2_b200 import _lib
from ats_v2_b200.quantization import make_linear


class SwiGLU(nn.Module):
    linear_factory = staticmethod(make_linear)

    def __init__(self, hidden_size: int, intermediate_size: int, dropout: float = 0.0,
                 quantization: str = "none") -> None:
        super().__init__()
        if hidden_size <= 0 or intermediate_size <= 0:
            raise ValueError(
                f"SwiGLU requires positive hidden_size and intermediate_size, got "
                f"hidden_size={hidden_size}, intermediate_size={intermediate_size}."
            )
        self.hidden_size = hidden_size
        self.intermediate_size = intermediate_size
        self.quantization = quantization
        self.gate_up_proj = self.linear_factory(hidden_size, 2 * intermediate_size, quantization, bias=False)
        self.down_proj = self.linear_factory(intermediate_size, hidden_size, quantization, bias=False)
        self.dropout = nn.Dropout(dropout)

    def forward(self, x: torch.Tensor) -> torch.Tensor:
        if x.shape[-1] != self.hidden_size:
            raise ValueError(f"SwiGLU expected last dimension {self.hidden_size}, got {x.shape[-1]}.")
        if _lib.on_cpu("SwiGLU", x, self.gate_up_proj.weight, self.down_proj.weight):
            gate, up = self.gate_up_proj(x).chunk(2, dim=-1)
            return self.dropout(self.down_proj(F.silu(gate) * up))
        require_plain_weights(self.quantization, "SwiGLU")
        from ats_v2_b200.moe import dense_swiglu

        return self.dropout(dense_swiglu(x, self.gate_up_proj.weight, self.down_proj.weight))


def require_plain_weights(quantization: str, name: str) -> None:
    """The CUDA kernels multiply the stored bf16/fp32 weights; quantization-aware
    projections (fake-quantised weights and activations) are not built there."""
    if quantization != "none":
        raise NotImplementedError(
            f"{name}: quantization={quantization!r} experts construct and run on CPU tensors, but the "
            f"sm_100a kernels take plain bf16/float32 weights only. Fix: set model.quantization: none "
            f"for CUDA training with ats_v2_b200.")

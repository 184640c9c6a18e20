"""SwiGLU expert module -- mirror of ats/model/ffn.py:13-45.

Keeps the reference's parameter names and shapes (``gate_up_proj`` [2F, H],
``down_proj`` [H, F], no bias) so state dicts interchange.  Inside the MoE
layer the experts never run one by one: their weights are kept as views of
one stacked [E, ...] tensor and the grouped kernels read them from there.
A standalone ``SwiGLU.forward`` runs the same grouped kernels with a single
expert that every token selects with gate 1.0 (the combine then returns the
expert output unchanged).
"""

from __future__ import annotations

import torch
from torch import nn


class SwiGLU(nn.Module):
    def __init__(self, hidden_size: int, intermediate_size: int, dropout: float = 0.0,
                 quantization: str = "none") -> None:
        super().__init__()
        if hidden_size <= 0 or intermediate_size <= 0:
            raise ValueError(
                f"SwiGLU requires positive hidden_size and intermediate_size, got "
                f"hidden_size={hidden_size}, intermediate_size={intermediate_size}."
            )
        if quantization != "none":
            raise NotImplementedError(
                f"ats_v2_b200 SwiGLU runs bf16/fp32 experts only; quantization={quantization!r} is not built")
        self.hidden_size = hidden_size
        self.intermediate_size = intermediate_size
        self.gate_up_proj = nn.Linear(hidden_size, 2 * intermediate_size, bias=False)
        self.down_proj = nn.Linear(intermediate_size, hidden_size, bias=False)
        self.dropout = nn.Dropout(dropout)

    def forward(self, x: torch.Tensor) -> torch.Tensor:
        if x.shape[-1] != self.hidden_size:
            raise ValueError(f"SwiGLU expected last dimension {self.hidden_size}, got {x.shape[-1]}.")
        from ats_v2_b200.moe import dense_swiglu

        return self.dropout(dense_swiglu(x, self.gate_up_proj.weight, self.down_proj.weight))

"""Linear factory of the expert projections (counterpart of
ats/model/quantization.py:40-193).

``make_linear(in, out, quantization, bias)`` returns a plain ``nn.Linear``
for "none" and a ``QuantizedLinear`` otherwise.  ``QuantizedLinear`` is an
``nn.Linear`` subclass (so state-dict keys stay ``weight``/``bias``) whose
"int8" mode fake-quantises the weight (per tensor, symmetric) and the input
activations (per tensor, affine) to the int8 range on every forward with
torch.ao's FakeQuantize modules and moving-average min/max observers, with
straight-through gradients -- quantization-aware training as the reference
describes it.  "fp8" needs torchao, which this image does not ship: it raises
ImportError, as the reference does without a usable backend.

These modules run their own torch forward; the sm_100a expert kernels take
plain weights and refuse quantized experts (``ffn.require_plain_weights``).
"""

from __future__ import annotations

import torch
import torch.nn.functional as F
from torch import nn

MODES = ("none", "int8", "fp8")


class QuantizedLinear(nn.Linear):
    def __init__(self, in_features: int, out_features: int, quantization: str = "none", bias: bool = False) -> None:
        if quantization not in MODES:
            raise ValueError(f"Unknown quantization mode '{quantization}'. Fix: use one of 'none', 'int8', 'fp8'.")
        super().__init__(in_features, out_features, bias=bias)
        self.quantization = quantization
        if quantization == "int8":
            from torch.ao.quantization import FakeQuantize, MovingAverageMinMaxObserver

            def fq(scheme):
                return FakeQuantize(observer=MovingAverageMinMaxObserver, quant_min=-128, quant_max=127,
                                    dtype=torch.qint8, qscheme=scheme)

            self._weight_fake_quant = fq(torch.per_tensor_symmetric)
            self._act_fake_quant = fq(torch.per_tensor_affine)
        elif quantization == "fp8":
            try:
                import torchao  # noqa: F401
            except ImportError as exc:
                raise ImportError("FP8 training requires torchao (the supported backend). Install with: "
                                  "pip install torchao") from exc
            raise NotImplementedError("fp8 QuantizedLinear: torchao conversion is not built in ats_v2_b200")

    def forward(self, x: torch.Tensor) -> torch.Tensor:
        if self.quantization == "int8":
            return F.linear(self._act_fake_quant(x), self._weight_fake_quant(self.weight), self.bias)
        return F.linear(x, self.weight, self.bias)


def make_linear(in_features: int, out_features: int, quantization: str = "none", bias: bool = False) -> nn.Linear:
    if quantization == "none":
        return nn.Linear(in_features, out_features, bias=bias)
    return QuantizedLinear(in_features, out_features, quantization=quantization, bias=bias)

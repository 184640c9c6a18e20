"""ats/model/ffn.py on the sm_100a kernels: ats_v2_b200's SwiGLU, building its
projections with this tree's Linear factory (so quantized experts are
ats.model.quantization.QuantizedLinear)."""
from ats.model.quantization import make_linear

from ats_v2_b200.ffn import SwiGLU

SwiGLU.linear_factory = staticmethod(make_linear)

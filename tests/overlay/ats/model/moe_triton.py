"""ats/model/moe_triton.py on the sm_100a kernels: a re-export of ats_v2_b200.moe_fused."""
from ats_v2_b200.moe_fused import (HAS_TRITON, _pytorch_moe_routing, _triton_moe_routing,  # noqa: F401
                                   fused_moe_dispatch, fused_moe_routing)

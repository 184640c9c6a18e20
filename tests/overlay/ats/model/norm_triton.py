"""ats/model/norm_triton.py on the sm_100a kernels: a re-export of ats_v2_b200.norm_fused."""
from ats_v2_b200.norm_fused import (HAS_TRITON, _pytorch_rmsnorm_residual,  # noqa: F401
                                    _triton_rmsnorm_residual, fused_rmsnorm_residual)

"""ats/model/rope_triton.py on the sm_100a kernels: a re-export of ats_v2_b200.rope_fused."""
from ats_v2_b200.rope_fused import HAS_TRITON, _pytorch_apply_rope, _triton_apply_rope, fused_apply_rope  # noqa: F401

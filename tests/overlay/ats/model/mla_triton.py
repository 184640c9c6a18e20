"""ats/model/mla_triton.py on the sm_100a kernels: a re-export of ats_v2_b200.mla_fused."""
from ats_v2_b200.mla_fused import HAS_TRITON, _triton_matmul, fused_mla_kv_decompress  # noqa: F401

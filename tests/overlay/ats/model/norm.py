"""ats/model/norm.py on the sm_100a kernels: a re-export of ats_v2_b200.norm."""
from ats_v2_b200.norm import RMSNorm, rms_norm  # noqa: F401

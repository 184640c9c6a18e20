"""ats/model/moe.py on the sm_100a kernels: a re-export of ats_v2_b200.moe.
ats.model.ffn is imported first so that the experts use this tree's Linear factory."""
import ats.model.ffn  # noqa: F401

from ats_v2_b200.moe import MoELayer  # noqa: F401

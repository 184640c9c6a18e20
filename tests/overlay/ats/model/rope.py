"""ats/model/rope.py on the sm_100a kernels: a re-export of ats_v2_b200.rope."""
from ats_v2_b200.rope import RotaryEmbedding, apply_rotary_pos_emb, rotate_half  # noqa: F401

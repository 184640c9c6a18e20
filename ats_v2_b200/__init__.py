"""ats_v2_b200 -- B200 (sm_100a) kernels for the ats-v2 hot path.

RMSNorm, rotary embedding, the MoE layer and the MLA KV decompression GEMM,
forward and backward, as hand-written CUDA behind a C ABI
(``include/ats_b200.h``, ``libats_b200.so``), with PyTorch as the host.  The Python modules mirror
the reference's ``ats/model`` interfaces:

    ats/model/norm.py         -> ats_v2_b200.norm        (RMSNorm)
    ats/model/norm_triton.py  -> ats_v2_b200.norm_fused  (fused_rmsnorm_residual)
    ats/model/rope.py         -> ats_v2_b200.rope        (RotaryEmbedding, apply_rotary_pos_emb)
    ats/model/rope_triton.py  -> ats_v2_b200.rope_fused  (fused_apply_rope)
    ats/model/moe.py          -> ats_v2_b200.moe         (MoELayer)
    ats/model/moe_triton.py   -> ats_v2_b200.moe_fused   (fused_moe_routing, fused_moe_dispatch)
    ats/model/ffn.py          -> ats_v2_b200.ffn         (SwiGLU)
    ats/model/mla_triton.py   -> ats_v2_b200.mla_fused   (fused_mla_kv_decompress)

All compute runs on CUDA tensors; CPU tensors raise.
"""

__version__ = "0.1.0"

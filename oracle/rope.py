"""Oracle for rotary position embedding (test-only).

Reference:
  * ``ats/model/rope.py:29``     inv_freq = 1/theta^(arange(0, D, 2)/D), float32.
  * ``ats/model/rope.py:37-43``  cache: freqs = outer(t, inv_freq);
                                  emb = cat([freqs, freqs]); cos/sin of emb.
  * ``ats/model/rope.py:60-61``  tables sliced to seq_len and cast to x.dtype.
  * ``ats/model/rope.py:65-68``  rotate_half(x) = cat(-x2, x1).
  * ``ats/model/rope.py:71-87``  apply_rotary_pos_emb: x*cos + rotate_half(x)*sin
    for q [B,Hq,S,D] and k [B,Hk,S,D] with cos/sin [S,D] broadcast.
  * ``ats/model/rope_triton.py:100-105``  _pytorch_apply_rope: the same for one tensor.
  * backward: autograd of the expression above.  Each torch op rounds to the
    tensor dtype, so the oracle rounds after every multiply and the add.
"""

from __future__ import annotations

import numpy as np

from oracle.bf16 import round_to


def inv_freq(dim: int, theta: float) -> np.ndarray:
    """1 / theta^(2i/dim) in float32 (rope.py:29).

    The exponent is the float32 quotient; the power is the correctly rounded
    float32 of theta^e (torch evaluates a Python-scalar base to a tensor
    power that way); the reciprocal is a float32 division."""
    if dim % 2 != 0:
        raise ValueError(f"RotaryEmbedding dim must be even, got {dim}.")
    expo = np.arange(0, dim, 2, dtype=np.float32) / np.float32(dim)
    pw = np.power(np.float64(theta), expo.astype(np.float64)).astype(np.float32)
    return (np.float32(1.0) / pw).astype(np.float32)


def cos_sin_cache(seq_len: int, dim: int, theta: float, dtype: str = "f32"):
    """cos/sin tables [seq_len, dim] as rope.py:37-43 then :60-61 build them.

    The angle t*inv_freq is the float32 product; cos/sin of that float32 value
    are evaluated in float64 and rounded, i.e. correctly rounded float32."""
    f = inv_freq(dim, theta)
    t = np.arange(seq_len, dtype=np.float32)
    freqs = (t[:, None] * f[None, :]).astype(np.float32)
    emb = np.concatenate([freqs, freqs], axis=-1).astype(np.float64)
    cos = np.cos(emb).astype(np.float32)
    sin = np.sin(emb).astype(np.float32)
    return round_to(cos, dtype), round_to(sin, dtype)


def rotate_half(x: np.ndarray) -> np.ndarray:
    """cat(-x2, x1) along the last dim (rope.py:65-68)."""
    h = x.shape[-1] // 2
    return np.concatenate([-x[..., h:], x[..., :h]], axis=-1)


def _rotate_half_t(g: np.ndarray) -> np.ndarray:
    """Adjoint of rotate_half: cat(g2, -g1)."""
    h = g.shape[-1] // 2
    return np.concatenate([g[..., h:], -g[..., :h]], axis=-1)


def rope_fwd(x, cos, sin, dtype: str = "f32") -> np.ndarray:
    """x [B,H,S,D] -> round(round(x*cos) + round(rotate_half(x)*sin)) (rope.py:83-86)."""
    x = np.asarray(x, dtype=np.float32)
    c = np.asarray(cos, dtype=np.float32)[None, None]
    s = np.asarray(sin, dtype=np.float32)[None, None]
    a = round_to(x * c, dtype)
    b = round_to(rotate_half(x) * s, dtype)
    return round_to(a + b, dtype)


def rope_bwd(dout, cos, sin, dtype: str = "f32") -> np.ndarray:
    """Gradient of rope_fwd w.r.t. x: round(round(g*cos) + rotate_half^T(round(g*sin)))."""
    g = np.asarray(dout, dtype=np.float32)
    c = np.asarray(cos, dtype=np.float32)[None, None]
    s = np.asarray(sin, dtype=np.float32)[None, None]
    a = round_to(g * c, dtype)
    b = round_to(g * s, dtype)
    return round_to(a + _rotate_half_t(b), dtype)

"""Oracle for the fused MLA KV decompression (test-only).

Reference:
  * ``ats/model/mla_triton.py:122-151``  fused_mla_kv_decompress: (k, v) =
    (c @ w_uk.T, c @ w_uv.T) for c [..., latent] and w_uk, w_uv
    [out, latent].  The fused GPU path is one matmul against
    cat([w_uk, w_uv]) split in two (:144-148), the fallback two matmuls
    (:150-151): the same products.
  * ``ats/model/mla_triton.py:78-104``  _triton_matmul: float32 accumulation,
    one cast to the input dtype.
  * backward: autograd of the fallback's two matmuls.  dk w_uk and dv w_uv
    are each rounded to the tensor dtype and then added (autograd sums the
    two uses of c); dw_uk = dk^T c and dw_uv = dv^T c are rounded once.

This module is test infrastructure (the checker); no product path imports it.
"""

from __future__ import annotations

import numpy as np

from oracle.bf16 import round_to


def _mm(a: np.ndarray, b: np.ndarray, dtype: str) -> np.ndarray:
    """a @ b accumulated in float64, rounded once to dtype (float32 values)."""
    return round_to((a.astype(np.float64) @ b.astype(np.float64)).astype(np.float32), dtype)


def kv_decompress(c: np.ndarray, w_uk: np.ndarray, w_uv: np.ndarray, dtype: str = "f32"):
    """(k, v) for c [..., latent] (mla_triton.py:144-156)."""
    lead = c.shape[:-1]
    c2 = c.reshape(-1, c.shape[-1])
    k = _mm(c2, w_uk.T, dtype).reshape(*lead, w_uk.shape[0])
    v = _mm(c2, w_uv.T, dtype).reshape(*lead, w_uv.shape[0])
    return k, v


def kv_decompress_bwd(dk: np.ndarray, dv: np.ndarray, c: np.ndarray, w_uk: np.ndarray, w_uv: np.ndarray,
                      dtype: str = "f32"):
    """(dc, dw_uk, dw_uv): autograd of the fallback's two matmuls."""
    lead = c.shape[:-1]
    c2 = c.reshape(-1, c.shape[-1])
    dk2 = dk.reshape(-1, dk.shape[-1])
    dv2 = dv.reshape(-1, dv.shape[-1])
    dc = round_to(_mm(dk2, w_uk, dtype) + _mm(dv2, w_uv, dtype), dtype).reshape(*lead, c.shape[-1])
    return dc, _mm(dk2.T, c2, dtype), _mm(dv2.T, c2, dtype)

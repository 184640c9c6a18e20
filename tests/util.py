"""Helpers shared by the GPU parity tests."""

from __future__ import annotations

import numpy as np
import torch

# north-star tolerances
F32 = dict(rtol=1e-5, atol=1e-6)
BF16 = dict(rtol=2e-2, atol=1e-2)


def np32(t: torch.Tensor) -> np.ndarray:
    return t.detach().float().cpu().numpy()


def dev(a, dtype=torch.float32, requires_grad: bool = False) -> torch.Tensor:
    """numpy float32 (bf16-exact values for bf16) -> CUDA tensor of dtype (exact)."""
    t = torch.from_numpy(np.ascontiguousarray(a, dtype=np.float32)).to("cuda").to(dtype)
    return t.requires_grad_(requires_grad)


def exact_fraction(a: np.ndarray, b: np.ndarray) -> float:
    a = np.ascontiguousarray(a, dtype=np.float32)
    b = np.ascontiguousarray(b, dtype=np.float32)
    return float(np.mean(a.view(np.uint32) == b.view(np.uint32)))


def close(actual, expected, dtype: str, min_exact: float | None = None, **tol) -> None:
    a = np32(actual) if isinstance(actual, torch.Tensor) else np.asarray(actual, np.float32)
    b = np.asarray(expected, np.float32)
    kw = dict(F32 if dtype == "f32" else BF16)
    kw.update(tol)
    np.testing.assert_allclose(a, b, **kw)
    if min_exact is not None:
        fr = exact_fraction(a, b)
        assert fr >= min_exact, f"only {fr:.5f} bit-identical (need {min_exact})"


def seeded_normal(shape, seed: int, scale: float = 1.0, shift: float = 0.0) -> np.ndarray:
    rng = np.random.default_rng(seed)
    return (shift + scale * rng.standard_normal(shape)).astype(np.float32)


def close_f32_sum(actual, expected, abs_sum, rtol: float = 1e-5, k: float = 2e-6) -> None:
    """A float32 reduction against its float64 value: per element
    |a - e| <= rtol*|e| + k*sum|terms|.  The first term is the north-star
    1e-5 relative bound; the second is the rounding a float32 sum of those
    terms can carry (a sum that cancels to near zero has no relative accuracy
    to offer), the criterion torch's own float32 reductions meet."""
    a = np32(actual) if isinstance(actual, torch.Tensor) else np.asarray(actual, np.float32)
    e = np.asarray(expected, np.float64)
    bound = rtol * np.abs(e) + k * np.asarray(abs_sum, np.float64)
    err = np.abs(a.astype(np.float64) - e)
    bad = err > bound
    assert not bad.any(), (f"{int(bad.sum())} of {bad.size} elements outside rtol={rtol} + {k}*sum|terms|; "
                           f"worst excess {float((err - bound).max()):.3e}")

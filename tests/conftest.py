"""Shared pytest configuration.

Markers:
  gpu -- needs a CUDA device and the built sm_100a library; the CPU suite
         (``-m "not gpu"``) covers the oracle, the host-side logic and the
         C-ABI symbol table.
"""

from __future__ import annotations

import sys
from pathlib import Path

import numpy as np
import pytest

ROOT = Path(__file__).resolve().parents[1]
if str(ROOT) not in sys.path:
    sys.path.insert(0, str(ROOT))

GOLDEN = ROOT / "tests" / "golden"


def pytest_configure(config):
    config.addinivalue_line("markers", "gpu: requires a CUDA GPU (B200, sm_100a) and the built library")


def load_golden(name: str) -> dict:
    """Load tests/golden/<name>.npz; *_bf16 keys are decoded to float32."""
    from oracle.bf16 import bf16_bits_to_f32

    with np.load(GOLDEN / f"{name}.npz") as z:
        out = {}
        for k in z.files:
            v = z[k]
            if k.endswith("_bf16"):
                out[k[:-5]] = bf16_bits_to_f32(v)
                out[k[:-5] + "__is_bf16"] = True
            else:
                out[k] = v
        return out


@pytest.fixture
def golden():
    return load_golden

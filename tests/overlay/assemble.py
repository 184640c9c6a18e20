"""Assemble the reference tree with its hot-path modules swapped for ats_v2_b200.

    python tests/overlay/assemble.py <ats-v2 checkout> [--out baseline/_ref/overlay]

Copies the reference's ``ats/``, ``tests/``, ``configs/``, ``pyproject.toml``
and ``preprocess.py`` into ``--out`` (default ``baseline/_ref/overlay`` of this
repository, which git ignores) and replaces ``ats/model/{norm, rope, ffn, moe,
norm_triton, rope_triton, moe_triton, mla_triton}.py`` with the thin
re-exports under ``tests/overlay/ats/model``: the change a maintainer makes to
run the reference on these kernels.  The reference's own tests then run
unchanged against the swapped modules (``tests/test_reference_overlay.py``);
run them with ``PYTHONPATH=<out>:<this repository>``.
"""

from __future__ import annotations

import argparse
import shutil
import sys
from pathlib import Path

HERE = Path(__file__).resolve().parent
REPO = HERE.parents[1]
DEFAULT_OUT = REPO / "baseline" / "_ref" / "overlay"
SWAPPED = ("norm", "rope", "ffn", "moe", "norm_triton", "rope_triton", "moe_triton", "mla_triton")
COPIED = ("ats", "tests", "configs", "pyproject.toml", "preprocess.py")


def assemble(reference: Path, out: Path = DEFAULT_OUT) -> Path:
    reference = Path(reference).resolve()
    if not (reference / "ats" / "model" / "moe.py").is_file():
        raise SystemExit(f"{reference} is not an ats-v2 checkout (no ats/model/moe.py)")
    if out.exists():
        shutil.rmtree(out)
    out.mkdir(parents=True)
    ignore = shutil.ignore_patterns("__pycache__", "*.pyc", ".DS_Store")
    for name in COPIED:
        src = reference / name
        if src.is_dir():
            shutil.copytree(src, out / name, ignore=ignore)
        elif src.is_file():
            shutil.copy2(src, out / name)
    for mod in SWAPPED:
        shutil.copy2(HERE / "ats" / "model" / f"{mod}.py", out / "ats" / "model" / f"{mod}.py")
    return out


def main() -> None:
    ap = argparse.ArgumentParser(description=__doc__.splitlines()[0])
    ap.add_argument("reference", type=Path, help="an ats-v2 checkout")
    ap.add_argument("--out", type=Path, default=DEFAULT_OUT)
    a = ap.parse_args()
    print(assemble(a.reference, a.out))


if __name__ == "__main__":
    sys.exit(main())

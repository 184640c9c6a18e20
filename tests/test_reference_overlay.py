"""The reference's own tests, unchanged, on the reference tree with its hot-path
modules swapped for ats_v2_b200 (``tests/overlay/assemble.py``).

The assembled tree lives in ``baseline/_ref/overlay`` (git-ignored, built
from an ats-v2 checkout by the assembler; it is built again from
``ATS_REFERENCE_DIR`` when that names a checkout).  Without either the tests
skip and say so.

* CPU: the reference's whole suite.  Its CPU tests call the swapped modules
  with CPU tensors, which take the reference's torch formulas; the model
  tests build ``ATSTransformer`` (dense, MoE, MLA, quantized) from the swapped
  RMSNorm, RoPE, SwiGLU and MoELayer.
* GPU: ``tests/test_triton.py``, whose four kernel-parity tests run (none may
  skip) against the CUDA kernels, and ``ATSTransformer`` with ``use_moe`` run
  forward and backward on CUDA tensors, compared with the same model on CPU
  tensors (the reference's formulas).
"""

from __future__ import annotations

import os
import subprocess
import sys
from pathlib import Path

import pytest

REPO = Path(__file__).resolve().parents[1]
OVERLAY = REPO / "baseline" / "_ref" / "overlay"


def _overlay() -> Path:
    src = os.environ.get("ATS_REFERENCE_DIR")
    if src and Path(src, "ats", "model", "moe.py").is_file():
        sys.path.insert(0, str(REPO / "tests" / "overlay"))
        from assemble import assemble

        return assemble(Path(src), OVERLAY)
    if not (OVERLAY / "ats" / "model" / "moe.py").is_file():
        pytest.skip("no assembled reference tree: run tests/overlay/assemble.py <ats-v2 checkout> "
                    "(or set ATS_REFERENCE_DIR)")
    return OVERLAY


def _pytest(tree: Path, *args: str, timeout: int = 900) -> subprocess.CompletedProcess:
    env = dict(os.environ, PYTHONPATH=os.pathsep.join([str(tree), str(REPO)]))
    return subprocess.run([sys.executable, "-m", "pytest", "-q", "-p", "no:cacheprovider", "-rs", *args],
                          cwd=tree, env=env, capture_output=True, text=True, timeout=timeout)


def test_reference_suite_runs_unchanged_on_the_swapped_modules_cpu():
    tree = _overlay()
    r = _pytest(tree, "tests")
    tail = (r.stdout + r.stderr)[-3000:]
    assert r.returncode == 0, tail
    assert " passed" in r.stdout and " failed" not in r.stdout, tail


_MODEL_SCRIPT = r'''
import copy, torch
from ats.config.schema import ModelConfig
from ats.model.transformer import ATSTransformer
torch.backends.cuda.matmul.allow_tf32 = False
torch.backends.cudnn.allow_tf32 = False
torch.manual_seed(0)
cfg = ModelConfig(hidden_size=256, num_layers=2, num_heads=4, num_kv_heads=2, intermediate_size=512,
                  vocab_size=512, max_seq_len=64, use_moe=True, num_experts=4, moe_top_k=2,
                  use_flash_attention=False)
cpu = ATSTransformer(cfg, ep_size=1)
gpu = copy.deepcopy(cpu).cuda()
ids = torch.randint(0, cfg.vocab_size, (2, 64))
out_c = cpu(ids)
out_g = gpu(ids.cuda())
loss_c = out_c.logits.float().pow(2).mean() + out_c.aux_loss
loss_g = out_g.logits.float().pow(2).mean() + out_g.aux_loss
loss_c.backward()
loss_g.backward()
err = (out_g.logits.cpu() - out_c.logits).abs().max().item()
scale = out_c.logits.abs().max().item()
print("logits max err", err, "scale", scale, "aux", out_c.aux_loss.item(), out_g.aux_loss.item())
assert err <= 1e-4 * max(1.0, scale), err
assert abs(out_g.aux_loss.item() - out_c.aux_loss.item()) <= 1e-5 * max(1.0, abs(out_c.aux_loss.item()))
worst = 0.0
for (n, pc), (_, pg) in zip(cpu.named_parameters(), gpu.named_parameters()):
    if pc.grad is None:
        assert pg.grad is None, n
        continue
    d = (pg.grad.cpu() - pc.grad).abs().max().item() / max(pc.grad.abs().max().item(), 1e-12)
    worst = max(worst, d)
    assert d <= 1e-3, (n, d)
print("grads: worst relative max err", worst)
from ats.model.moe import MoELayer
assert isinstance(gpu.layers[0].ffn, MoELayer) and gpu.layers[0].ffn.uses_deepspeed is False
from ats_v2_b200 import _lib
print("kernel launches", _lib.load().ats_kernel_launches())
assert _lib.load().ats_kernel_launches() > 0
print("MODEL_OK")
'''


@pytest.mark.gpu
def test_reference_kernel_tests_run_on_the_cuda_kernels():
    tree = _overlay()
    r = _pytest(tree, "tests/test_triton.py")
    tail = (r.stdout + r.stderr)[-3000:]
    assert r.returncode == 0, tail
    assert "12 passed" in r.stdout and "skipped" not in r.stdout, tail


@pytest.mark.gpu
def test_reference_moe_transformer_forward_backward_on_cuda_matches_cpu():
    tree = _overlay()
    env = dict(os.environ, PYTHONPATH=os.pathsep.join([str(tree), str(REPO)]))
    r = subprocess.run([sys.executable, "-c", _MODEL_SCRIPT], cwd=tree, env=env, capture_output=True, text=True,
                       timeout=600)
    tail = (r.stdout + r.stderr)[-3000:]
    assert r.returncode == 0 and "MODEL_OK" in r.stdout, tail

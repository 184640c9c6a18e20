"""Benchmark of the ats-v2 hot path on B200.

    python bench.py [--gpus N] [--steps K] [--warmup W] [--workload NAME] [--impl ours|reference]

Workloads (synthetic, seeded; the reference publishes no dataset for this path):
  moe_ep    expert-parallel MoE layer forward+backward, 32768 tokens per GPU,
            hidden 4096, 64 experts top-2 sharded over the GPUs, ffn 1408,
            capacity factor 1.25, Zipf(1.1) expert skew (metric: tokens/s)  -- default
  ffn       dense SwiGLU FFN forward+backward, 16384 tokens, hidden 4096, ffn
            11008, bf16 (metric: tokens/s)
  mla       MLA KV decompression forward+backward, 16384 tokens, latent 1024,
            k and v 4096 each, bf16 (metric: tokens/s)
  rmsnorm   RMSNorm forward+backward, x [4,4096,4096] bf16, weight fp32, eps 1e-5
            (metric: HBM GB/s of algorithmic traffic)
  rope      fused q/k RoPE forward+backward, q [4,4096,32,128], k [4,4096,8,128]
            bf16, theta 5e5 (metric: HBM GB/s)
  moe       MoE layer forward+backward, 8192 tokens, hidden 2048, 8 experts
            top-2, ffn 5632, bf16, fp32 router, no capacity drop (metric: tokens/s)

The expert-parallel layer is the headline because it is the configuration
measured at 1, 2, 4 and 8 GPUs; at one GPU all 64 experts are local.  One JSON
line is printed by rank 0.  ``value`` is the device-timed throughput with
inputs resident in HBM (CUDA events on the launching stream, K steps after W
warm-up steps, barrier + synchronize on both sides, max over ranks); ``e2e`` is
the same metric through the public module API with pinned host inputs copied
in and all results copied out inside the timed region; ``roofline`` times the
dominant kernel with CUDA events inside the timed region, against the burst
tensor peak for a timed region under a second and the sustained one beyond;
``cpu_baseline`` times the reference's own modules (installed in
baseline/_ref) on the host cores on a bounded sample, or the numpy
restatement of its algorithm (``oracle/``) when the reference is not
installed.  Unless ``--no-extras``, the line also carries ``extras``: the
other workloads measured the same way, reduced to their numbers.  Under
torchrun every rank runs its own shard (weak scaling): RMSNorm, RoPE, the
dense FFN, MLA and the single-GPU MoE layer have no collective on the data
path; ``moe_ep`` exchanges expert rows between the ranks.

``--impl reference`` times the reference's own CPU implementation of the
workload (its modules from baseline/_ref, torch on every host thread) on the
same metric and configuration, rank 0 only.
"""

from __future__ import annotations

import argparse
import json
import os
import statistics
import subprocess
import sys
import time
from concurrent.futures import ThreadPoolExecutor
from pathlib import Path

import numpy as np

ROOT = Path(__file__).resolve().parent
sys.path.insert(0, str(ROOT))

PEAKS_FALLBACK = {"hbm_gbs": 6650.0, "bf16_tflops": 1590.0, "bf16_tflops_sustained": 1400.0}


def load_peaks() -> tuple[dict, str]:
    p = ROOT / "MEASURED_PEAKS.json"
    if p.exists():
        try:
            return json.loads(p.read_text()), "measured"
        except Exception:
            pass
    return dict(PEAKS_FALLBACK), "fallback"


# ---------------------------------------------------------------- clocks
class ClockSampler:
    """nvidia-smi clocks/throttle sampling during the timed region."""

    FIELDS = ("index,clocks.sm,clocks.max.sm,power.draw,clocks_event_reasons.hw_slowdown,"
              "clocks_event_reasons.hw_thermal_slowdown,clocks_event_reasons.sw_thermal_slowdown,"
              "clocks_event_reasons.sw_power_cap")

    def __init__(self, gpu_index: int):
        self.gpu = gpu_index
        self.proc = None

    def __enter__(self):
        try:
            self.proc = subprocess.Popen(
                ["nvidia-smi", f"--query-gpu={self.FIELDS}", "--format=csv,noheader,nounits", "-lms", "100",
                 "-i", str(self.gpu)], stdout=subprocess.PIPE, stderr=subprocess.DEVNULL, text=True)
        except Exception:
            self.proc = None
        time.sleep(0.25)
        return self

    def __exit__(self, *exc):
        self.summary = {"error": "nvidia-smi unavailable"}
        if self.proc is None:
            return False
        time.sleep(0.15)
        self.proc.terminate()
        try:
            out, _ = self.proc.communicate(timeout=5)
        except Exception:
            self.proc.kill()
            out = ""
        mhz, mx, reasons, power = [], None, set(), []
        names = ["hw_slowdown", "hw_thermal_slowdown", "sw_thermal_slowdown", "sw_power_cap"]
        for line in out.strip().splitlines():
            parts = [p.strip() for p in line.split(",")]
            if len(parts) < 8:
                continue
            try:
                mhz.append(float(parts[1]))
                mx = float(parts[2])
                power.append(float(parts[3]))
            except ValueError:
                continue
            for nm, v in zip(names, parts[4:8]):
                if v.lower() in ("active", "1", "yes"):
                    reasons.add(nm)
        if mhz:
            self.summary = {"sm_mhz": statistics.median(mhz), "sm_max_mhz": mx, "reasons": sorted(reasons),
                            "samples": len(mhz), "power_w_max": max(power) if power else None}
        return False


# ---------------------------------------------------------------- helpers
def dist_env():
    world = int(os.environ.get("WORLD_SIZE", "1"))
    rank = int(os.environ.get("RANK", "0"))
    local = int(os.environ.get("LOCAL_RANK", "0"))
    return world, rank, local


def cpu_threads() -> int:
    try:
        return len(os.sched_getaffinity(0))
    except Exception:
        return os.cpu_count() or 1


def run_threads(fn, chunks, threads):
    with ThreadPoolExecutor(max_workers=threads) as ex:
        return list(ex.map(fn, chunks))


# ---------------------------------------------------------------- workloads
REF_DIR = ROOT / "baseline" / "_ref"


def reference_modules():
    """The unmodified reference's ats.model modules, as pip installed them into
    baseline/_ref (git-ignored; it travels with the repository to the GPU box),
    or None when it is not there."""
    if not (REF_DIR / "ats" / "model" / "moe.py").is_file():
        return None
    import importlib
    import logging

    if str(REF_DIR) not in sys.path:
        sys.path.insert(0, str(REF_DIR))
    logging.getLogger("ats.model.moe").setLevel(logging.ERROR)  # its "no DeepSpeed" notice, once per layer
    mods = {n: importlib.import_module(f"ats.model.{n}") for n in ("norm", "rope", "moe", "ffn", "mla_triton")}
    if Path(mods["moe"].__file__).resolve().parent != (REF_DIR / "ats" / "model").resolve():
        raise RuntimeError(f"ats.model resolved to {mods['moe'].__file__}, not the reference in {REF_DIR}")
    return mods


def timed_passes(fn, seconds: float):
    """Run fn() until `seconds` have passed (at least once); (passes, elapsed s)."""
    t0 = time.perf_counter()
    n = 0
    while True:
        fn()
        n += 1
        if time.perf_counter() - t0 >= seconds:
            return n, time.perf_counter() - t0


class Workload:
    name = ""
    metric = ""
    unit = ""
    dtype = "bf16"

    def __init__(self, torch, rank: int, world: int, peaks: dict, peaks_kind: str):
        self.torch = torch
        self.rank, self.world = rank, world
        self.peaks, self.peaks_kind = peaks, peaks_kind

    def cpu_baseline(self, seconds: float) -> dict:
        """The reference's own modules on the host cores (torch on CPU, every
        host thread), on a bounded sample of the workload; the numpy
        restatement of its algorithm (oracle/) when the reference is not
        installed in baseline/_ref."""
        mods = reference_modules()
        if mods is None:
            return self.port_baseline(seconds)
        import torch
        threads = cpu_threads()
        torch.set_num_threads(threads)
        fn, units, sample = self.reference_pass(mods, torch)
        fn()  # warm-up pass
        n, dt = timed_passes(fn, seconds)
        return {"value": units * n / dt, "unit": self.unit, "cores": threads, "kind": "reference",
                "sample": f"{sample}; {n} passes in {dt:.1f} s (the reference's modules from baseline/_ref, "
                          f"torch on CPU, {threads} threads)"}


class RMSNormWorkload(Workload):
    name = "rmsnorm"
    metric = "rmsnorm_fwd_bwd_hbm_gbs"
    unit = "GB/s"
    ROWS, H = 16384, 4096

    def bytes_per_step(self) -> int:
        # fwd: read x, write y; bwd: read x, dy, write dx; + w read twice, dw write (fp32)
        n = self.ROWS * self.H * 2
        return 5 * n + 3 * self.H * 4

    def config(self):
        return {"workload": "RMSNorm fwd+bwd, x[4,4096,4096] bf16, weight fp32, eps 1e-5",
                "rows": self.ROWS, "hidden": self.H, "per_rank": "full workload per GPU (replicas)",
                "l2": "inputs larger than L2 (x and dy 134 MB each)"}

    def setup(self):
        t = self.torch
        from ats_v2_b200.norm import RMSNorm
        g = t.Generator(device="cuda").manual_seed(self.rank)
        self.x = t.randn(self.ROWS, self.H, device="cuda", generator=g).bfloat16().requires_grad_()
        self.dy = t.randn(self.ROWS, self.H, device="cuda", generator=g).bfloat16()
        self.mod = RMSNorm(self.H, eps=1e-5).cuda()
        with t.no_grad():
            self.mod.weight.copy_(1 + 0.02 * t.randn(self.H, device="cuda", generator=g))

    def step(self, evs):
        y = self.mod(self.x)
        self.x.grad = None
        self.mod.weight.grad = None
        if evs:
            evs[0].record()
        y.backward(self.dy)
        if evs:
            evs[1].record()

    def dominant(self):
        # rmsnorm_bwd_kernel (+ the tiny dw reduce): reads x, dy, writes dx
        return {"kernel": "rmsnorm_bwd_kernel<bf16,float>", "bytes": 3 * self.ROWS * self.H * 2 + 2 * self.H * 4,
                "bound": "hbm",
                # DRAM read+write of one backward launch (ring kernel + dw reduce), ncu, cold caches
                "traffic": (268.5 + 100.8 + 2.4) * 1e6,
                "traffic_source": "profiles/rmsnorm_ring_16384x4096_bf16_fp32w.md (writes still in L2 at kernel "
                                  "end are not counted)"}

    # e2e through the public module with pinned host buffers
    def e2e_setup(self):
        t = self.torch
        self.hx = self.x.detach().cpu().pin_memory()
        self.hdy = self.dy.cpu().pin_memory()
        self.hy = t.empty_like(self.hx).pin_memory()
        self.hdx = t.empty_like(self.hx).pin_memory()
        self.hdw = t.empty(self.H, dtype=t.float32).pin_memory()
        self.dx_in = t.empty_like(self.x.detach())
        self.ddy = t.empty_like(self.dy)
        self.h2d = self.hx.numel() * 2 + self.hdy.numel() * 2
        self.d2h = self.hy.numel() * 2 + self.hdx.numel() * 2 + self.H * 4

    def e2e_step(self):
        self.dx_in.copy_(self.hx, non_blocking=True)
        self.ddy.copy_(self.hdy, non_blocking=True)
        x = self.dx_in.requires_grad_()
        self.mod.weight.grad = None
        y = self.mod(x)
        y.backward(self.ddy)
        self.hy.copy_(y.detach(), non_blocking=True)
        self.hdx.copy_(x.grad, non_blocking=True)
        self.hdw.copy_(self.mod.weight.grad, non_blocking=True)
        x.grad = None
        x.requires_grad_(False)

    def units_to_value(self, steps, ms):  # GB/s over all work
        return self.bytes_per_step() * steps / (ms * 1e-3) / 1e9

    # CPU restatement timed on host cores (bounded sample of rows)
    def port_baseline(self, seconds: float):
        from oracle import norm as onorm
        from oracle.bf16 import round_bf16
        threads = cpu_threads()
        rows = 64 * threads
        rng = np.random.default_rng(0)
        x = round_bf16(rng.standard_normal((rows, self.H)).astype(np.float32))
        dy = round_bf16(rng.standard_normal((rows, self.H)).astype(np.float32))
        w = (1 + 0.02 * rng.standard_normal(self.H)).astype(np.float32)
        parts = np.array_split(np.arange(rows), threads)

        def work(ix):
            onorm.rmsnorm_fwd(x[ix], w, 1e-5, "bf16")
            onorm.rmsnorm_bwd(dy[ix], x[ix], w, 1e-5, "bf16", "f32")

        t0 = time.perf_counter()
        n = 0
        while True:
            run_threads(work, parts, threads)
            n += 1
            if time.perf_counter() - t0 >= seconds:
                break
        dt = time.perf_counter() - t0
        bytes_ = (5 * rows * self.H * 2 + 3 * self.H * 4) * n
        return {"value": bytes_ / dt / 1e9, "unit": self.unit, "cores": threads, "kind": "port",
                "sample": f"{rows} of {self.ROWS} rows per pass, {n} passes in {dt:.1f} s (numpy oracle, "
                          f"{threads} threads)"}


    def reference_pass(self, mods, torch):
        rows = self.ROWS // 4
        g = torch.Generator().manual_seed(0)
        x = torch.randn(rows, self.H, generator=g).bfloat16().requires_grad_()
        dy = torch.randn(rows, self.H, generator=g).bfloat16()
        m = mods["norm"].RMSNorm(self.H, eps=1e-5)
        with torch.no_grad():
            m.weight.copy_(1 + 0.02 * torch.randn(self.H, generator=g))

        def fn():
            x.grad = None
            m.weight.grad = None
            m(x).backward(dy)

        return fn, (5 * rows * self.H * 2 + 3 * self.H * 4) / 1e9, f"{rows} of {self.ROWS} rows per pass"


class RopeWorkload(Workload):
    name = "rope"
    metric = "rope_qk_fwd_bwd_hbm_gbs"
    unit = "GB/s"
    B, S, HQ, HK, D = 4, 4096, 32, 8, 128

    def bytes_per_step(self) -> int:
        n = self.B * self.S * (self.HQ + self.HK) * self.D * 2
        return 4 * n  # fwd read+write, bwd read+write

    def config(self):
        return {"workload": "q/k RoPE fwd+bwd, q[4,4096,32,128] k[4,4096,8,128] bf16 BSHD views, theta 5e5",
                "per_rank": "full workload per GPU (replicas)", "l2": "inputs larger than L2 (q 134 MB)"}

    def setup(self):
        t = self.torch
        from ats_v2_b200.rope import RotaryEmbedding, apply_rotary_pos_emb
        self.apply = apply_rotary_pos_emb
        g = t.Generator(device="cuda").manual_seed(self.rank)
        self.qm = t.randn(self.B, self.S, self.HQ, self.D, device="cuda", generator=g).bfloat16()
        self.km = t.randn(self.B, self.S, self.HK, self.D, device="cuda", generator=g).bfloat16()
        # upstream gradients in the layout attention hands back: BSHD memory viewed as [B,H,S,D]
        self.gq = t.randn(self.B, self.S, self.HQ, self.D, device="cuda", generator=g).bfloat16().transpose(1, 2)
        self.gk = t.randn(self.B, self.S, self.HK, self.D, device="cuda", generator=g).bfloat16().transpose(1, 2)
        self.rope = RotaryEmbedding(self.D, self.S, 500000.0).cuda()

    def step(self, evs):
        t = self.torch
        q = self.qm.transpose(1, 2).requires_grad_()
        k = self.km.transpose(1, 2).requires_grad_()
        cos, sin = self.rope(self.S, self.qm.device, t.bfloat16)
        if evs:
            evs[0].record()
        qo, ko = self.apply(q, k, cos, sin)
        if evs:
            evs[1].record()
        t.autograd.backward([qo, ko], [self.gq, self.gk])

    def dominant(self):
        return {"kernel": "rope_vec_kernel<bf16> (forward launch)", "bytes": self.bytes_per_step() // 2,
                "bound": "hbm", "traffic": (174.2 + 117.4) * 1e6,
                "traffic_source": "profiles/rope_vec_q4x4096x32x128_k4x4096x8x128_bf16.md (ncu, cold caches; "
                                  "writes still in L2 at kernel end are not counted)"}

    def e2e_setup(self):
        t = self.torch
        self.hq = self.qm.cpu().pin_memory()
        self.hk = self.km.cpu().pin_memory()
        self.hgq = self.gq.transpose(1, 2).cpu().pin_memory()  # BSHD host buffers
        self.hgk = self.gk.transpose(1, 2).cpu().pin_memory()
        self.hqo = t.empty_like(self.hq).pin_memory()
        self.hko = t.empty_like(self.hk).pin_memory()
        self.hdq = t.empty_like(self.hq).pin_memory()
        self.hdk = t.empty_like(self.hk).pin_memory()
        self.dq_in, self.dk_in = t.empty_like(self.qm), t.empty_like(self.km)
        self.dgq_m, self.dgk_m = t.empty_like(self.qm), t.empty_like(self.km)
        n = (self.hq.numel() + self.hk.numel()) * 2
        self.h2d = 2 * n
        self.d2h = 2 * n

    def e2e_step(self):
        t = self.torch
        for dst, src in ((self.dq_in, self.hq), (self.dk_in, self.hk), (self.dgq_m, self.hgq), (self.dgk_m, self.hgk)):
            dst.copy_(src, non_blocking=True)
        q = self.dq_in.transpose(1, 2).requires_grad_()
        k = self.dk_in.transpose(1, 2).requires_grad_()
        cos, sin = self.rope(self.S, self.qm.device, t.bfloat16)
        qo, ko = self.apply(q, k, cos, sin)
        t.autograd.backward([qo, ko], [self.dgq_m.transpose(1, 2), self.dgk_m.transpose(1, 2)])
        self.hqo.copy_(qo.detach().transpose(1, 2), non_blocking=True)
        self.hko.copy_(ko.detach().transpose(1, 2), non_blocking=True)
        self.hdq.copy_(q.grad.transpose(1, 2), non_blocking=True)
        self.hdk.copy_(k.grad.transpose(1, 2), non_blocking=True)

    def units_to_value(self, steps, ms):
        return self.bytes_per_step() * steps / (ms * 1e-3) / 1e9

    def port_baseline(self, seconds: float):
        from oracle import rope as orope
        from oracle.bf16 import round_bf16
        threads = cpu_threads()
        pos = 8 * threads
        rng = np.random.default_rng(0)
        q = round_bf16(rng.standard_normal((1, self.HQ, pos, self.D)).astype(np.float32))
        k = round_bf16(rng.standard_normal((1, self.HK, pos, self.D)).astype(np.float32))
        cos, sin = orope.cos_sin_cache(pos, self.D, 500000.0, "bf16")
        parts = np.array_split(np.arange(pos), threads)

        def work(ix):
            for x in (q[:, :, ix], k[:, :, ix]):
                y = orope.rope_fwd(x, cos[ix], sin[ix], "bf16")
                orope.rope_bwd(y, cos[ix], sin[ix], "bf16")

        t0 = time.perf_counter()
        n = 0
        while True:
            run_threads(work, parts, threads)
            n += 1
            if time.perf_counter() - t0 >= seconds:
                break
        dt = time.perf_counter() - t0
        bytes_ = 4 * pos * (self.HQ + self.HK) * self.D * 2 * n
        return {"value": bytes_ / dt / 1e9, "unit": self.unit, "cores": threads, "kind": "port",
                "sample": f"{pos} of {self.B * self.S} (batch, position) rows of q and k per pass, {n} passes "
                          f"in {dt:.1f} s (numpy oracle, {threads} threads)"}


    def reference_pass(self, mods, torch):
        B = 1  # one of the 4 sequences per pass
        g = torch.Generator().manual_seed(0)
        qm = torch.randn(B, self.S, self.HQ, self.D, generator=g).bfloat16()
        km = torch.randn(B, self.S, self.HK, self.D, generator=g).bfloat16()
        gq = torch.randn(B, self.HQ, self.S, self.D, generator=g).bfloat16()
        gk = torch.randn(B, self.HK, self.S, self.D, generator=g).bfloat16()
        rope = mods["rope"].RotaryEmbedding(self.D, self.S, 500000.0)

        def fn():
            q = qm.transpose(1, 2).requires_grad_()
            k = km.transpose(1, 2).requires_grad_()
            cos, sin = rope(self.S, torch.device("cpu"), torch.bfloat16)
            qo, ko = mods["rope"].apply_rotary_pos_emb(q, k, cos, sin)
            torch.autograd.backward([qo, ko], [gq, gk])

        return (fn, 4 * B * self.S * (self.HQ + self.HK) * self.D * 2 / 1e9,
                f"{B} of {self.B} sequences (all {self.S} positions, q and k) per pass")


class MoEWorkload(Workload):
    name = "moe"
    metric = "moe_layer_fwd_bwd_tokens_per_s"
    unit = "tokens/s"
    T, H, F, E, K = 8192, 2048, 5632, 8, 2

    def flops_per_step(self) -> int:
        return 3 * 6 * self.T * self.K * self.H * self.F  # expert GEMMs, fwd + bwd

    def config(self):
        return {"workload": "MoE layer fwd+bwd, 8192 tokens, hidden 2048, 8 experts top-2, ffn 5632, bf16, "
                            "fp32 router, capacity factor E/k (no drop)",
                "per_rank": "full workload per GPU (replicas)",
                "l2": "inputs larger than L2 (expert weights 553 MB)"}

    def setup(self):
        t = self.torch
        from ats_v2_b200.moe import MoELayer
        t.manual_seed(1000 + self.rank)
        layer = MoELayer(self.H, self.F, self.E, num_layers=2, top_k=self.K, capacity_factor=self.E / self.K)
        with t.no_grad():
            layer.moe.gate.weight.normal_(0, 0.02)
            for ex in layer.moe.experts:
                ex.gate_up_proj.weight.normal_(0, 0.02)
                ex.down_proj.weight.normal_(0, 0.02)
        self.layer = layer.cuda()
        self.layer.moe.experts.to(t.bfloat16)
        g = t.Generator(device="cuda").manual_seed(self.rank)
        self.x = t.randn(1, self.T, self.H, device="cuda", generator=g).bfloat16().requires_grad_()
        self.dy = t.randn(1, self.T, self.H, device="cuda", generator=g).bfloat16()
        self.one = t.ones((), device="cuda")

    def _zero(self):
        for p in self.layer.parameters():
            p.grad = None

    def step(self, evs):
        t = self.torch
        self._zero()
        self.x.grad = None
        if evs:
            evs[0].record()
        out, aux = self.layer(self.x)
        t.autograd.backward([out, aux], [self.dy, self.one])
        if evs:
            evs[1].record()

    def dominant(self):
        return {"kernel": "expert grouped GEMMs (whole layer fwd+bwd timed)", "flops": self.flops_per_step(),
                "bound": "tensor", "traffic": (3523.6 + 1488.0) * 1e6,
                "traffic_source": "profiles/moe_gemms_8192tok_h2048_e8_top2_f5632_bf16.md: DRAM read+write of "
                                  "the six expert GEMM launches of one step (ncu, cold caches)"}

    def e2e_setup(self):
        t = self.torch
        self.hx = self.x.detach().cpu().pin_memory()
        self.hdy = self.dy.cpu().pin_memory()
        self.hout = t.empty_like(self.hx).pin_memory()
        self.hdx = t.empty_like(self.hx).pin_memory()
        self.haux = t.empty((), dtype=t.float32).pin_memory()
        self.dx_in = t.empty_like(self.x.detach())
        self.ddy = t.empty_like(self.dy)
        self.h2d = 2 * self.hx.numel() * 2
        self.d2h = 2 * self.hx.numel() * 2 + 4

    def e2e_step(self):
        t = self.torch
        self.dx_in.copy_(self.hx, non_blocking=True)
        self.ddy.copy_(self.hdy, non_blocking=True)
        x = self.dx_in.requires_grad_()
        self._zero()
        out, aux = self.layer(x)
        t.autograd.backward([out, aux], [self.ddy, self.one])
        self.hout.copy_(out.detach(), non_blocking=True)
        self.hdx.copy_(x.grad, non_blocking=True)
        self.haux.copy_(aux.detach(), non_blocking=True)
        x.grad = None
        x.requires_grad_(False)

    def units_to_value(self, steps, ms):
        return self.T * steps / (ms * 1e-3)

    def port_baseline(self, seconds: float):
        from oracle import moe as omoe
        from oracle.bf16 import round_bf16
        threads = cpu_threads()
        T = 256
        rng = np.random.default_rng(0)
        x = round_bf16(rng.standard_normal((T, self.H)).astype(np.float32))
        wg = (0.02 * rng.standard_normal((self.E, self.H))).astype(np.float32)
        wgu = round_bf16((0.02 * rng.standard_normal((self.E, 2 * self.F, self.H))).astype(np.float32))
        wd = round_bf16((0.02 * rng.standard_normal((self.E, self.H, self.F))).astype(np.float32))
        dy = round_bf16(rng.standard_normal((T, self.H)).astype(np.float32))
        t0 = time.perf_counter()
        n = 0
        while True:
            logits = omoe.router_logits(x, wg)
            fwd = omoe.moe_forward(x, logits, wgu, wd, self.K, self.E / self.K, 0.01, "bf16")
            omoe.moe_layer_backward_full(dy, fwd, x, wg, wgu, wd, 0.01, "bf16")
            n += 1
            if time.perf_counter() - t0 >= seconds:
                break
        dt = time.perf_counter() - t0
        return {"value": T * n / dt, "unit": self.unit, "cores": threads, "kind": "port",
                "sample": f"{T} of {self.T} tokens per pass (full expert weights), {n} passes in {dt:.1f} s "
                          f"(numpy oracle, BLAS on {threads} threads)"}


    def reference_pass(self, mods, torch):
        T = 512
        torch.manual_seed(0)
        layer = mods["moe"].MoELayer(self.H, self.F, self.E, num_layers=2, top_k=self.K,
                                     capacity_factor=self.E / self.K).bfloat16()
        x = torch.randn(1, T, self.H).bfloat16().requires_grad_()
        dy = torch.randn(1, T, self.H).bfloat16()

        def fn():
            layer.zero_grad(set_to_none=True)
            x.grad = None
            out, aux = layer(x)
            torch.autograd.backward([out, aux], [dy, torch.ones_like(aux)])

        return fn, T, f"{T} of {self.T} tokens per pass (all 8 experts, no capacity drop, bf16)"


class FFNWorkload(Workload):
    """Dense SwiGLU FFN (ffn.py:37-45) of a 7B-shaped block on the expert GEMMs (one expert, no routing)."""
    name = "ffn"
    metric = "swiglu_ffn_fwd_bwd_tokens_per_s"
    unit = "tokens/s"
    T, H, F = 16384, 4096, 11008

    def flops_per_step(self) -> int:
        return 18 * self.T * self.H * self.F  # 3 GEMMs forward (4HF + 2HF per token), twice that backward

    def config(self):
        return {"workload": "dense SwiGLU FFN fwd+bwd, 16384 tokens, hidden 4096, ffn 11008, bf16",
                "per_rank": "full workload per GPU (replicas)", "l2": "inputs larger than L2"}

    def setup(self):
        t = self.torch
        from ats_v2_b200.ffn import SwiGLU
        t.manual_seed(3000 + self.rank)
        with t.device("cuda"):
            self.m = SwiGLU(self.H, self.F)
        with t.no_grad():
            self.m.gate_up_proj.weight.normal_(0, 0.02)
            self.m.down_proj.weight.normal_(0, 0.02)
        self.m.bfloat16()
        g = t.Generator(device="cuda").manual_seed(self.rank)
        self.x = t.randn(4, self.T // 4, self.H, device="cuda", generator=g).bfloat16().requires_grad_()
        self.dy = t.randn(4, self.T // 4, self.H, device="cuda", generator=g).bfloat16()

    def step(self, evs):
        for p in self.m.parameters():
            p.grad = None
        self.x.grad = None
        if evs:
            evs[0].record()
        self.m(self.x).backward(self.dy)
        if evs:
            evs[1].record()

    def dominant(self):
        return {"kernel": "dense SwiGLU GEMMs (whole FFN fwd+bwd timed)", "flops": self.flops_per_step(),
                "bound": "tensor", "traffic": (14244.6 + 2283.7) * 1e6,
                "traffic_source": "profiles/ffn_gemms_16384tok_h4096_f11008_bf16.md: DRAM read+write of the six "
                                  "GEMM launches of one step (ncu, cold caches)"}

    def e2e_setup(self):
        t = self.torch
        self.hx = self.x.detach().cpu().pin_memory()
        self.hdy = self.dy.cpu().pin_memory()
        self.hdx = t.empty_like(self.hx).pin_memory()
        self.hout = t.empty_like(self.hx).pin_memory()
        self.dx_in = t.empty_like(self.x.detach())
        self.ddy = t.empty_like(self.dy)
        self.h2d = 2 * self.hx.numel() * 2
        self.d2h = 2 * self.hx.numel() * 2

    def e2e_step(self):
        self.dx_in.copy_(self.hx, non_blocking=True)
        self.ddy.copy_(self.hdy, non_blocking=True)
        x = self.dx_in.requires_grad_()
        for p in self.m.parameters():
            p.grad = None
        out = self.m(x)
        out.backward(self.ddy)
        self.hout.copy_(out.detach(), non_blocking=True)
        self.hdx.copy_(x.grad, non_blocking=True)
        x.grad = None
        x.requires_grad_(False)

    def units_to_value(self, steps, ms):
        return self.T * steps / (ms * 1e-3)

    def port_baseline(self, seconds: float):
        from oracle import moe as omoe
        from oracle.bf16 import round_bf16
        threads = cpu_threads()
        T = 256
        rng = np.random.default_rng(0)
        x = round_bf16(rng.standard_normal((T, self.H)).astype(np.float32))
        wgu = round_bf16((0.02 * rng.standard_normal((2 * self.F, self.H))).astype(np.float32))
        wd = round_bf16((0.02 * rng.standard_normal((self.H, self.F))).astype(np.float32))
        t0 = time.perf_counter()
        n = 0
        while True:
            omoe.expert_fwd(x, wgu, wd, "bf16")
            n += 1
            if time.perf_counter() - t0 >= seconds:
                break
        dt = time.perf_counter() - t0
        # the backward costs twice the forward's GEMMs; count a pass as forward + backward
        return {"value": T * n / dt / 3.0, "unit": self.unit, "cores": threads, "kind": "port",
                "sample": f"{T} tokens, forward only ({n} passes in {dt:.1f} s), scaled by 1/3 for the backward's "
                          f"two GEMMs per forward GEMM (numpy oracle, BLAS on {threads} threads)"}


    def reference_pass(self, mods, torch):
        T = 256
        torch.manual_seed(0)
        m = mods["ffn"].SwiGLU(self.H, self.F).bfloat16()
        x = torch.randn(T, self.H).bfloat16().requires_grad_()
        dy = torch.randn(T, self.H).bfloat16()

        def fn():
            m.zero_grad(set_to_none=True)
            x.grad = None
            m(x).backward(dy)

        return fn, T, f"{T} of {self.T} tokens per pass (bf16)"


class MLAWorkload(Workload):
    """MLA KV decompression (mla_triton.py:122-151) of a 7B-shaped block with MLA on: latent
    hidden/4 = 1024 (mla_compression_ratio 0.25), k and v each 32 heads x 128."""
    name = "mla"
    metric = "mla_kv_decompress_fwd_bwd_tokens_per_s"
    unit = "tokens/s"
    T, L, O = 16384, 1024, 4096

    def flops_per_step(self) -> int:
        return 12 * self.T * self.O * self.L  # forward 2*T*(2*O)*L, backward twice that

    def config(self):
        return {"workload": "MLA KV decompression fwd+bwd, 16384 tokens, latent 1024, k and v 4096 each, bf16",
                "per_rank": "full workload per GPU (replicas)", "l2": "outputs larger than L2"}

    def setup(self):
        t = self.torch
        g = t.Generator(device="cuda").manual_seed(4000 + self.rank)
        self.c = t.randn(4, self.T // 4, self.L, device="cuda", generator=g).bfloat16().requires_grad_()
        self.w_uk = (0.02 * t.randn(self.O, self.L, device="cuda", generator=g)).bfloat16().requires_grad_()
        self.w_uv = (0.02 * t.randn(self.O, self.L, device="cuda", generator=g)).bfloat16().requires_grad_()
        self.dk = t.randn(4, self.T // 4, self.O, device="cuda", generator=g).bfloat16()
        self.dv = t.randn(4, self.T // 4, self.O, device="cuda", generator=g).bfloat16()

    def _run(self, c, dk, dv):
        from ats_v2_b200.mla_fused import fused_mla_kv_decompress
        self.w_uk.grad = None
        self.w_uv.grad = None
        k, v = fused_mla_kv_decompress(c, self.w_uk, self.w_uv)
        self.torch.autograd.backward([k, v], [dk, dv])
        return k, v

    def step(self, evs):
        self.c.grad = None
        if evs:
            evs[0].record()
        self._run(self.c, self.dk, self.dv)
        if evs:
            evs[1].record()

    def dominant(self):
        return {"kernel": "MLA KV decompression GEMMs (forward, dgrad, weight gradient; whole fwd+bwd timed)",
                "flops": self.flops_per_step(), "bound": "tensor"}

    def e2e_setup(self):
        t = self.torch
        self.hc = self.c.detach().cpu().pin_memory()
        self.hdk = self.dk.cpu().pin_memory()
        self.hdv = self.dv.cpu().pin_memory()
        self.hk = t.empty_like(self.hdk).pin_memory()
        self.hv = t.empty_like(self.hdv).pin_memory()
        self.hdc = t.empty_like(self.hc).pin_memory()
        self.c_in = t.empty_like(self.c.detach())
        self.dk_in = t.empty_like(self.dk)
        self.dv_in = t.empty_like(self.dv)
        self.h2d = 2 * (self.hc.numel() + self.hdk.numel() + self.hdv.numel())
        self.d2h = 2 * (self.hk.numel() + self.hv.numel() + self.hc.numel())

    def e2e_step(self):
        self.c_in.copy_(self.hc, non_blocking=True)
        self.dk_in.copy_(self.hdk, non_blocking=True)
        self.dv_in.copy_(self.hdv, non_blocking=True)
        c = self.c_in.requires_grad_()
        k, v = self._run(c, self.dk_in, self.dv_in)
        self.hk.copy_(k.detach(), non_blocking=True)
        self.hv.copy_(v.detach(), non_blocking=True)
        self.hdc.copy_(c.grad, non_blocking=True)
        c.grad = None
        c.requires_grad_(False)

    def units_to_value(self, steps, ms):
        return self.T * steps / (ms * 1e-3)

    def port_baseline(self, seconds: float):
        from oracle import mla as omla
        from oracle.bf16 import round_bf16
        threads = cpu_threads()
        T = 512
        rng = np.random.default_rng(0)
        c = round_bf16(rng.standard_normal((T, self.L)).astype(np.float32))
        w_uk = round_bf16((0.02 * rng.standard_normal((self.O, self.L))).astype(np.float32))
        w_uv = round_bf16((0.02 * rng.standard_normal((self.O, self.L))).astype(np.float32))
        t0 = time.perf_counter()
        n = 0
        while True:
            omla.kv_decompress(c, w_uk, w_uv, "bf16")
            n += 1
            if time.perf_counter() - t0 >= seconds:
                break
        dt = time.perf_counter() - t0
        return {"value": T * n / dt / 3.0, "unit": self.unit, "cores": threads, "kind": "port",
                "sample": f"{T} tokens, forward only ({n} passes in {dt:.1f} s), scaled by 1/3 for the backward's "
                          f"two GEMMs per forward GEMM (numpy oracle, float64 BLAS on {threads} threads)"}


    def reference_pass(self, mods, torch):
        T = 1024
        g = torch.Generator().manual_seed(0)
        c = torch.randn(T, self.L, generator=g).bfloat16().requires_grad_()
        w_uk = (0.02 * torch.randn(self.O, self.L, generator=g)).bfloat16().requires_grad_()
        w_uv = (0.02 * torch.randn(self.O, self.L, generator=g)).bfloat16().requires_grad_()
        dk = torch.randn(T, self.O, generator=g).bfloat16()
        dv = torch.randn(T, self.O, generator=g).bfloat16()

        def fn():
            for t in (c, w_uk, w_uv):
                t.grad = None
            k, v = mods["mla_triton"].fused_mla_kv_decompress(c, w_uk, w_uv)
            torch.autograd.backward([k, v], [dk, dv])

        return fn, T, f"{T} of {self.T} tokens per pass (bf16)"


def zipf_bias(E: int, s_exp: float = 1.1, seed: int = 1):
    """Per-expert router-logit bias log(p_pi(e)), p_r ~ r^-s over ranks r=1..E,
    pi a fixed permutation (generator seed 1), mean-centred."""
    import torch
    p = torch.arange(1, E + 1, dtype=torch.float64) ** (-s_exp)
    p = p / p.sum()
    perm = torch.randperm(E, generator=torch.Generator().manual_seed(seed))
    b = torch.log(p[perm])
    return (b - b.mean()).float()


class MoEEPWorkload(Workload):
    name = "moe_ep"
    metric = "moe_ep_layer_fwd_bwd_tokens_per_s"
    unit = "tokens/s"
    T, H, F, E, K, CF = 32768, 4096, 1408, 64, 2, 1.25
    # row exchange: kernels store the kept rows into the expert ranks' mapped buffers and load the
    # results back, with the split sizes never on the host; in the backward the returning input
    # gradients move on 16 SMs while the weight-gradient GEMMs run on the rest (--ep-exchange peer:
    # copy-engine copies planned on the host, in overlapped parts).  At 2 GPUs this measured 4.47 ms a
    # step against 4.72 ms without the backward overlap, and 4.81 / 5.26 ms with the forward split
    # into 2 / 4 overlapped expert parts (the SM limit and the smaller parts cost the GEMMs more than
    # the hidden transfer saves).
    EXCHANGE, PARTS, COMM_SMS = "device", 1, 16

    def parts(self):
        return self.PARTS if self.world > 1 else 1

    def exchange_text(self):
        if self.EXCHANGE == "device":
            how = ("kernels store the kept rows into the expert ranks' IPC-mapped buffers over NVLink and load "
                   "the results back; split sizes stay on the device")
        elif self.EXCHANGE == "peer":
            how = "copy-engine copies of the kept rows into the peers' IPC-mapped buffers over NVLink"
        elif self.EXCHANGE == "packed":
            how = "NCCL all-to-all of the kept rows (variable splits)"
        else:
            how = "NCCL all-to-all of the capacity slots"
        if self.parts() > 1:
            how += f", in {self.parts()} expert parts overlapped with the expert GEMMs"
            if self.COMM_SMS:
                how += f" (GEMMs leave {self.COMM_SMS} SMs free)"
        if self.EXCHANGE == "device" and self.COMM_SMS:
            how += (f"; the backward's returning input gradients move on {self.COMM_SMS} SMs beside the "
                    "weight-gradient GEMMs")
        return how

    def config(self):
        return {"workload": "expert-parallel MoE layer fwd+bwd, 32768 tokens per GPU, hidden 4096, 64 experts "
                            "top-2, ffn 1408, capacity factor 1.25, Zipf(1.1) router-logit bias, bf16, fp32 router",
                "experts_per_gpu": self.E // self.world,
                "exchange": self.exchange_text() if self.world > 1 else "none (all experts local)",
                "expert_placement": "balanced by the rows each expert received on a calibration forward "
                                    "(ExpertParallelMoE.rebalance)",
                "per_rank": "32768 tokens per GPU (weak scaling)", "l2": "inputs larger than L2"}

    def setup(self):
        t = self.torch
        from ats_v2_b200.ep import ExpertParallelMoE
        t.manual_seed(2000 + self.rank)
        with t.device("cuda"):
            layer = ExpertParallelMoE(self.H, self.F, self.E, num_layers=2, top_k=self.K, capacity_factor=self.CF,
                                      exchange=self.EXCHANGE, overlap_parts=self.parts(), comm_sms=self.COMM_SMS)
        with t.no_grad():
            # the router weight is replicated: every rank draws the same one
            layer.gate.weight.copy_(0.02 * t.randn(layer.gate.weight.shape, generator=t.Generator().manual_seed(7)))
            for ex in layer.experts:
                ex.gate_up_proj.weight.normal_(0, 0.02)
                ex.down_proj.weight.normal_(0, 0.02)
        self.layer = layer
        self.layer.experts.to(t.bfloat16)
        self.bias = zipf_bias(self.E).cuda()
        g = t.Generator(device="cuda").manual_seed(self.rank)
        self.x = t.randn(1, self.T, self.H, device="cuda", generator=g).bfloat16().requires_grad_()
        self.dy = t.randn(1, self.T, self.H, device="cuda", generator=g).bfloat16()
        self.one = t.ones((), device="cuda")
        # expert placement: rows each expert receives on a calibration forward (kept counts rounded up to
        # 128, summed over the ranks), experts spread so every rank gets about the same; one rank: no change
        from ats_v2_b200.moe import capacity_for
        with t.no_grad():
            self.layer(self.x.detach(), logit_bias=self.bias)
        cap = capacity_for(self.T, self.K, self.E, self.CF)
        load = ((self.layer.last_counts.clamp(max=cap) + 127) // 128 * 128).to(t.float64)
        if self.world > 1:
            import torch.distributed as tdist
            tdist.all_reduce(load)
        self.perm = self.layer.rebalance(load.cpu())
        self.bias = self.bias[self.perm.cuda()]
        self.load_max_over_mean = float(self._rank_loads(load.cpu()).max() / self._rank_loads(load.cpu()).mean())

    def _rank_loads(self, load):
        el = self.E // self.world
        return load[self.perm].view(self.world, el).sum(1)

    def _zero(self):
        for p in self.layer.parameters():
            p.grad = None

    def step(self, evs):
        t = self.torch
        self._zero()
        self.x.grad = None
        if evs:
            evs[0].record()
        out, aux = self.layer(self.x, logit_bias=self.bias)
        t.autograd.backward([out, aux], [self.dy, self.one])
        if evs:
            evs[1].record()

    def phases(self):
        """Device time of each phase of one more step (device exchange, more than one GPU): routing, the
        exchange each way (waits for the slowest rank included), the expert GEMMs, the combine and the router
        backward; and the exchange's share of the step."""
        if self.world == 1 or self.EXCHANGE != "device":
            return None
        from ats_v2_b200 import ep
        t = self.torch
        t.cuda.synchronize()
        ep.PHASE_EVENTS = []
        try:
            self.step(None)
            t.cuda.synchronize()
            evs = ep.PHASE_EVENTS
        finally:
            ep.PHASE_EVENTS = None
        out = {}
        for (_, a), (name, b) in zip(evs, evs[1:]):
            if name != "bwd_start":  # from the forward's end to the backward's start: autograd, not the layer
                out[name] = out.get(name, 0.0) + a.elapsed_time(b)
        total = sum(out.values())
        ex = sum(v for k, v in out.items() if k.startswith("exchange"))
        out["exchange_share"] = ex / total if total else None
        return out

    def kept_rows(self) -> int:
        """Expert rows computed per GPU: kept rows of all ranks / ranks."""
        from ats_v2_b200.moe import capacity_for
        t = self.torch
        cap = capacity_for(self.T, self.K, self.E, self.CF)
        kept = self.layer.last_counts.clamp(max=cap).sum().to(t.float64).reshape(1)
        if self.world > 1:
            import torch.distributed as tdist
            tdist.all_reduce(kept)
        return int(round(float(kept.item()) / self.world))

    def dominant(self):
        rows = self.kept_rows()
        return {"kernel": "whole expert-parallel layer fwd+bwd (expert GEMMs 18*rows*H*F flops)",
                "flops": 18 * rows * self.H * self.F, "bound": "tensor", "kept_rows": rows,
                "rank_rows_max_over_mean": round(self.load_max_over_mean, 4)}

    def e2e_setup(self):
        t = self.torch
        self.hx = self.x.detach().cpu().pin_memory()
        self.hdy = self.dy.cpu().pin_memory()
        self.hout = t.empty_like(self.hx).pin_memory()
        self.hdx = t.empty_like(self.hx).pin_memory()
        self.haux = t.empty((), dtype=t.float32).pin_memory()
        self.dx_in = t.empty_like(self.x.detach())
        self.ddy = t.empty_like(self.dy)
        self.h2d = 2 * self.hx.numel() * 2
        self.d2h = 2 * self.hx.numel() * 2 + 4

    def e2e_step(self):
        t = self.torch
        self.dx_in.copy_(self.hx, non_blocking=True)
        self.ddy.copy_(self.hdy, non_blocking=True)
        x = self.dx_in.requires_grad_()
        self._zero()
        out, aux = self.layer(x, logit_bias=self.bias)
        t.autograd.backward([out, aux], [self.ddy, self.one])
        self.hout.copy_(out.detach(), non_blocking=True)
        self.hdx.copy_(x.grad, non_blocking=True)
        self.haux.copy_(aux.detach(), non_blocking=True)
        x.grad = None
        x.requires_grad_(False)

    def units_to_value(self, steps, ms):
        return self.T * steps / (ms * 1e-3)

    def reference_pass(self, mods, torch):
        # the reference's single-process layer with all 64 experts (it has no CPU expert parallelism), the same
        # Zipf skew added to its router logits (as the gate's bias), so the same share of rows is kept
        T = 1024
        torch.manual_seed(0)
        layer = mods["moe"].MoELayer(self.H, self.F, self.E, num_layers=2, top_k=self.K,
                                     capacity_factor=self.CF).bfloat16()
        layer.moe.gate.bias = torch.nn.Parameter(zipf_bias(self.E).bfloat16(), requires_grad=False)
        x = torch.randn(1, T, self.H).bfloat16().requires_grad_()
        dy = torch.randn(1, T, self.H).bfloat16()

        def fn():
            layer.zero_grad(set_to_none=True)
            x.grad = None
            out, aux = layer(x)
            torch.autograd.backward([out, aux], [dy, torch.ones_like(aux)])

        return (fn, T, f"{T} of {self.T} tokens per pass, all {self.E} experts in one process, capacity from the "
                       f"{T} tokens, Zipf(1.1) logit bias, bf16")

    def port_baseline(self, seconds: float):
        # a token's cost is its k experts' FFNs whatever E is: time 256 tokens on 8 of the experts
        from oracle import moe as omoe
        from oracle.bf16 import round_bf16
        threads = cpu_threads()
        T, E = 256, 8
        rng = np.random.default_rng(0)
        x = round_bf16(rng.standard_normal((T, self.H)).astype(np.float32))
        wg = (0.02 * rng.standard_normal((E, self.H))).astype(np.float32)
        wgu = round_bf16((0.02 * rng.standard_normal((E, 2 * self.F, self.H))).astype(np.float32))
        wd = round_bf16((0.02 * rng.standard_normal((E, self.H, self.F))).astype(np.float32))
        dy = round_bf16(rng.standard_normal((T, self.H)).astype(np.float32))
        t0 = time.perf_counter()
        n = 0
        while True:
            logits = omoe.router_logits(x, wg)
            fwd = omoe.moe_forward(x, logits, wgu, wd, self.K, self.CF, 0.01, "bf16")
            omoe.moe_layer_backward_full(dy, fwd, x, wg, wgu, wd, 0.01, "bf16")
            n += 1
            if time.perf_counter() - t0 >= seconds:
                break
        dt = time.perf_counter() - t0
        return {"value": T * n / dt, "unit": self.unit, "cores": threads, "kind": "port",
                "sample": f"{T} tokens per pass routed over 8 of the experts (a token's cost is its top-2 "
                          f"experts' FFNs), {n} passes in {dt:.1f} s (numpy oracle, BLAS on {threads} threads)"}


# the expert-parallel layer is the headline: it is the one configuration measured at 1, 2, 4 and 8 GPUs;
# the extras follow in this order, the north-star configurations last
WORKLOADS = {"moe_ep": MoEEPWorkload, "ffn": FFNWorkload, "mla": MLAWorkload, "rmsnorm": RMSNormWorkload,
             "rope": RopeWorkload, "moe": MoEWorkload}


# ---------------------------------------------------------------- timing
def enqueue_seconds(torch, fn) -> float:
    """Host time to enqueue one step while the GPU is held busy."""
    torch.cuda.synchronize()
    torch.cuda._sleep(int(0.3 * 1.9e9))
    t0 = time.perf_counter()
    fn(None)
    fn(None)
    dt = (time.perf_counter() - t0) / 2
    torch.cuda.synchronize()
    return dt


def timed(torch, dist, fn, steps: int, warmup: int, probe: bool = False, prefill_s: float = 0.0):
    """Run warmup then `steps` calls of fn(evs); returns (max-over-ranks ms,
    mean probe ms).  With probe=True each timed call gets its own CUDA event
    pair, recorded on the launching (current) stream around the probed call.
    prefill_s > 0 holds the GPU in a sleep kernel queued before the start
    event for that long, so all steps are queued before the first one runs and
    the events measure device time without host launch gaps."""
    for _ in range(warmup):
        fn(None)
    torch.cuda.synchronize()
    if dist is not None:
        dist.barrier()
    torch.cuda.synchronize()
    pairs = [(torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True))
             for _ in range(steps)] if probe else [None] * steps
    s, e = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    if prefill_s > 0:
        torch.cuda._sleep(int(prefill_s * 1.9e9))
    s.record()
    for i in range(steps):
        fn(pairs[i])
    e.record()
    torch.cuda.synchronize()
    if dist is not None:
        dist.barrier()
    torch.cuda.synchronize()
    ms = s.elapsed_time(e)
    pms = statistics.mean(a.elapsed_time(b) for a, b in pairs) if probe else None
    if dist is not None:
        t = torch.tensor([ms], device="cuda", dtype=torch.float64)
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
        ms = float(t.item())
    return ms, pms


def measure(torch, dist, wl: Workload, steps: int, warmup: int, world: int, with_cpu: bool, cpu_seconds: float,
            gpu_index: int, lib) -> dict:
    wl.setup()
    for _ in range(warmup):
        wl.step(None)
    torch.cuda.synchronize()
    enq = enqueue_seconds(torch, wl.step)
    prefill = min(3.0, 1.5 * enq * steps + 0.005)
    with ClockSampler(gpu_index) as clk:
        launches0 = lib.ats_kernel_launches()
        ms, kms = timed(torch, dist, wl.step, steps, 0, probe=True, prefill_s=prefill)
        launches = lib.ats_kernel_launches() - launches0
    clocks = clk.summary
    value = wl.units_to_value(steps, ms) * world
    cfg = dict(wl.config())
    cfg["timing"] = (f"device time of {steps} queued steps (launch queue pre-filled: host enqueue "
                     f"{enq * 1e3:.3f} ms/step); e2e is timed without pre-fill")
    res = {"metric": wl.metric, "value": value, "unit": wl.unit, "ms_per_step": ms / steps,
           "higher_is_better": True, "dtype": wl.dtype, "config": cfg, "clocks": clocks,
           "gpu_launches": int(launches), "host_enqueue_ms_per_step": enq * 1e3}
    dom = wl.dominant()
    if kms:
        if dom["bound"] == "hbm":
            ach = dom["bytes"] / (kms * 1e-3) / 1e9
            peak = wl.peaks["hbm_gbs"]
            res["roofline"] = {"bound": "hbm", "kernel": dom["kernel"], "achieved": ach, "peak": peak,
                               "unit": "GB/s", "frac": ach / peak, "peak_source": wl.peaks_kind,
                               "traffic": dom.get("traffic"), "algorithmic_bytes": dom["bytes"], "kernel_ms": kms}
        else:
            ach = dom["flops"] / (kms * 1e-3) / 1e12
            # the burst peak for a timed region under a second, the sustained (power-capped) one beyond
            sustained = ms >= 1000.0 and "bf16_tflops_sustained" in wl.peaks
            peak = wl.peaks["bf16_tflops_sustained"] if sustained else wl.peaks["bf16_tflops"]
            res["roofline"] = {"bound": "tensor", "kernel": dom["kernel"], "achieved": ach, "peak": peak,
                               "unit": "TFLOP/s", "frac": ach / peak,
                               "peak_source": wl.peaks_kind + (" sustained" if sustained else " burst"),
                               "traffic": dom.get("traffic"), "algorithmic_flops": dom["flops"], "kernel_ms": kms}
            for key in ("kept_rows", "rank_rows_max_over_mean"):
                if key in dom:
                    res["roofline"][key] = dom[key]
        if "traffic_source" in dom:
            res["roofline"]["traffic_source"] = dom["traffic_source"]
    phases = wl.phases() if hasattr(wl, "phases") else None
    if phases:
        res["phases_ms"] = phases
    # end to end through the public module with host buffers
    wl.e2e_setup()
    e2e_steps = max(3, min(steps, 10))
    ems, _ = timed(torch, dist, lambda evs: wl.e2e_step(), e2e_steps, 2)
    res["e2e"] = {"value": wl.units_to_value(e2e_steps, ems) * world, "unit": wl.unit,
                  "h2d_bytes_per_step": int(wl.h2d), "d2h_bytes_per_step": int(wl.d2h),
                  "ms_per_step": ems / e2e_steps}
    if with_cpu:
        try:
            res["cpu_baseline"] = wl.cpu_baseline(cpu_seconds)
        except Exception as exc:  # a baseline failure must not hide the GPU number
            res["cpu_baseline"] = {"error": repr(exc)[:300]}
    return res


def _r(v, n=4):
    return float(f"{v:.{n}g}") if isinstance(v, (int, float)) else v


def compact(res: dict) -> dict:
    """An extra workload's numbers only (its configuration and sampling are
    described in the repository's design notes), so that every extra fits the
    tail of the output that is kept."""
    out = {"metric": res["metric"], "value": _r(res["value"]), "unit": res["unit"],
           "ms_per_step": _r(res["ms_per_step"])}
    rf = res.get("roofline")
    if rf:
        out["roofline"] = {k: _r(rf[k]) for k in ("bound", "frac", "achieved", "peak", "unit", "kernel_ms", "traffic")
                           if k in rf}
        out["roofline"]["peak_source"] = rf.get("peak_source")
    if "phases_ms" in res:
        out["phases_ms"] = {k: _r(v, 3) for k, v in res["phases_ms"].items()}
    if "cpu_baseline" in res:
        cb = res["cpu_baseline"]
        out["cpu_baseline"] = {k: _r(cb[k]) for k in ("value", "kind", "cores", "error") if k in cb}
    out["e2e"] = {"value": _r(res["e2e"]["value"])}
    ck = res.get("clocks") or {}
    out["clocks"] = {"sm_mhz": ck.get("sm_mhz"), "reasons": ck.get("reasons")}
    out["gpu_launches"] = res.get("gpu_launches")
    return out


def main() -> int:
    ap = argparse.ArgumentParser(description="ats-v2 hot path benchmark on B200")
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=20)
    ap.add_argument("--warmup", type=int, default=5)
    ap.add_argument("--workload", default="moe_ep", choices=sorted(WORKLOADS))
    ap.add_argument("--impl", default="ours", choices=["ours", "reference"])
    ap.add_argument("--no-extras", action="store_true", help="only the selected workload")
    ap.add_argument("--cpu-seconds", type=float, default=8.0)
    ap.add_argument("--ep-exchange", default=None, choices=["device", "peer", "packed", "slots"],
                    help="row exchange of the expert-parallel workload")
    ap.add_argument("--ep-parts", type=int, default=None, help="expert parts of the expert-parallel exchange")
    ap.add_argument("--ep-comm-sms", type=int, default=None,
                    help="SMs the expert-parallel exchange keeps while it overlaps the expert GEMMs")
    ap.add_argument("--gemm-pairs", type=int, default=0, choices=[0, 1],
                    help="1: tensor-core GEMMs on CTA pairs (256-row tiles); 0: single CTAs (128-row tiles)")
    args = ap.parse_args()
    if args.ep_exchange:
        MoEEPWorkload.EXCHANGE = args.ep_exchange
    if args.ep_parts:
        MoEEPWorkload.PARTS = args.ep_parts
    if args.ep_comm_sms is not None:
        MoEEPWorkload.COMM_SMS = args.ep_comm_sms
    if args.warmup < 3 and args.impl == "ours":
        print("warning: fewer than 3 warm-up steps", file=sys.stderr)
    world, rank, local = dist_env()
    peaks, pk = load_peaks()

    if args.impl == "reference":
        if rank != 0:
            return 0
        return reference_arm(args, world, peaks, pk)

    import torch
    torch.cuda.set_device(local)
    dist = None
    if world > 1:
        import datetime

        import torch.distributed as tdist
        tdist.init_process_group("nccl", timeout=datetime.timedelta(seconds=120),
                                 device_id=torch.device("cuda", local))
        dist = tdist
    from ats_v2_b200 import _lib
    lib = _lib.load()
    _lib.call("ats_set_gemm_pairs", args.gemm_pairs)
    gpu_index = int(os.environ.get("CUDA_VISIBLE_DEVICES", str(local)).split(",")[local]) \
        if os.environ.get("CUDA_VISIBLE_DEVICES") else local
    main_wl = WORKLOADS[args.workload](torch, rank, world, peaks, pk)
    with_cpu = (world == 1 and rank == 0)
    res = measure(torch, dist, main_wl, args.steps, args.warmup, world, with_cpu, args.cpu_seconds, gpu_index, lib)
    line = {"metric": res["metric"], "value": res["value"], "unit": res["unit"], "n_gpus": world,
            "steps": args.steps, "warmup": args.warmup, "ms_per_step": res["ms_per_step"],
            "higher_is_better": True, "scaling": "weak", "vs_baseline": None, "dtype": res["dtype"],
            "data": "synthetic (seeded normal inputs of the config's shapes)", "config": res["config"],
            "e2e": res["e2e"], "roofline": res.get("roofline"), "clocks": res["clocks"],
            "gpu_launches": res["gpu_launches"]}
    if "cpu_baseline" in res:
        line["cpu_baseline"] = res["cpu_baseline"]
    if "phases_ms" in res:
        line["phases_ms"] = {k: _r(v, 3) for k, v in res["phases_ms"].items()}
    if not args.no_extras:
        extras = {}
        for name, cls in WORKLOADS.items():
            if name == args.workload:
                continue
            try:
                wl = cls(torch, rank, world, peaks, pk)
                extras[name] = compact(measure(torch, dist, wl, args.steps, args.warmup, world, with_cpu,
                                               args.cpu_seconds, gpu_index, lib))
                del wl
                torch.cuda.empty_cache()
            except Exception as exc:
                extras[name] = {"error": repr(exc)[:400]}
        line["extras"] = extras
    if rank == 0:
        print(json.dumps(line))
    if dist is not None:
        dist.barrier()
        dist.destroy_process_group()
    return 0


def reference_arm(args, world: int, peaks: dict, pk: str) -> int:
    """The reference's own CPU implementation of the workload -- its modules from
    baseline/_ref, torch on every host thread -- on the same metric and
    configuration (the numpy restatement of its algorithm when the reference is
    not installed).  Each step is a bounded sample of the workload."""
    wl = WORKLOADS[args.workload](None, 0, world, peaks, pk)
    per_step = max(1.0, min(6.0, 120.0 / max(1, args.steps + args.warmup)))
    mods = reference_modules()
    if mods is None:
        for _ in range(args.warmup):
            wl.port_baseline(per_step * 0.25)
        vals = [wl.port_baseline(per_step) for _ in range(args.steps)]
        base = dict(vals[-1])
        v = statistics.mean(x["value"] for x in vals)
    else:
        import torch
        threads = cpu_threads()
        torch.set_num_threads(threads)
        fn, units, sample = wl.reference_pass(mods, torch)
        for _ in range(args.warmup):
            fn()
        rates = []
        for _ in range(args.steps):
            n, dt = timed_passes(fn, per_step)
            rates.append(units * n / dt)
        v = statistics.mean(rates)
        base = {"unit": wl.unit, "cores": threads, "kind": "reference",
                "sample": f"{sample}; each of the {args.steps} steps runs passes for {per_step:.1f} s (the "
                          f"reference's modules from baseline/_ref, torch on CPU, {threads} threads)"}
    base["value"] = v
    line = {"impl": "reference", "metric": wl.metric, "value": v, "unit": wl.unit, "n_gpus": world,
            "steps": args.steps, "warmup": args.warmup, "higher_is_better": True, "scaling": "weak",
            "vs_baseline": None, "dtype": wl.dtype, "data": "synthetic (seeded normal inputs of the config's shapes)",
            "config": wl.config(), "cpu_baseline": base,
            "e2e": {"value": v, "unit": wl.unit, "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0}}
    print(json.dumps(line))
    return 0


if __name__ == "__main__":
    sys.exit(main())

"""Mixture-of-Experts layer on the sm_100a kernels -- mirror of ats/model/moe.py.

``MoELayer(hidden_size, intermediate_size, num_experts, num_layers, top_k=2,
capacity_factor=1.25, load_balancing_weight=0.01, ep_size=1, quantization)``
keeps the reference constructor (moe.py:167-230), attribute names
(``uses_deepspeed``, ``moe.gate``, ``moe.experts[i].gate_up_proj/down_proj``,
``moe.compute_routing``, ``last_expert_utilization``) and the forward
contract ``(output [B,S,H], aux_loss scalar)`` (moe.py:232-274), with the
semantics of the single-process fallback _PyTorchMoEFallback (moe.py:36-164):
softmax -> top-k -> renormalise, capacity ``max(1, int(cf*T*k/E))``, per expert
the first `capacity` tokens in ascending token order, SwiGLU experts, gate-
weighted combine in ascending expert order, Switch aux loss.

What changes is how it runs.  The router is float32 (logits from a float32
matmul of the tokens with the gate weight).  Everything after the logits is a
fixed sequence of device stages with no host synchronisation (the reference
synchronises once per expert in ``nonzero`` and once per expert in ``.item()``):
route+plan+permute, gather, grouped SwiGLU experts (tcgen05 tensor cores for
bf16), combine; the backward runs the adjoint stages.  The utilisation dict is
filled lazily from a device tensor the first time it is read.
"""

from __future__ import annotations

import math

import torch
import torch.nn.functional as F
from torch import nn

from ats_v2_b200 import _lib
from ats_v2_b200.ffn import SwiGLU, require_plain_weights

BASE_LINEAR_STD = 0.02


def residual_output_std(num_layers: int) -> float:
    """Depth-scaled std of residual-stream projections (ats/model/initialization.py:52-57)."""
    if num_layers <= 0:
        raise ValueError(f"num_layers must be positive, got {num_layers}.")
    return BASE_LINEAR_STD / math.sqrt(2 * num_layers)


def init_residual_projection(module: nn.Linear, num_layers: int) -> None:
    """N(0, residual_output_std) init, marked so a later blanket init skips it
    (ats/model/initialization.py:60-73)."""
    nn.init.normal_(module.weight, mean=0.0, std=residual_output_std(num_layers))
    if module.bias is not None:
        nn.init.zeros_(module.bias)
    module.weight._ats_residual_init = True  # type: ignore[attr-defined]


def capacity_for(num_tokens: int, top_k: int, num_experts: int, capacity_factor: float) -> int:
    """moe.py:103-105."""
    return max(1, int(capacity_factor * num_tokens * top_k / num_experts))


def stacked(params: list[torch.Tensor]) -> torch.Tensor:
    """Return an [E, ...] tensor whose slice e IS params[e]'s storage.

    If the parameters are not already consecutive views of one buffer (a fresh
    module, or one moved with .to()), they are copied into a new stacked
    buffer and each parameter is re-pointed at its slice, once."""
    p0 = params[0]
    E = len(params)
    n = p0.numel()
    d0 = p0.data
    ok = d0.is_contiguous() and all(
        p.data.is_contiguous() and p.dtype == p0.dtype and p.device == p0.device
        and p.data.untyped_storage().data_ptr() == d0.untyped_storage().data_ptr()
        and p.data.storage_offset() == d0.storage_offset() + e * n for e, p in enumerate(params))
    if ok:
        return torch.as_strided(d0, (E,) + tuple(p0.shape), (n,) + tuple(d0.stride()), d0.storage_offset())
    stack = torch.stack([p.data for p in params])
    for e, p in enumerate(params):
        p.data = stack[e]
    return stack


class LazyUtilization(dict):
    """dict[int, float] of per-expert utilisation, read from the device the
    first time any entry is accessed (no synchronisation inside forward)."""

    def __init__(self, t: torch.Tensor) -> None:
        super().__init__()
        self._t: torch.Tensor | None = t

    def _fill(self) -> None:
        if self._t is not None:
            t, self._t = self._t, None
            vals = t.tolist()
            dict.update(self, {i: float(v) for i, v in enumerate(vals)})
            if t.is_cuda:  # the host has waited for the device here anyway: report a wait that gave up
                with torch.cuda.device(t.device):
                    _lib.check_device_status("MoE layer")

    def __getitem__(self, key):
        self._fill()
        return dict.__getitem__(self, key)

    def __iter__(self):
        self._fill()
        return dict.__iter__(self)

    def __len__(self):
        self._fill()
        return dict.__len__(self)

    def __contains__(self, key):
        self._fill()
        return dict.__contains__(self, key)

    def __eq__(self, other):
        self._fill()
        return dict.__eq__(self, other)

    __hash__ = None  # type: ignore[assignment]

    def __repr__(self):
        self._fill()
        return dict.__repr__(self)

    def keys(self):
        self._fill()
        return dict.keys(self)

    def values(self):
        self._fill()
        return dict.values(self)

    def items(self):
        self._fill()
        return dict.items(self)

    def get(self, key, default=None):
        self._fill()
        return dict.get(self, key, default)


def router_forward(x2: torch.Tensor, gate_w: torch.Tensor, bias: torch.Tensor | None):
    """float32 router logits [T,E] = x2.float() @ gate_w.float().T (+ bias) and the
    router workspace (None when the tensor-core path does not cover the shape
    and a library GEMM computed them)."""
    T, H = x2.shape
    E = gate_w.shape[0]
    w32 = gate_w.detach().float().contiguous()
    b32 = bias.detach().float().contiguous() if bias is not None else None
    dt = _lib.dtype_code(x2.dtype)
    if _lib.query("ats_moe_router_supported", dt, T, H, E) == 1:
        wsb = _lib.query("ats_moe_router_workspace_bytes", T, H, E)
        rws = torch.empty(wsb, dtype=torch.uint8, device=x2.device)
        logits = torch.empty((T, E), dtype=torch.float32, device=x2.device)
        _lib.call("ats_moe_router_fwd", x2.data_ptr(), w32.data_ptr(), _lib.ptr(b32), logits.data_ptr(), T, H, E,
                  rws.data_ptr(), wsb, _lib.stream_of(x2))
        return logits, rws, w32
    logits = F.linear(x2.float(), w32)
    if b32 is not None:
        logits = logits + b32
    return logits, None, w32


class _MoEFn(torch.autograd.Function):
    """Device stages of the MoE layer on flattened tokens x2 [T,H].

    Inputs: x2, then either float32 logits [T,E] (gate_w None) or the router
    weight gate_w [E,H] (logits None; the router runs inside, and its
    gradient and its share of dx come out of the backward), an optional
    constant logit bias [E], meta=(E,k,C,lbw,F,layout), the two weight stacks,
    then the per-expert weights (only so autograd routes their gradients)."""

    @staticmethod
    def forward(ctx, x2, logits, gate_w, bias, meta, wgu_stack, wd_stack, *expert_weights):
        E, k, C, lbw, Fdim, L = meta
        T, H = x2.shape
        dev = x2.device
        dt = _lib.dtype_code(x2.dtype)
        st = _lib.stream_of(x2)
        rws = w32 = None
        if gate_w is not None:
            logits, rws, w32 = router_forward(x2, gate_w, bias)
        ws_bytes = _lib.query("ats_moe_workspace_bytes", T, E, k, C, L)
        max_rows = _lib.query("ats_moe_max_rows", T, E, k, C, L)
        ws = torch.empty(ws_bytes, dtype=torch.uint8, device=dev)
        gates = torch.empty((T, k), dtype=torch.float32, device=dev)
        idx = torch.empty((T, k), dtype=torch.int64, device=dev)
        aux = torch.empty((), dtype=torch.float32, device=dev)
        util = torch.empty(E, dtype=torch.float32, device=dev)
        counts = torch.empty(E, dtype=torch.int32, device=dev)
        _lib.call("ats_moe_route_plan", logits.data_ptr(), T, E, k, C, L, float(lbw), gates.data_ptr(),
                  idx.data_ptr(), aux.data_ptr(), util.data_ptr(), counts.data_ptr(), ws.data_ptr(), ws_bytes,
                  st)
        xp = torch.empty((max_rows, H), dtype=x2.dtype, device=dev)
        _lib.call("ats_moe_gather", x2.data_ptr(), xp.data_ptr(), dt, T, H, E, k, C, L, ws.data_ptr(), ws_bytes, st)
        h = torch.empty((max_rows, 2 * Fdim), dtype=x2.dtype, device=dev)
        a = torch.empty((max_rows, Fdim), dtype=x2.dtype, device=dev)
        y = torch.empty((max_rows, H), dtype=x2.dtype, device=dev)
        _lib.call("ats_moe_experts_fwd", xp.data_ptr(), wgu_stack.data_ptr(), wd_stack.data_ptr(), h.data_ptr(),
                  a.data_ptr(), y.data_ptr(), dt, T, E, k, C, L, H, Fdim, ws.data_ptr(), ws_bytes, st)
        out = torch.empty((T, H), dtype=x2.dtype, device=dev)
        _lib.call("ats_moe_combine", y.data_ptr(), out.data_ptr(), dt, T, H, E, k, C, L, ws.data_ptr(), ws_bytes, st)
        ctx.save_for_backward(logits, gates, idx, ws, xp, h, a, y, wgu_stack, wd_stack, x2, w32, rws)
        ctx.meta = (E, k, C, lbw, Fdim, L, T, H, ws_bytes, max_rows, gate_w is not None,
                    gate_w.dtype if gate_w is not None else None)
        ctx.mark_non_differentiable(util, counts, idx)
        return out, aux, util, counts, idx

    @staticmethod
    def backward(ctx, dout, daux, _dutil, _dcounts, _didx):
        logits, gates, idx, ws, xp, h, a, y, wgu_stack, wd_stack, x2, w32, rws = ctx.saved_tensors
        E, k, C, lbw, Fdim, L, T, H, ws_bytes, max_rows, has_router, gate_dtype = ctx.meta
        dev = xp.device
        dt = _lib.dtype_code(xp.dtype)
        st = _lib.stream_of(xp)
        if dout is None:
            dout = torch.zeros((T, H), dtype=xp.dtype, device=dev)
        dout = dout.to(xp.dtype).contiguous()
        dy = torch.empty((max_rows, H), dtype=xp.dtype, device=dev)
        dgate_row = torch.empty(max_rows, dtype=torch.float32, device=dev)
        _lib.call("ats_moe_combine_bwd", dout.data_ptr(), y.data_ptr(), dy.data_ptr(), dgate_row.data_ptr(), dt,
                  T, H, E, k, C, L, ws.data_ptr(), ws_bytes, st)
        dh = torch.empty((max_rows, 2 * Fdim), dtype=xp.dtype, device=dev)
        dxp = torch.empty((max_rows, H), dtype=xp.dtype, device=dev)
        dwgu = torch.empty_like(wgu_stack)
        dwd = torch.empty_like(wd_stack)
        _lib.call("ats_moe_experts_bwd", dy.data_ptr(), xp.data_ptr(), h.data_ptr(), a.data_ptr(),
                  wgu_stack.data_ptr(), wd_stack.data_ptr(), dh.data_ptr(), dxp.data_ptr(), dwgu.data_ptr(),
                  dwd.data_ptr(), dt, T, E, k, C, L, H, Fdim, ws.data_ptr(), ws_bytes, st)
        dlogits = torch.empty((T, E), dtype=torch.float32, device=dev)
        daux_t = daux.to(torch.float32).contiguous() if daux is not None else None
        _lib.call("ats_moe_route_bwd", logits.data_ptr(), gates.data_ptr(), idx.data_ptr(), dgate_row.data_ptr(),
                  _lib.ptr(daux_t), dlogits.data_ptr(), T, E, k, C, L, float(lbw), ws.data_ptr(), ws_bytes, st)
        grads = [dwgu[e] for e in range(E)] + [dwd[e] for e in range(E)]
        dx, dgate_w = router_backward(dlogits, x2, w32, rws, dxp, ws, ws_bytes, (T, E, k, C, L), has_router)
        if not has_router:
            return (dx, dlogits, None, None, None, None, None, *grads)
        return (dx, None, dgate_w.to(gate_dtype), None, None, None, None, *grads)


def router_weight_grad(dlogits, x2, w32, rws):
    """First stage of the tensor-core router backward: the router weight gradient
    (float32 [E, H]); the split gradient parts stay in ``rws`` for
    ``router_backward(..., dw=...)``.  It needs no expert result, so an
    expert-parallel backward runs it while rows are in flight."""
    T, H = x2.shape
    E = dlogits.shape[1]
    dw = torch.empty((E, H), dtype=torch.float32, device=x2.device)
    _lib.call("ats_moe_router_bwd_staged", dlogits.data_ptr(), x2.data_ptr(), w32.data_ptr(), None, None, 0, 1, 1,
              _lib.ATS_MOE_PACKED, None, dw.data_ptr(), T, H, E, rws.data_ptr(), rws.numel(), _lib.ATS_ROUTER_BWD_DW,
              _lib.stream_of(x2))
    return dw


def router_backward(dlogits, x2, w32, rws, dxp, ws, ws_bytes, plan, has_router, dw=None):
    """(dx, dgate_w): the token gradient (the permuted-row gradients summed per
    token, plus the router's share when the router ran inside) and the router
    weight gradient (float32, None without a router).  ``dw`` from
    ``router_weight_grad`` (same ``rws``) skips that stage here."""
    T, E, k, C, L = plan
    H = x2.shape[1]
    st = _lib.stream_of(x2)
    dt = _lib.dtype_code(x2.dtype)
    dx = torch.empty((T, H), dtype=x2.dtype, device=x2.device)
    if has_router and rws is not None:
        stages = _lib.ATS_ROUTER_BWD_DX
        if dw is None:
            dw = torch.empty((E, H), dtype=torch.float32, device=x2.device)
            stages = _lib.ATS_ROUTER_BWD_ALL
        _lib.call("ats_moe_router_bwd_staged", dlogits.data_ptr(), x2.data_ptr(), w32.data_ptr(), dxp.data_ptr(),
                  ws.data_ptr(), ws_bytes, k, C, L, dx.data_ptr(), dw.data_ptr(), T, H, E, rws.data_ptr(),
                  rws.numel(), stages, st)
        return dx, dw
    _lib.call("ats_moe_scatter_grad", dxp.data_ptr(), dx.data_ptr(), dt, T, H, E, k, C, L, ws.data_ptr(), ws_bytes,
              st)
    if not has_router:
        return dx, None
    # library-GEMM router (shapes the tensor-core router does not cover): the two bf16 token
    # gradients add as autograd would add them
    dx = dx + (dlogits @ w32).to(x2.dtype)
    return dx, dlogits.t() @ x2.float()


def moe_apply(x2: torch.Tensor, logits: torch.Tensor | None, wgu: list[torch.Tensor], wd: list[torch.Tensor],
              top_k: int, capacity: int, lbw: float, layout: int = _lib.ATS_MOE_PACKED,
              gate_w: torch.Tensor | None = None, bias: torch.Tensor | None = None):
    """Run the device MoE stages; returns (out [T,H], aux (0-dim), util [E], counts [E], idx [T,k]).

    Either float32 logits or the router weight gate_w (the router then runs
    inside, on the tensor cores for bf16 tokens)."""
    E = len(wgu)
    Fdim = wgu[0].shape[0] // 2
    wgu_stack = stacked(wgu)
    wd_stack = stacked(wd)
    if gate_w is None:
        logits = logits.float().contiguous()
    return _MoEFn.apply(x2.contiguous(), logits, gate_w, bias, (E, top_k, capacity, lbw, Fdim, layout), wgu_stack,
                        wd_stack, *wgu, *wd)


class _DenseSwiGLUFn(torch.autograd.Function):
    """SwiGLU FFN on the tensor-core GEMMs as one expert over the token rows
    (no routing, no gather or combine pass)."""

    @staticmethod
    def forward(ctx, x2, w_gate_up, w_down):
        T, H = x2.shape
        Fdim = w_down.shape[1]
        dev = x2.device
        dt = _lib.dtype_code(x2.dtype)
        st = _lib.stream_of(x2)
        R = _lib.query("ats_swiglu_rows", T)
        wsb = _lib.query("ats_swiglu_workspace_bytes")
        ws = torch.empty(wsb, dtype=torch.uint8, device=dev)
        wgu, wd = w_gate_up.contiguous(), w_down.contiguous()
        h = torch.empty((R, 2 * Fdim), dtype=x2.dtype, device=dev)
        a = torch.empty((R, Fdim), dtype=x2.dtype, device=dev)
        y = torch.empty((T, H), dtype=x2.dtype, device=dev)
        _lib.call("ats_swiglu_fwd", x2.data_ptr(), wgu.data_ptr(), wd.data_ptr(), h.data_ptr(), a.data_ptr(),
                  y.data_ptr(), dt, T, H, Fdim, ws.data_ptr(), wsb, st)
        ctx.save_for_backward(x2, h, a, wgu, wd, ws)
        return y

    @staticmethod
    def backward(ctx, dy):
        x2, h, a, wgu, wd, ws = ctx.saved_tensors
        T, H = x2.shape
        Fdim = wd.shape[1]
        dt = _lib.dtype_code(x2.dtype)
        st = _lib.stream_of(x2)
        dy = dy.to(x2.dtype).contiguous()
        dh = torch.empty_like(h)
        dx = torch.empty_like(x2)
        dwgu = torch.empty_like(wgu)
        dwd = torch.empty_like(wd)
        _lib.call("ats_swiglu_bwd", dy.data_ptr(), x2.data_ptr(), h.data_ptr(), a.data_ptr(), wgu.data_ptr(),
                  wd.data_ptr(), dh.data_ptr(), dx.data_ptr(), dwgu.data_ptr(), dwd.data_ptr(), dt, T, H, Fdim,
                  ws.data_ptr(), ws.numel(), st)
        return dx, dwgu, dwd


def dense_swiglu(x: torch.Tensor, w_gate_up: torch.Tensor, w_down: torch.Tensor) -> torch.Tensor:
    """One SwiGLU FFN (ffn.py:42-44).  bf16 shapes the tensor-core tiling covers
    run as one expert directly over the token rows; others as a single expert
    that every token selects with gate 1.0 through the MoE stages."""
    _lib.require_cuda("SwiGLU", x, w_gate_up, w_down)
    H = x.shape[-1]
    x2 = x.reshape(-1, H).contiguous()
    if x2.dtype != w_gate_up.dtype:
        raise TypeError(f"SwiGLU: input dtype {x2.dtype} does not match weight dtype {w_gate_up.dtype}")
    T = x2.shape[0]
    Fdim = w_down.shape[1]
    if _lib.query("ats_swiglu_supported", _lib.dtype_code(x2.dtype), T, H, Fdim) == 1:
        return _DenseSwiGLUFn.apply(x2, w_gate_up, w_down).view(x.shape)
    return routed_swiglu(x2, w_gate_up, w_down).view(x.shape)


def routed_swiglu(x2: torch.Tensor, w_gate_up: torch.Tensor, w_down: torch.Tensor) -> torch.Tensor:
    """The SwiGLU FFN through the MoE stages as one expert with gate 1.0."""
    T = x2.shape[0]
    logits = torch.zeros((T, 1), dtype=torch.float32, device=x2.device)
    return moe_apply(x2, logits, [w_gate_up], [w_down], 1, max(1, T), 0.0)[0]


class _CudaMoE(nn.Module):
    """Counterpart of _PyTorchMoEFallback (moe.py:36-164): the device stages for
    CUDA tensors; for CPU tensors the reference's own loop over the experts
    (``_forward_cpu``), so the reference's CPU tests and CPU-built models run
    unchanged.  A CUDA tensor never takes the CPU loop."""

    def __init__(self, hidden_size: int, intermediate_size: int, num_experts: int, top_k: int,
                 capacity_factor: float, load_balancing_weight: float, num_layers: int,
                 quantization: str = "none") -> None:
        super().__init__()
        if not 1 <= top_k <= min(num_experts, 16):
            raise ValueError(f"MoE top_k must be in [1, min(num_experts, 16)], got {top_k}")
        self.hidden_size = hidden_size
        self.intermediate_size = intermediate_size
        self.num_experts = num_experts
        self.top_k = top_k
        self.capacity_factor = capacity_factor
        self.load_balancing_weight = load_balancing_weight
        self.quantization = quantization
        self.gate = nn.Linear(hidden_size, num_experts, bias=False)
        self.experts = nn.ModuleList(
            [SwiGLU(hidden_size, intermediate_size, quantization=quantization) for _ in range(num_experts)])
        for expert in self.experts:
            init_residual_projection(expert.down_proj, num_layers)
        self.last_expert_utilization: dict[int, float] | None = None
        self.last_counts: torch.Tensor | None = None

    def router_logits(self, flat_x: torch.Tensor) -> torch.Tensor:
        """float32 router: x @ Wg^T in float32 whatever the token dtype -- the
        logits forward() routes on (tensor cores for bf16 tokens)."""
        with torch.no_grad():
            return router_forward(flat_x.contiguous(), self.gate.weight, None)[0]

    def compute_routing(self, flat_x: torch.Tensor):
        """(top_k_probs [T,k] f32, top_k_idx [T,k] int64, router_probs [T,E] f32)
        as moe.py:76-90, on the router kernel; no gradient is tracked.  CPU
        tensors: the reference's torch formula, with gradients."""
        if _lib.on_cpu("compute_routing", flat_x, self.gate.weight):
            router_probs = F.softmax(self.gate(flat_x), dim=-1)
            top_k_probs, top_k_idx = torch.topk(router_probs, self.top_k, dim=-1)
            return top_k_probs / top_k_probs.sum(dim=-1, keepdim=True), top_k_idx, router_probs
        logits = self.router_logits(flat_x)
        from ats_v2_b200.moe_fused import _topk

        return _topk(logits, self.top_k, want_probs=True)

    def _weights(self):
        return ([e.gate_up_proj.weight for e in self.experts], [e.down_proj.weight for e in self.experts])

    def _forward_cpu(self, x: torch.Tensor):
        """The reference's single-process loop (moe.py:92-164) on CPU tensors."""
        batch, seq_len, hidden_size = x.shape
        flat_x = x.reshape(-1, hidden_size)
        T = flat_x.shape[0]
        top_k_probs, top_k_idx, router_probs = self.compute_routing(flat_x)
        cap = capacity_for(T, self.top_k, self.num_experts, self.capacity_factor)
        output = torch.zeros_like(flat_x)
        for e, expert in enumerate(self.experts):
            tokens = (top_k_idx == e).any(dim=-1).nonzero(as_tuple=True)[0][:cap]
            if tokens.numel() == 0:
                continue
            gate = (top_k_probs[tokens] * (top_k_idx[tokens] == e)).sum(dim=-1, keepdim=True)
            output.index_add_(0, tokens, expert(flat_x[tokens]) * gate)
        frac = F.one_hot(top_k_idx, self.num_experts).float().sum(dim=1).mean(dim=0)
        aux = self.num_experts * torch.sum(router_probs.mean(dim=0) * frac) * self.load_balancing_weight
        util = frac / frac.sum().clamp(min=1e-8)
        self.last_expert_utilization = {i: float(v) for i, v in enumerate(util.tolist())}
        return output.reshape(batch, seq_len, hidden_size), aux

    def forward(self, x: torch.Tensor):
        batch, seq_len, hidden_size = x.shape
        if hidden_size != self.hidden_size:
            raise ValueError(f"MoE expected hidden_size={self.hidden_size}, got {hidden_size}.")
        if _lib.on_cpu("MoELayer", x, self.gate.weight):
            return self._forward_cpu(x)
        require_plain_weights(self.quantization, "MoELayer")
        flat_x = x.reshape(-1, hidden_size)
        T = flat_x.shape[0]
        cap = capacity_for(T, self.top_k, self.num_experts, self.capacity_factor)
        wgu, wd = self._weights()
        if wgu[0].dtype != flat_x.dtype:
            raise TypeError(f"MoE: token dtype {flat_x.dtype} does not match expert weight dtype {wgu[0].dtype}")
        out, aux, util, counts, _ = moe_apply(flat_x, None, wgu, wd, self.top_k, cap, self.load_balancing_weight,
                                              gate_w=self.gate.weight)
        self.last_expert_utilization = LazyUtilization(util)
        self.last_counts = counts
        return out.view(batch, seq_len, hidden_size), aux


def expert_parallel_world(ep_size: int) -> bool:
    """True when ``ep_size`` > 1 ranks can hold the experts: torch.distributed is
    initialised, or a launcher (torchrun, DeepSpeed) has set WORLD_SIZE for a
    group it will initialise before the first forward, and the world size is a
    multiple of ep_size."""
    if ep_size <= 1:
        return False
    import os

    import torch.distributed as dist

    if dist.is_available() and dist.is_initialized():
        world = dist.get_world_size()
    else:
        world = int(os.environ.get("WORLD_SIZE", "1"))
    return world > 1 and world % ep_size == 0


class MoELayer(nn.Module):
    """Drop-in for ats.model.moe.MoELayer (moe.py:167-274); uses_deepspeed=False.

    ``ep_size`` > 1 in a multi-process run (see ``expert_parallel_world``) makes
    the layer expert-parallel, as the reference's DeepSpeed MoE does with the
    same argument (moe.py:193-214, set from gpus*nodes by ats/cli/train.py:
    400-402): ``self.moe`` is an ``ExpertParallelMoE`` holding num_experts /
    ep_size local experts, with the router replicated; the ranks of an
    expert-parallel group are consecutive, bound at the first forward.
    Otherwise all experts are local, which is what the reference's
    single-process fallback computes whatever ep_size says."""

    def __init__(self, hidden_size: int, intermediate_size: int, num_experts: int, num_layers: int,
                 top_k: int = 2, capacity_factor: float = 1.25, load_balancing_weight: float = 0.01,
                 ep_size: int = 1, quantization: str = "none") -> None:
        super().__init__()
        self.hidden_size = hidden_size
        self.uses_deepspeed = False
        self.ep_size = ep_size
        self.last_expert_utilization: dict[int, float] | None = None
        self.load_balancing_weight = load_balancing_weight
        if expert_parallel_world(ep_size):
            require_plain_weights(quantization, "MoELayer(ep_size > 1)")
            from ats_v2_b200.ep import ExpertParallelMoE

            self.moe = ExpertParallelMoE(hidden_size, intermediate_size, num_experts, num_layers, top_k=top_k,
                                         capacity_factor=capacity_factor,
                                         load_balancing_weight=load_balancing_weight, ep_size=ep_size,
                                         exchange="device")
        else:
            self.moe = _CudaMoE(hidden_size, intermediate_size, num_experts, top_k, capacity_factor,
                                load_balancing_weight, num_layers=num_layers, quantization=quantization)

    def forward(self, x: torch.Tensor):
        output, aux_loss = self.moe(x)
        self.last_expert_utilization = self.moe.last_expert_utilization
        return output, aux_loss

"""Expert-parallel MoE layer over torch.distributed (NCCL over NVLink).

The reference delegates expert parallelism to DeepSpeed's MoE
(ats/model/moe.py:193-214, ``ep_size`` = number of GPUs from
ats/cli/train.py:400-402).  Here rank r of a W-rank process group owns the
E_local = E/W experts [r*E_local, (r+1)*E_local); the router weight is
replicated.  One forward:

  1. every rank routes its own T tokens (float32 router, capacity
     ``max(1, int(cf*T*k/E))`` from its own token count, as the fallback and
     DeepSpeed compute it) and gathers its kept rows by expert;
  2. the kept-row counts [W][E_local] go to the experts' ranks with
     ``all_to_all_single``, then the rows themselves:
       exchange="packed" (default): the packed layout, where the experts of a
         destination rank are one contiguous run of segments (each kept count
         rounded up to 128 rows), sent with variable splits -- only rows the
         expert GEMMs read cross NVLink; the split sizes are read from the
         device once per forward;
       exchange="slots": the capacity-slot layout [E][Cp] (Cp = capacity
         rounded up to 128), equal splits, no host synchronisation (what
         DeepSpeed's capacity-padded exchange does);
  3. the receiving rank runs its local experts on the received (source,
     expert) segments through a segment table that covers only their kept
     rows;
  4. the outputs go back with the mirror exchange and are combined by each
     source rank in ascending expert order.

The backward sends the expert-output gradients out, runs the expert
backward (weight gradients reduce over the W segments of each local expert),
and sends the input gradients back.  Expert weights are rank-local, so their
gradients need no all-reduce; the replicated router weight's gradient is the
usual data-parallel all-reduce of the training loop.

The exchange steps (``exchange_counts``, ``exchange_rows``, ``_Exchange``)
only move tensors and work on any device and backend; the device stages are
the library's.  With ``overlap_parts`` P > 1 the local experts run in P parts
and each part's row transfers overlap the other parts' expert GEMMs, which
then leave ``comm_sms`` SMs to the transfers.
"""

from __future__ import annotations

import torch
import torch.distributed as dist
from torch import nn

from ats_v2_b200 import _lib
from ats_v2_b200.ffn import SwiGLU
from ats_v2_b200.moe import (LazyUtilization, capacity_for, init_residual_projection, router_backward,
                             router_forward, stacked)

SLOTS = _lib.ATS_MOE_SLOTS


def slot_rows(capacity: int) -> int:
    """Rows of one expert's slot: the capacity rounded up to 128."""
    return (capacity + 127) // 128 * 128


def exchange_counts(send_kept: torch.Tensor, group=None) -> torch.Tensor:
    """send_kept [E] int32 (kept rows per global expert, viewed [W][E_local])
    -> recv_kept [W*E_local]: row src holds the rows rank src keeps for each of
    this rank's experts."""
    recv = torch.empty_like(send_kept)
    dist.all_to_all_single(recv, send_kept.contiguous(), group=group)
    return recv


def exchange_rows(buf: torch.Tensor, group=None) -> torch.Tensor:
    """Equal-split all-to-all of a [W*E_local*Cp, H] row buffer: chunk r goes to
    rank r, chunk src of the result came from rank src.  The same call sends
    expert inputs out and expert outputs back (the layout is symmetric)."""
    out = torch.empty_like(buf)
    dist.all_to_all_single(out, buf.contiguous(), group=group)
    return out


class _Pending:
    """Exchange steps in flight; wait() orders the current stream after them."""

    def __init__(self, works):
        self.works = [w for w in works if w is not None]

    def wait(self) -> None:
        for w in self.works:
            w.wait()


def _rounded(count: int, Cp: int) -> int:
    """Rows a received segment takes in the packed layout: its kept count,
    clamped to [0, Cp], rounded up to 128."""
    return (min(max(count, 0), Cp) + 127) // 128 * 128


class _Exchange:
    """How rows cross between ranks.

    Layouts: "slots" sends the [W][E_local][Cp] capacity-slot buffer; "packed"
    only the rows the expert GEMMs read (each (source, expert) segment's kept
    count rounded up to 128), with split sizes read once per forward from the
    device.

    ``parts`` P splits each rank's local experts into P runs of E_local/P.  Part
    p's rows leave as soon as they are gathered; the expert GEMMs of part p
    start when its rows have arrived, and its results go back while part p+1
    computes, so all but one part's transfer each way hides behind the GEMMs.
    With P = 1 a part is the whole exchange, one all_to_all_single; with P > 1
    each part is a batch of per-peer sends and receives of contiguous row runs
    (this rank's own run is a local copy).  The expert-side buffer of part p
    holds its (source, expert) segments in that order, W*(E_local/P)*Cp rows."""

    def __init__(self, mode: str, W: int, El: int, Cp: int, group, seg_start: torch.Tensor | None,
                 recv_kept: torch.Tensor, parts: int = 1):
        if W == 1:
            parts = 1
        if El % parts != 0:
            raise ValueError(f"{El} local experts do not split into {parts} parts")
        self.mode, self.W, self.El, self.Cp, self.group, self.parts = mode, W, El, Cp, group, parts
        self.Ep = El // parts
        if W == 1 or (mode == "slots" and parts == 1):
            return
        self.me = dist.get_rank(group)
        self.peers = [dist.get_global_rank(group, r) if group is not None else r for r in range(W)]
        E = W * El
        if mode == "packed":
            host = torch.cat([seg_start.to(torch.int64), recv_kept.to(torch.int64)]).cpu().tolist()
            seg, rk = host[:E + 1], host[E + 1:]
            rr = [_rounded(c, Cp) for c in rk]
        else:
            seg = [e * Cp for e in range(E + 1)]
            rr = [Cp] * E
        Ep = self.Ep
        # send[p][r]: (first row, rows) of part p for rank r in the token-side buffer;
        # recv[p][src]: (first row, rows) of source src in part p's expert-side buffer.
        self.send, self.recv = [], []
        for p in range(parts):
            self.send.append([(seg[r * El + p * Ep], seg[r * El + (p + 1) * Ep] - seg[r * El + p * Ep])
                              for r in range(W)])
            runs, off = [], 0
            for src in range(W):
                n = sum(rr[src * El + p * Ep:src * El + (p + 1) * Ep])
                runs.append((off, n))
                off += n
            self.recv.append(runs)

    def part_rows(self) -> int:
        """Rows of one part's expert-side buffer (an upper bound in the packed layout)."""
        return self.W * self.Ep * self.Cp

    def out(self, buf: torch.Tensor, p: int):
        """Start sending part p of this rank's rows to their experts' ranks.
        Returns (expert-side buffer of part p, pending)."""
        if self.W == 1:
            return buf, _Pending([])
        dst = torch.empty((self.part_rows(),) + tuple(buf.shape[1:]), dtype=buf.dtype, device=buf.device)
        if self.parts == 1:
            if self.mode == "slots":
                w = dist.all_to_all_single(dst, buf.contiguous(), group=self.group, async_op=True)
            else:
                sizes_in = [n for _, n in self.send[0]]
                sizes_out = [n for _, n in self.recv[0]]
                w = dist.all_to_all_single(dst[:sum(sizes_out)], buf[:sum(sizes_in)], output_split_sizes=sizes_out,
                                           input_split_sizes=sizes_in, group=self.group, async_op=True)
            return dst, _Pending([w])
        sends = [buf[s:s + n] for s, n in self.send[p]]
        recvs = [dst[s:s + n] for s, n in self.recv[p]]
        return dst, self._p2p(sends, recvs)

    def back(self, buf: torch.Tensor, dst: torch.Tensor | None, p: int):
        """Start sending part p's expert-side rows back into the token-side
        buffer dst (at the rows they left from).  Returns (dst, pending); with
        one rank dst is buf itself."""
        if self.W == 1:
            return buf, _Pending([])
        if self.parts == 1:
            if self.mode == "slots":
                w = dist.all_to_all_single(dst, buf, group=self.group, async_op=True)
            else:
                sizes_in = [n for _, n in self.recv[0]]
                sizes_out = [n for _, n in self.send[0]]
                w = dist.all_to_all_single(dst[:sum(sizes_out)], buf[:sum(sizes_in)], output_split_sizes=sizes_out,
                                           input_split_sizes=sizes_in, group=self.group, async_op=True)
            return dst, _Pending([w])
        sends = [buf[s:s + n] for s, n in self.recv[p]]
        recvs = [dst[s:s + n] for s, n in self.send[p]]
        return dst, self._p2p(sends, recvs)

    def _p2p(self, sends: list, recvs: list) -> _Pending:
        ops = []
        for r in range(self.W):
            if r == self.me:
                if recvs[r].shape[0]:
                    recvs[r].copy_(sends[r])
                continue
            if sends[r].shape[0]:
                ops.append(dist.P2POp(dist.isend, sends[r], self.peers[r], self.group))
            if recvs[r].shape[0]:
                ops.append(dist.P2POp(dist.irecv, recvs[r], self.peers[r], self.group))
        return _Pending(dist.batch_isend_irecv(ops) if ops else [])


class _EPMoEFn(torch.autograd.Function):
    @staticmethod
    def forward(ctx, x2, gate_w, bias, meta, wgu_stack, wd_stack, *local_weights):
        E, El, k, C, lbw, Fdim, W, group, mode, parts, gemm_sms = meta
        L = SLOTS if mode == "slots" else _lib.ATS_MOE_PACKED
        T, H = x2.shape
        dev = x2.device
        dt = _lib.dtype_code(x2.dtype)
        st = _lib.stream_of(x2)
        Cp = slot_rows(C)
        logits, rws, w32 = router_forward(x2, gate_w, bias)
        wsb = _lib.query("ats_moe_workspace_bytes", T, E, k, C, L)
        R = _lib.query("ats_moe_max_rows", T, E, k, C, L)  # this rank's permuted rows (upper bound)
        ws = torch.empty(wsb, dtype=torch.uint8, device=dev)
        gates = torch.empty((T, k), dtype=torch.float32, device=dev)
        idx = torch.empty((T, k), dtype=torch.int64, device=dev)
        aux = torch.empty((), dtype=torch.float32, device=dev)
        util = torch.empty(E, dtype=torch.float32, device=dev)
        counts = torch.empty(E, dtype=torch.int32, device=dev)
        _lib.call("ats_moe_route_plan", logits.data_ptr(), T, E, k, C, L, float(lbw), gates.data_ptr(),
                  idx.data_ptr(), aux.data_ptr(), util.data_ptr(), counts.data_ptr(), ws.data_ptr(), wsb, st)
        kept = torch.empty(E, dtype=torch.int32, device=dev)
        seg_start = torch.empty(E + 1, dtype=torch.int32, device=dev)
        _lib.call("ats_moe_plan_export", ws.data_ptr(), wsb, T, E, k, C, L, seg_start.data_ptr(), None,
                  kept.data_ptr(), st)
        xs = torch.empty((R, H), dtype=x2.dtype, device=dev)
        _lib.call("ats_moe_gather", x2.data_ptr(), xs.data_ptr(), dt, T, H, E, k, C, L, ws.data_ptr(), wsb, st)
        recv_kept = exchange_counts(kept, group) if W > 1 else kept
        ex = _Exchange(mode, W, El, Cp, group, seg_start, recv_kept, parts)
        P, Ep = ex.parts, ex.Ep
        pend = [ex.out(xs, p) for p in range(P)]
        segb = _lib.query("ats_moe_ep_segments_bytes", W, Ep)
        rk = recv_kept.view(W, El)
        ys = torch.empty((R, H), dtype=x2.dtype, device=dev) if W > 1 else None
        keep, backs = [], []
        with _lib.gemm_sm_limit(gemm_sms if P > 1 else 0):
            for p in range(P):
                seg = torch.empty(segb, dtype=torch.uint8, device=dev)
                _lib.call("ats_moe_ep_segments", rk[:, p * Ep:(p + 1) * Ep].contiguous().data_ptr(), W, Ep, C, L,
                          seg.data_ptr(), segb, st)
                xr, arrived = pend[p]
                arrived.wait()
                RR = xr.shape[0]
                h = torch.empty((RR, 2 * Fdim), dtype=x2.dtype, device=dev)
                a = torch.empty((RR, Fdim), dtype=x2.dtype, device=dev)
                yr = torch.empty((RR, H), dtype=x2.dtype, device=dev)
                _lib.call("ats_moe_ep_experts_fwd", xr.data_ptr(), wgu_stack[p * Ep].data_ptr(),
                          wd_stack[p * Ep].data_ptr(), h.data_ptr(), a.data_ptr(), yr.data_ptr(), dt, W, Ep, C, H,
                          Fdim, seg.data_ptr(), segb, st)
                ys, sent = ex.back(yr, ys, p)
                backs.append(sent)
                keep += [xr, h, a, seg]
        for b in backs:
            b.wait()
        out = torch.empty((T, H), dtype=x2.dtype, device=dev)
        _lib.call("ats_moe_combine", ys.data_ptr(), out.data_ptr(), dt, T, H, E, k, C, L, ws.data_ptr(), wsb, st)
        ctx.save_for_backward(logits, gates, idx, ws, ys, wgu_stack, wd_stack, x2, w32, rws, *keep)
        ctx.meta = (E, El, k, C, lbw, Fdim, W, group, T, H, wsb, R, segb, gate_w.dtype, L, gemm_sms)
        ctx.ex = ex
        ctx.mark_non_differentiable(util, counts, idx)
        return out, aux, util, counts, idx

    @staticmethod
    def backward(ctx, dout, daux, _dutil, _dcounts, _didx):
        logits, gates, idx, ws, ys, wgu_stack, wd_stack, x2, w32, rws, *keep = ctx.saved_tensors
        E, El, k, C, lbw, Fdim, W, group, T, H, wsb, R, segb, gate_dtype, L, gemm_sms = ctx.meta
        ex = ctx.ex
        P, Ep = ex.parts, ex.Ep
        dev = x2.device
        dt = _lib.dtype_code(x2.dtype)
        st = _lib.stream_of(x2)
        if dout is None:
            dout = torch.zeros((T, H), dtype=x2.dtype, device=dev)
        dout = dout.to(x2.dtype).contiguous()
        dys = torch.empty((R, H), dtype=x2.dtype, device=dev)
        dgate_row = torch.empty(R, dtype=torch.float32, device=dev)
        _lib.call("ats_moe_combine_bwd", dout.data_ptr(), ys.data_ptr(), dys.data_ptr(), dgate_row.data_ptr(), dt,
                  T, H, E, k, C, L, ws.data_ptr(), wsb, st)
        pend = [ex.out(dys, p) for p in range(P)]
        dxs = torch.empty((R, H), dtype=x2.dtype, device=dev) if W > 1 else None
        dwgu = torch.empty_like(wgu_stack)
        dwd = torch.empty_like(wd_stack)
        backs = []
        with _lib.gemm_sm_limit(gemm_sms if P > 1 else 0):
            for p in range(P):
                xr, h, a, seg = keep[4 * p:4 * p + 4]
                dyr, arrived = pend[p]
                arrived.wait()
                RR = xr.shape[0]
                dh = torch.empty((RR, 2 * Fdim), dtype=x2.dtype, device=dev)
                dxr = torch.empty((RR, H), dtype=x2.dtype, device=dev)
                _lib.call("ats_moe_ep_experts_bwd", dyr.data_ptr(), xr.data_ptr(), h.data_ptr(), a.data_ptr(),
                          wgu_stack[p * Ep].data_ptr(), wd_stack[p * Ep].data_ptr(), dh.data_ptr(), dxr.data_ptr(),
                          dwgu[p * Ep].data_ptr(), dwd[p * Ep].data_ptr(), dt, W, Ep, C, H, Fdim, seg.data_ptr(),
                          segb, st)
                dxs, sent = ex.back(dxr, dxs, p)
                backs.append(sent)
        # the routing gradient needs only the gate-row gradients: it runs while the last part returns
        dlogits = torch.empty((T, E), dtype=torch.float32, device=dev)
        daux_t = daux.to(torch.float32).contiguous() if daux is not None else None
        _lib.call("ats_moe_route_bwd", logits.data_ptr(), gates.data_ptr(), idx.data_ptr(), dgate_row.data_ptr(),
                  _lib.ptr(daux_t), dlogits.data_ptr(), T, E, k, C, L, float(lbw), ws.data_ptr(), wsb, st)
        for b in backs:
            b.wait()
        dx, dgate_w = router_backward(dlogits, x2, w32, rws, dxs, ws, wsb, (T, E, k, C, L), True)
        grads = [dwgu[e] for e in range(El)] + [dwd[e] for e in range(El)]
        return (dx, dgate_w.to(gate_dtype), None, None, None, None, *grads)


def balanced_placement(load: list[float], world: int) -> list[int]:
    """A permutation perm of the experts such that rank r hosts the experts
    perm[r*E_local:(r+1)*E_local] and the ranks' summed loads are close:
    experts in decreasing load (ties by label) go to the rank with the least
    load so far that still has a free slot (every rank hosts E_local
    experts).  Within a rank the experts keep ascending label order."""
    E = len(load)
    if world < 1 or E % world != 0:
        raise ValueError(f"{E} experts do not split over {world} ranks")
    el = E // world
    order = sorted(range(E), key=lambda e: (-float(load[e]), e))
    bins: list[list[int]] = [[] for _ in range(world)]
    tot = [0.0] * world
    for e in order:
        r = min((r for r in range(world) if len(bins[r]) < el), key=lambda r: (tot[r], r))
        bins[r].append(e)
        tot[r] += float(load[e])
    return [e for b in bins for e in sorted(b)]


class ExpertParallelMoE(nn.Module):
    """MoE layer with its experts sharded over a process group.

    ``experts[i]`` is expert ``rank*E_local + i``; ``gate`` is the replicated
    router (Linear(hidden, num_experts)).  With a world size of 1 it is the
    single-GPU layer on the expert-parallel path.  ``rebalance`` relabels the
    experts so that the ranks carry about equal expected rows.

    ``overlap_parts`` P runs the local experts in P parts so that each part's
    row transfers overlap the expert GEMMs of the others (P must divide the
    local expert count; 1 exchanges everything at once); meanwhile the GEMMs
    leave ``comm_sms`` SMs to the transfers."""

    def __init__(self, hidden_size: int, intermediate_size: int, num_experts: int, num_layers: int,
                 top_k: int = 2, capacity_factor: float = 1.25, load_balancing_weight: float = 0.01,
                 group=None, exchange: str = "packed", overlap_parts: int = 1, comm_sms: int = 16) -> None:
        super().__init__()
        if exchange not in ("packed", "slots"):
            raise ValueError(f"exchange must be 'packed' or 'slots', got {exchange!r}")
        self.exchange = exchange
        self.group = group
        self.world = dist.get_world_size(group) if dist.is_available() and dist.is_initialized() else 1
        self.rank = dist.get_rank(group) if self.world > 1 else 0
        if num_experts % self.world != 0:
            raise ValueError(f"num_experts={num_experts} must be divisible by the expert-parallel size {self.world}")
        if not 1 <= top_k <= min(num_experts, 16):
            raise ValueError(f"MoE top_k must be in [1, min(num_experts, 16)], got {top_k}")
        self.hidden_size = hidden_size
        self.num_experts = num_experts
        self.num_local_experts = num_experts // self.world
        if overlap_parts < 1 or self.num_local_experts % overlap_parts != 0:
            raise ValueError(f"overlap_parts={overlap_parts} must divide the {self.num_local_experts} local experts")
        if comm_sms < 0:
            raise ValueError(f"comm_sms must be >= 0, got {comm_sms}")
        self.overlap_parts = overlap_parts
        self.comm_sms = comm_sms
        self.top_k = top_k
        self.capacity_factor = capacity_factor
        self.load_balancing_weight = load_balancing_weight
        self.gate = nn.Linear(hidden_size, num_experts, bias=False)
        self.experts = nn.ModuleList([SwiGLU(hidden_size, intermediate_size) for _ in range(self.num_local_experts)])
        for ex in self.experts:
            init_residual_projection(ex.down_proj, num_layers)
        self.last_expert_utilization: dict[int, float] | None = None
        self.last_counts: torch.Tensor | None = None

    @torch.no_grad()
    def rebalance(self, load=None, perm=None) -> torch.Tensor:
        """Relabel the experts so that every rank's experts carry about the same
        expected rows, and return the permutation perm (int64 [E]): the expert
        now labelled j is the one that was labelled perm[j].

        ``load`` [E] is the expected rows per expert label, the same on every
        rank (for example the kept counts of a calibration batch, summed over
        the ranks).  An expert's gate row and weights move with it, so the layer
        computes the same function; the experts only change rank (the gate
        weight is replicated; the expert weights are all-gathered once and each
        rank keeps its new experts).  Which rank runs an expert changes no
        result.  What does change is the label order: ties in the top-k go to
        the lower new label, a token's expert outputs are summed in new label
        order (with top_k = 2 the sum of two rows rounds the same in either
        order), and the router's share of the input gradient sums over the
        experts in new label order (float32, so its last bits can differ).
        Per-expert inputs indexed by label, such as a logit
        bias, must be re-indexed with perm by the caller.  Call it before an
        optimizer holds per-parameter state: that state does not move.  An
        explicit ``perm`` (same on every rank) may be given instead of ``load``."""
        if perm is None:
            load = [float(v) for v in torch.as_tensor(load).flatten().tolist()]
            if len(load) != self.num_experts:
                raise ValueError(f"rebalance: load has {len(load)} entries, expected {self.num_experts}")
            perm = balanced_placement(load, self.world)
        else:
            perm = [int(v) for v in torch.as_tensor(perm).flatten().tolist()]
            if sorted(perm) != list(range(self.num_experts)):
                raise ValueError("rebalance: perm must be a permutation of the expert labels")
        W, El = self.world, self.num_local_experts
        gw = self.gate.weight
        gw.copy_(gw[torch.as_tensor(perm, device=gw.device)].clone())
        for name in ("gate_up_proj", "down_proj"):
            local = torch.stack([getattr(ex, name).weight.detach() for ex in self.experts])
            if W > 1:
                parts = [torch.empty_like(local) for _ in range(W)]
                dist.all_gather(parts, local.contiguous(), group=self.group)
                full = torch.cat(parts)
            else:
                full = local.clone()
            for i, ex in enumerate(self.experts):
                getattr(ex, name).weight.copy_(full[perm[self.rank * El + i]])
        return torch.as_tensor(perm, dtype=torch.int64)

    def _gemm_sms(self, device: torch.device) -> int:
        """SMs the expert GEMMs may use while transfers are in flight."""
        if self.overlap_parts == 1 or self.world == 1 or self.comm_sms == 0:
            return 0
        return max(1, torch.cuda.get_device_properties(device).multi_processor_count - self.comm_sms)

    def router_logits(self, flat_x: torch.Tensor) -> torch.Tensor:
        """The float32 logits forward() routes on (without a logit bias)."""
        with torch.no_grad():
            return router_forward(flat_x.contiguous(), self.gate.weight, None)[0]

    def forward(self, x: torch.Tensor, logit_bias: torch.Tensor | None = None):
        """x [B,S,H] -> (out [B,S,H], aux).  ``logit_bias`` [E] is a constant added
        to the router logits (used to impose a skewed expert load in benchmarks)."""
        batch, seq, H = x.shape
        if H != self.hidden_size:
            raise ValueError(f"MoE expected hidden_size={self.hidden_size}, got {H}.")
        _lib.require_cuda("ExpertParallelMoE", x)
        flat = x.reshape(-1, H).contiguous()
        T = flat.shape[0]
        cap = capacity_for(T, self.top_k, self.num_experts, self.capacity_factor)
        wgu = [e.gate_up_proj.weight for e in self.experts]
        wd = [e.down_proj.weight for e in self.experts]
        if wgu[0].dtype != flat.dtype:
            raise TypeError(f"MoE: token dtype {flat.dtype} does not match expert weight dtype {wgu[0].dtype}")
        meta = (self.num_experts, self.num_local_experts, self.top_k, cap, self.load_balancing_weight,
                wgu[0].shape[0] // 2, self.world, self.group, self.exchange, self.overlap_parts,
                self._gemm_sms(flat.device))
        bias = logit_bias.detach().float().contiguous() if logit_bias is not None else None
        out, aux, util, counts, _ = _EPMoEFn.apply(flat, self.gate.weight, bias, meta, stacked(wgu), stacked(wd),
                                                   *wgu, *wd)
        self.last_expert_utilization = LazyUtilization(util)
        self.last_counts = counts
        return out.view(batch, seq, H), aux

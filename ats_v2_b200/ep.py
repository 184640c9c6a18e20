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
     ``all_to_all_single`` (the peer exchange all-gathers every rank's counts
     instead, to place its copies), then the rows themselves:
       exchange="packed" (default): the packed layout, where the experts of a
         destination rank are one contiguous run of segments (each kept count
         rounded up to 128 rows), sent with variable splits -- only rows the
         expert GEMMs read cross NVLink; the split sizes are read from the
         device once per forward;
       exchange="slots": the capacity-slot layout [E][Cp] (Cp = capacity
         rounded up to 128), equal splits, no host synchronisation (what
         DeepSpeed's capacity-padded exchange does);
       exchange="peer" (one node): the packed rows, copied by the copy
         engines straight into receive buffers every peer mapped once through
         CUDA IPC, with collectives as the ordering points (no SMs spent on
         the transfers, so they overlap the expert GEMMs);
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

The NCCL exchange steps (``exchange_counts``, ``exchange_rows``,
``_Exchange``) only move tensors and work on any device and backend; the copy
plan of the peer exchange (``peer_plan``) is plain host arithmetic; the device
stages are the library's.  With ``overlap_parts`` P > 1 the local experts run
in P parts and each part's row transfers overlap the other parts' expert
GEMMs, which then leave ``comm_sms`` SMs to the collectives.
"""

from __future__ import annotations

import ctypes
import socket
import weakref

import torch
import torch.distributed as dist
from torch import nn

from ats_v2_b200 import _lib
from ats_v2_b200.ffn import SwiGLU
from ats_v2_b200.moe import (LazyUtilization, capacity_for, init_residual_projection, router_backward,
                             router_forward, router_weight_grad, stacked)

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


def peer_plan(kept: list[list[int]], Cp: int, El: int, parts: int, me: int):
    """Copy plan of the peer-memory exchange for rank ``me``.

    kept[s][e] is the rows source rank s keeps for global expert e.  Clamped to
    [0, Cp] and rounded up to 128 they are the segment sizes of the packed
    layout: the token side of rank s holds its segments in global expert order,
    and part p of rank d's expert side holds, for each source in rank order,
    the segments of d's local experts [p*Ep, (p+1)*Ep), Ep = El/parts (the
    layout ``ats_moe_ep_segments`` reads).  Returns (seg, out, back):
      seg[s]   the token-side segment starts of rank s ([E+1]);
      out[p]   (d, src_row, dst_row, rows): my token-side rows [src_row, +rows)
               go to rows [dst_row, +rows) of part p on rank d;
      back[p]  (s, src_row, dst_row, rows): rows [src_row, +rows) of my part p
               go back to rows [dst_row, +rows) of rank s's token side.
    Runs of zero rows are left out."""
    W = len(kept)
    E = W * El
    if El % parts != 0:
        raise ValueError(f"{El} local experts do not split into {parts} parts")
    Ep = El // parts
    rnd = [[_rounded(int(c), Cp) for c in row] for row in kept]
    seg = []
    for s in range(W):
        acc = [0]
        for e in range(E):
            acc.append(acc[-1] + rnd[s][e])
        seg.append(acc)

    def run(s, d, p):  # rows source s holds for part p of rank d
        return sum(rnd[s][d * El + p * Ep:d * El + (p + 1) * Ep])

    out, back = [], []
    for p in range(parts):
        o = []
        for d in range(W):
            n = run(me, d, p)
            if n:
                o.append((d, seg[me][d * El + p * Ep], sum(run(s, d, p) for s in range(me)), n))
        out.append(o)
        b, off = [], 0
        for src in range(W):
            n = run(src, me, p)
            if n:
                b.append((src, off, seg[src][me * El + p * Ep], n))
            off += n
        back.append(b)
    return seg, out, back


_OPENED: dict[bytes, list] = {}  # IPC handle -> [mapped base, opens]; one open per handle and process


def _ipc_open(handle: bytes) -> int:
    ent = _OPENED.get(handle)
    if ent is None:
        base = ctypes.c_void_p()
        _lib.call("ats_ipc_open", handle, ctypes.byref(base))
        ent = _OPENED[handle] = [base.value, 0]
    ent[1] += 1
    return ent[0]


def _ipc_close(handle: bytes) -> None:
    ent = _OPENED[handle]
    ent[1] -= 1
    if ent[1] == 0:
        del _OPENED[handle]
        _lib.call("ats_ipc_close", ctypes.c_void_p(ent[0]))


def _copies(copies: list, stream) -> None:
    """copies: (dst address, src address, bytes); one copy-engine copy each."""
    n = len(copies)
    if n == 0:
        return
    dst = (ctypes.c_void_p * n)(*[c[0] for c in copies])
    src = (ctypes.c_void_p * n)(*[c[1] for c in copies])
    nb = (ctypes.c_uint64 * n)(*[c[2] for c in copies])
    _lib.call("ats_peer_copies", n, dst, src, nb, stream.cuda_stream)


class _PeerSet:
    """The buffers other ranks copy into for one forward and backward of the
    layer, allocated on every rank and mapped by every peer:
      xr  [rows_x, H]  expert-side input rows (part p from row p*W*Ep*Cp)
      ys  [rows_t, H]  token-side expert outputs
      dyr [rows_x, H]  expert-side output gradients
      dxs [rows_t, H]  token-side input gradients
    ``addr[r][name]`` is rank r's buffer as an address in this process."""

    NAMES = ("xr", "ys", "dyr", "dxs")

    def __init__(self, rows_x: int, rows_t: int, H: int, dtype, device, group, W: int, me: int,
                 names: tuple = NAMES, expert_side: tuple = ("xr", "dyr")):
        self.rows_x, self.rows_t, self.H, self.dtype = rows_x, rows_t, H, dtype
        self.local = {n: torch.empty((rows_x if n in expert_side else rows_t, H), dtype=dtype, device=device)
                      for n in names}
        self._tables: dict = {}
        hb = _lib.query("ats_ipc_handle_bytes")
        mine = {}
        for n, t in self.local.items():
            h = ctypes.create_string_buffer(hb)
            off, size = ctypes.c_uint64(), ctypes.c_uint64()
            _lib.call("ats_ipc_export", t.data_ptr(), h, ctypes.byref(off), ctypes.byref(size))
            mine[n] = (h.raw, off.value)
        every = [None] * W
        dist.all_gather_object(every, (socket.gethostname(), mine), group=group)
        if len({host for host, _ in every}) != 1:
            raise ValueError("ExpertParallelMoE(exchange='peer') maps the peers' memory with CUDA IPC, which needs "
                             "every rank of the group on one node; use exchange='packed' across nodes")
        every = [m for _, m in every]
        self.handles: list[bytes] = []
        self.addr: list[dict] = []
        for r in range(W):
            if r == me:
                self.addr.append({n: t.data_ptr() for n, t in self.local.items()})
                continue
            a = {}
            for n, (h, off) in every[r].items():
                a[n] = _ipc_open(h) + off
                self.handles.append(h)
            self.addr.append(a)
        self.busy = False
        self.owner = None  # weak reference to the autograd context of the forward holding the set

    def fits(self, rows_x: int, rows_t: int, H: int, dtype) -> bool:
        return rows_x <= self.rows_x and rows_t <= self.rows_t and H == self.H and dtype == self.dtype

    def table(self, name: str) -> torch.Tensor:
        """Every rank's buffer `name` as an address of this process, in device
        memory (int64 [W]): what the device-driven exchange kernels index."""
        t = self._tables.get(name)
        if t is None:
            t = torch.tensor([a[name] for a in self.addr], dtype=torch.int64).to(self.local[name].device)
            self._tables[name] = t
        return t

    def close(self) -> None:
        for h in self.handles:
            _ipc_close(h)
        self.handles = []


class _PeerState:
    """Per-layer state of the peer-memory exchange: a pool of buffer sets (one
    per forward whose backward has not run yet), the streams the copies run on,
    the one-element tensor of the collectives that order them and a pinned
    buffer for the counts.  A set goes back to the pool when its backward has
    run, at the end of a forward no backward will follow, or -- when no free
    set fits -- once its forward's graph is gone on every rank."""

    MAX_SETS = 4

    def __init__(self):
        self.sets: list[_PeerSet] = []
        self.streams: dict = {}
        self.flags: dict = {}
        self.host: torch.Tensor | None = None

    def acquire(self, rows_x, rows_t, H, dtype, device, group, W, me, names=_PeerSet.NAMES,
                expert_side=("xr", "dyr")) -> _PeerSet:
        # every rank makes the same choice: the sizes are maxima over the ranks and
        # the ranks run the same sequence of forwards and backwards
        ps = self._free(rows_x, rows_t, H, dtype)
        if ps is None and any(q.busy for q in self.sets):
            # a forward whose graph is gone without a backward (activation checkpointing
            # recomputes the forward inside the backward and drops that graph) leaves its set
            # busy; take such sets back, but only those orphaned on every rank
            mask = [int(q.busy and q.owner is not None and q.owner() is None) for q in self.sets]
            for q, m in zip(self.sets, self._agree(mask, group, device)):
                if m:
                    q.busy = False
            ps = self._free(rows_x, rows_t, H, dtype)
        if ps is not None:
            ps.busy = True
            return ps
        for ps in [q for q in self.sets if not q.busy]:
            ps.close()
            self.sets.remove(ps)
        if len(self.sets) >= self.MAX_SETS:
            raise RuntimeError(f"ExpertParallelMoE: {len(self.sets)} forwards are waiting for their backward; the "
                               f"peer exchange keeps one buffer set per forward")
        ps = _PeerSet(rows_x, rows_t, H, dtype, device, group, W, me, names, expert_side)
        ps.busy = True
        self.sets.append(ps)
        return ps

    def _free(self, rows_x, rows_t, H, dtype):
        for ps in self.sets:
            if not ps.busy and ps.fits(rows_x, rows_t, H, dtype):
                return ps
        return None

    @staticmethod
    def _agree(mask: list, group, device) -> list:
        """Element-wise minimum of the mask over the ranks."""
        t = torch.tensor(mask, dtype=torch.int32, device=device)
        dist.all_reduce(t, op=dist.ReduceOp.MIN, group=group)
        return t.tolist()

    @staticmethod
    def release(ps: _PeerSet) -> None:
        ps.busy = False
        ps.owner = None

    def copy_streams(self, device, W: int) -> list:
        """One stream per destination rank, so that the copies to different
        ranks (and this rank's own rows) run on different copy engines at once;
        the first also carries the collectives that order them."""
        key = (device, W)
        if key not in self.streams:
            self.streams[key] = [torch.cuda.Stream(device=device) for _ in range(W)]
        return self.streams[key]

    def host_buffer(self, n: int) -> torch.Tensor:
        """Pinned int32 host buffer for the counts every forward reads."""
        if self.host is None or self.host.numel() < n:
            self.host = torch.empty(n, dtype=torch.int32, pin_memory=True)
        return self.host[:n]

    def flag(self, device) -> torch.Tensor:
        if device not in self.flags:
            self.flags[device] = torch.zeros(1, dtype=torch.int32, device=device)
        return self.flags[device]

    def close(self) -> None:
        for ps in self.sets:
            ps.close()
        self.sets = []


def _route(x2, gate_w, bias, E, k, C, L, lbw):
    """Route this rank's tokens over all E experts into layout L.  R is this
    rank's permuted rows (an upper bound); kept [E] and seg_start [E+1] (int32,
    device) describe the segments the gather writes."""
    T, H = x2.shape
    dev = x2.device
    st = _lib.stream_of(x2)
    logits, rws, w32 = router_forward(x2, gate_w, bias)
    wsb = _lib.query("ats_moe_workspace_bytes", T, E, k, C, L)
    R = _lib.query("ats_moe_max_rows", T, E, k, C, L)
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
    return logits, rws, w32, ws, wsb, R, gates, idx, aux, util, counts, kept, seg_start


def _row_tokens(ws, wsb, T, E, k, C, L, R, dev):
    """The token of every permuted row (int32 [R], -1 = padding) from the plan."""
    rt = torch.empty(R, dtype=torch.int32, device=dev)
    _lib.call("ats_moe_plan_export", ws.data_ptr(), wsb, T, E, k, C, L, None, rt.data_ptr(), None,
              _lib.stream_of(rt))
    return rt


def _gather(x2, ws, wsb, R, E, k, C, L):
    """This rank's kept rows, gathered by segment: [R, H]."""
    T, H = x2.shape
    xs = torch.empty((R, H), dtype=x2.dtype, device=x2.device)
    _lib.call("ats_moe_gather", x2.data_ptr(), xs.data_ptr(), _lib.dtype_code(x2.dtype), T, H, E, k, C, L,
              ws.data_ptr(), wsb, _lib.stream_of(x2))
    return xs


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
        (logits, rws, w32, ws, wsb, R, gates, idx, aux, util, counts, kept,
         seg_start) = _route(x2, gate_w, bias, E, k, C, L, lbw)
        xs = _gather(x2, ws, wsb, R, E, k, C, L)
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


def _issue_copies(plan_p: list, streams: list, dst_addr, src_base: int, rowb: int) -> None:
    """Copies of one part, grouped by the rank on the other side: entry
    (r, src_row, dst_row, rows) goes on streams[r] to dst_addr(r) + dst_row."""
    by_rank: dict[int, list] = {}
    for r, src_row, dst_row, n in plan_p:
        by_rank.setdefault(r, []).append((dst_addr(r) + dst_row * rowb, src_base + src_row * rowb, n * rowb))
    for r, cps in by_rank.items():
        with torch.cuda.stream(streams[r]):
            _copies(cps, streams[r])


def _barrier_after(streams: list, flag: torch.Tensor, group):
    """A collective on streams[0] after the copies queued so far on every stream:
    when it completes, every rank's copies have landed."""
    for st in streams[1:]:
        streams[0].wait_stream(st)
    with torch.cuda.stream(streams[0]):
        return dist.all_reduce(flag, group=group, async_op=True)


def _follow(streams: list, cur, *tensors) -> None:
    """Make every copy stream wait for the current stream's work so far, and
    keep the tensors' memory until the copies that read them have run."""
    for st in streams:
        st.wait_stream(cur)
        for t in tensors:
            t.record_stream(st)


class _EPPeerFn(torch.autograd.Function):
    """The expert-parallel layer with the rows copied by the copy engines
    straight into the peers' buffers (packed layout, in overlapped parts), one
    stream per destination rank.

    Ordering between ranks comes from collectives on the layer's group, each
    issued on the stream whose work it must follow:
      - the all-gather of the kept counts, issued right after routing: every
        rank's earlier work on its buffers (the last backward) is done when it
        completes, and the copies wait for it.  Its result reaches the host
        through a pinned buffer while the gather kernel runs, so the host plans
        the copies in the gather's shadow;
      - a one-element all-reduce after each part's copies: when it completes,
        every rank's rows of that part have landed, and the expert GEMMs of the
        part wait for it;
      - one more after the return copies, before the combine (forward) or the
        router backward (backward)."""

    @staticmethod
    def forward(ctx, x2, gate_w, bias, meta, wgu_stack, wd_stack, *local_weights):
        E, El, k, C, lbw, Fdim, W, group, parts, gemm_sms, state, me, will_backward = meta
        L = _lib.ATS_MOE_PACKED
        T, H = x2.shape
        dev = x2.device
        dt = _lib.dtype_code(x2.dtype)
        st = _lib.stream_of(x2)
        Cp = slot_rows(C)
        cur = torch.cuda.current_stream(dev)
        cs = state.copy_streams(dev, W)
        flag = state.flag(dev)
        (logits, rws, w32, ws, wsb, R, gates, idx, aux, util, counts, kept,
         seg_start) = _route(x2, gate_w, bias, E, k, C, L, lbw)
        mine = torch.cat([kept, torch.tensor([Cp, R], dtype=torch.int32, device=dev), seg_start])
        allv = torch.empty((W, 2 * E + 3), dtype=torch.int32, device=dev)
        gathered = dist.all_gather_into_tensor(allv, mine, group=group, async_op=True)
        xs = _gather(x2, ws, wsb, R, E, k, C, L)
        host_buf = state.host_buffer(allv.numel())
        with torch.cuda.stream(cs[0]):
            gathered.wait()
            allv.record_stream(cs[0])
            host_buf.copy_(allv.view(-1), non_blocking=True)
            ready = torch.cuda.Event()
            ready.record(cs[0])
        gathered.wait()  # the copies below follow the current stream
        ready.synchronize()
        host = host_buf.tolist()
        rows = [host[s_ * (2 * E + 3):(s_ + 1) * (2 * E + 3)] for s_ in range(W)]
        if len({r[E] for r in rows}) != 1:
            raise ValueError("ExpertParallelMoE: every rank must route the same number of tokens")
        seg, out_plan, back_plan = peer_plan([r[:E] for r in rows], Cp, El, parts, me)
        if any(seg[s_] != rows[s_][E + 2:] for s_ in range(W)):
            raise RuntimeError("ExpertParallelMoE: the packed layout differs from the copy plan")
        rows_t = max(r[E + 1] for r in rows)
        ps = state.acquire(W * El * Cp, rows_t, H, x2.dtype, dev, group, W, me)
        ps.owner = weakref.ref(ctx)
        Ep = El // parts
        part_rows = W * Ep * Cp
        rowb = H * x2.element_size()
        for p in range(parts):
            for d, src_row, dst_row, n in out_plan[p]:
                assert src_row + n <= R and dst_row + n <= part_rows
            for s_, src_row, dst_row, n in back_plan[p]:
                assert src_row + n <= part_rows and dst_row + n <= rows_t
        _follow(cs, cur, xs)
        arrived = []
        for p in range(parts):
            _issue_copies(out_plan[p], cs, lambda d, p=p: ps.addr[d]["xr"] + p * part_rows * rowb, xs.data_ptr(),
                          rowb)
            arrived.append(_barrier_after(cs, flag, group))
        segb = _lib.query("ats_moe_ep_segments_bytes", W, Ep)
        keep = []
        with _lib.gemm_sm_limit(gemm_sms):
            for p in range(parts):
                seg_ws = torch.empty(segb, dtype=torch.uint8, device=dev)
                rk = allv[:, me * El + p * Ep:me * El + (p + 1) * Ep].contiguous()
                _lib.call("ats_moe_ep_segments", rk.data_ptr(), W, Ep, C, L, seg_ws.data_ptr(), segb, st)
                arrived[p].wait()
                xr = ps.local["xr"][p * part_rows:(p + 1) * part_rows]
                h = torch.empty((part_rows, 2 * Fdim), dtype=x2.dtype, device=dev)
                a = torch.empty((part_rows, Fdim), dtype=x2.dtype, device=dev)
                yr = torch.empty((part_rows, H), dtype=x2.dtype, device=dev)
                _lib.call("ats_moe_ep_experts_fwd", xr.data_ptr(), wgu_stack[p * Ep].data_ptr(),
                          wd_stack[p * Ep].data_ptr(), h.data_ptr(), a.data_ptr(), yr.data_ptr(), dt, W, Ep, C, H,
                          Fdim, seg_ws.data_ptr(), segb, st)
                _follow(cs, cur, yr)
                _issue_copies(back_plan[p], cs, lambda s_: ps.addr[s_]["ys"], yr.data_ptr(), rowb)
                keep += [h, a, seg_ws]
        _barrier_after(cs, flag, group).wait()
        out = torch.empty((T, H), dtype=x2.dtype, device=dev)
        _lib.call("ats_moe_combine", ps.local["ys"].data_ptr(), out.data_ptr(), dt, T, H, E, k, C, L, ws.data_ptr(),
                  wsb, st)
        ctx.save_for_backward(logits, gates, idx, ws, wgu_stack, wd_stack, x2, w32, rws, *keep)
        ctx.meta = (E, El, k, C, lbw, Fdim, W, group, T, H, wsb, R, segb, gate_w.dtype, gemm_sms, parts, part_rows)
        ctx.plans = (out_plan, back_plan)
        ctx.ps, ctx.state = ps, state
        if not will_backward:
            state.release(ps)
        ctx.mark_non_differentiable(util, counts, idx)
        return out, aux, util, counts, idx

    @staticmethod
    def backward(ctx, dout, daux, _dutil, _dcounts, _didx):
        logits, gates, idx, ws, wgu_stack, wd_stack, x2, w32, rws, *keep = ctx.saved_tensors
        E, El, k, C, lbw, Fdim, W, group, T, H, wsb, R, segb, gate_dtype, gemm_sms, parts, part_rows = ctx.meta
        out_plan, back_plan = ctx.plans
        ps, state = ctx.ps, ctx.state
        L = _lib.ATS_MOE_PACKED
        Ep = El // parts
        dev = x2.device
        dt = _lib.dtype_code(x2.dtype)
        st = _lib.stream_of(x2)
        rowb = H * x2.element_size()
        cur = torch.cuda.current_stream(dev)
        cs = state.copy_streams(dev, W)
        flag = state.flag(dev)
        if dout is None:
            dout = torch.zeros((T, H), dtype=x2.dtype, device=dev)
        dout = dout.to(x2.dtype).contiguous()
        dys = torch.empty((R, H), dtype=x2.dtype, device=dev)
        dgate_row = torch.empty(R, dtype=torch.float32, device=dev)
        _lib.call("ats_moe_combine_bwd", dout.data_ptr(), ps.local["ys"].data_ptr(), dys.data_ptr(),
                  dgate_row.data_ptr(), dt, T, H, E, k, C, L, ws.data_ptr(), wsb, st)
        _follow(cs, cur, dys)
        arrived = []
        for p in range(parts):
            _issue_copies(out_plan[p], cs, lambda d, p=p: ps.addr[d]["dyr"] + p * part_rows * rowb, dys.data_ptr(),
                          rowb)
            arrived.append(_barrier_after(cs, flag, group))
        dwgu = torch.empty_like(wgu_stack)
        dwd = torch.empty_like(wd_stack)
        with _lib.gemm_sm_limit(gemm_sms):
            for p in range(parts):
                h, a, seg_ws = keep[3 * p:3 * p + 3]
                arrived[p].wait()
                xr = ps.local["xr"][p * part_rows:(p + 1) * part_rows]
                dyr = ps.local["dyr"][p * part_rows:(p + 1) * part_rows]
                dh = torch.empty((part_rows, 2 * Fdim), dtype=x2.dtype, device=dev)
                dxr = torch.empty((part_rows, H), dtype=x2.dtype, device=dev)
                _lib.call("ats_moe_ep_experts_bwd", dyr.data_ptr(), xr.data_ptr(), h.data_ptr(), a.data_ptr(),
                          wgu_stack[p * Ep].data_ptr(), wd_stack[p * Ep].data_ptr(), dh.data_ptr(), dxr.data_ptr(),
                          dwgu[p * Ep].data_ptr(), dwd[p * Ep].data_ptr(), dt, W, Ep, C, H, Fdim, seg_ws.data_ptr(),
                          segb, st)
                _follow(cs, cur, dxr)
                _issue_copies(back_plan[p], cs, lambda s_: ps.addr[s_]["dxs"], dxr.data_ptr(), rowb)
        # the routing gradient needs only the gate-row gradients: it runs while the last part returns
        dlogits = torch.empty((T, E), dtype=torch.float32, device=dev)
        daux_t = daux.to(torch.float32).contiguous() if daux is not None else None
        _lib.call("ats_moe_route_bwd", logits.data_ptr(), gates.data_ptr(), idx.data_ptr(), dgate_row.data_ptr(),
                  _lib.ptr(daux_t), dlogits.data_ptr(), T, E, k, C, L, float(lbw), ws.data_ptr(), wsb, st)
        _barrier_after(cs, flag, group).wait()
        dx, dgate_w = router_backward(dlogits, x2, w32, rws, ps.local["dxs"], ws, wsb, (T, E, k, C, L), True)
        state.release(ps)
        grads = [dwgu[e] for e in range(El)] + [dwd[e] for e in range(El)]
        return (dx, dgate_w.to(gate_dtype), None, None, None, None, *grads)


# The device exchange's backward runs the router weight gradient beside the output-gradient push (needs
# comm_sms > 0 and the tensor-core router).
_ROUTER_BESIDE_PUSH = True
# The device exchange's forward combines straight from the expert ranks' buffers (ats_moe_ep_combine)
# instead of pulling the rows, then combining them.
_FUSED_COMBINE = True
# The device exchange's forward computes a rank's own rows beside the transfer of the others' (one part,
# comm_sms > 0).  Off: measured slower (the GEMMs beside the transfer run 1.8x longer than alone).
_OWN_ROWS_FIRST = False

_DEVICE_SET = ("xr", "yr", "dyr", "dxr")  # every buffer of a device-exchange set is expert-side

# When a list, the device exchange records a CUDA event on the current stream at each phase boundary
# of its forward and backward, as (phase, event) pairs: how a benchmark splits a step between routing,
# the exchange (waits for the slowest rank included) and the expert GEMMs.  None: nothing is recorded.
PHASE_EVENTS: list | None = None


def _mark(name: str) -> None:
    if PHASE_EVENTS is not None:
        ev = torch.cuda.Event(enable_timing=True)
        ev.record()
        PHASE_EVENTS.append((name, ev))


def _exchange_args(allv, W, me, El, parts, lo, hi, table, part_rows, H, dt, sms=0):
    return (allv.data_ptr(), W, me, El, parts, lo, hi, table.data_ptr(), part_rows, H, dt, sms)


class _EPDeviceFn(torch.autograd.Function):
    """The expert-parallel layer with a device-driven exchange: no split size
    ever reaches the host, and no gathered copy of the rows is made.

      forward:  route -> all-gather the [W][2E+3] counts -> zero the padding
                rows of this rank's expert-side buffer, push this rank's kept
                token rows (gathered through row_token) into the expert ranks'
                buffers -> all-reduce(flag) -> expert GEMMs into the mapped y
                buffer -> all-reduce(flag) -> pull this rank's expert outputs
                into the local packed layout -> combine.
      backward: combine backward -> push the output-gradient rows ->
                all-reduce(flag) -> expert data gradient into the mapped dx
                buffer -> all-reduce(flag) -> pull the input-gradient rows ->
                routing and router backward.  The expert weight gradients
                come after the data gradient; with ``comm_sms`` > 0 they run
                on the other SMs while the all-reduce and the pull run on a
                side stream with those SMs, so the return transfer hides
                behind them.

    Ordering between ranks comes only from the collectives, each on the
    current stream after the kernels it must follow; no kernel waits on
    another rank.  A buffer set is reused only after its backward: the next
    forward's counts all-gather completes on no rank before every rank has
    finished the work queued before it, that backward included."""

    @staticmethod
    def forward(ctx, x2, gate_w, bias, meta, wgu_stack, wd_stack, *local_weights):
        E, El, k, C, lbw, Fdim, W, group, parts, comm_sms, state, me, will_backward = meta
        L = _lib.ATS_MOE_PACKED
        T, H = x2.shape
        dev = x2.device
        dt = _lib.dtype_code(x2.dtype)
        st = _lib.stream_of(x2)
        Cp = slot_rows(C)
        Ep = El // parts
        part_rows = W * Ep * Cp
        flag = state.flag(dev)
        _mark("start")
        (logits, rws, w32, ws, wsb, R, gates, idx, aux, util, counts, kept,
         seg_start) = _route(x2, gate_w, bias, E, k, C, L, lbw)
        row_token = _row_tokens(ws, wsb, T, E, k, C, L, R, dev)
        mine = torch.cat([kept, torch.tensor([Cp, R], dtype=torch.int32, device=dev), seg_start])
        allv = torch.empty((W, 2 * E + 3), dtype=torch.int32, device=dev)
        _mark("route")
        dist.all_gather_into_tensor(allv, mine, group=group)
        _mark("exchange_counts")
        ps = state.acquire(parts * part_rows, 0, H, x2.dtype, dev, group, W, me, _DEVICE_SET, _DEVICE_SET)
        ps.owner = weakref.ref(ctx)
        _lib.call("ats_moe_ep_zero_padding", ps.local["xr"].data_ptr(), allv.data_ptr(), W, me, El, parts, 0,
                  parts, part_rows, H, dt, st)
        segb = _lib.query("ats_moe_ep_segments_bytes", W, Ep)
        keep = []
        ys = torch.empty((R, H), dtype=x2.dtype, device=dev)

        def push(lo, hi, sms, stream):
            _lib.call("ats_moe_ep_push", x2.data_ptr(), row_token.data_ptr(), T,
                      *_exchange_args(allv, W, me, El, parts, lo, hi, ps.table("xr"), part_rows, H, dt, sms),
                      stream.cuda_stream)

        def pull(lo, hi, sms, stream):
            _lib.call("ats_moe_ep_pull", ys.data_ptr(), R,
                      *_exchange_args(allv, W, me, El, parts, lo, hi, ps.table("yr"), part_rows, H, dt, sms),
                      stream.cuda_stream)

        def experts_prep(p):
            seg_ws = torch.empty(segb, dtype=torch.uint8, device=dev)
            rk = allv[:, me * El + p * Ep:me * El + (p + 1) * Ep].contiguous()
            _lib.call("ats_moe_ep_segments", rk.data_ptr(), W, Ep, C, L, seg_ws.data_ptr(), segb, st)
            xr = ps.local["xr"][p * part_rows:(p + 1) * part_rows]
            yr = ps.local["yr"][p * part_rows:(p + 1) * part_rows]
            h = torch.empty((part_rows, 2 * Fdim), dtype=x2.dtype, device=dev)
            a = torch.empty((part_rows, Fdim), dtype=x2.dtype, device=dev)
            keep.extend([h, a, seg_ws])
            return p, xr, yr, h, a, seg_ws

        def experts_run(bufs, sources=None):  # sources: a range of source ranks, or all
            p, xr, yr, h, a, seg_ws = bufs
            args = (xr.data_ptr(), wgu_stack[p * Ep].data_ptr(), wd_stack[p * Ep].data_ptr(), h.data_ptr(),
                    a.data_ptr(), yr.data_ptr(), dt, W, Ep, C, H, Fdim, seg_ws.data_ptr(), segb)
            if sources is None:
                _lib.call("ats_moe_ep_experts_fwd", *args, st)
            elif sources[0] < sources[1]:
                _lib.call("ats_moe_ep_experts_fwd_sources", *args, sources[0], sources[1], st)

        def experts(p):
            experts_run(experts_prep(p))

        cur = torch.cuda.current_stream(dev)
        if parts > 1 and comm_sms > 0:
            # part p+1's rows go out, and part p-1's results come back, on side streams with comm_sms SMs
            # while part p's GEMMs run on the others; each transfer is ordered by its own all-reduce
            out_s, back_s = state.copy_streams(dev, max(W, 2))[:2]
            push(0, 1, 0, cur)
            dist.all_reduce(flag, group=group)
            _mark("exchange_out")
            out_s.wait_stream(cur)
            for t in (x2, row_token, allv, ys, flag):
                t.record_stream(out_s)
                t.record_stream(back_s)
            sms = max(1, torch.cuda.get_device_properties(dev).multi_processor_count - comm_sms)
            for p in range(parts):
                if p + 1 < parts:
                    with torch.cuda.stream(out_s):
                        push(p + 1, p + 2, comm_sms, out_s)
                        dist.all_reduce(flag, group=group)
                with _lib.gemm_sm_limit(sms):
                    experts(p)
                back_s.wait_stream(cur)
                with torch.cuda.stream(back_s):
                    dist.all_reduce(flag, group=group)
                    pull(p, p + 1, comm_sms, back_s)
                if p + 1 < parts:
                    cur.wait_stream(out_s)
            _mark("experts")
            cur.wait_stream(back_s)
            _mark("exchange_back")
        elif parts == 1 and comm_sms > 0 and _OWN_ROWS_FIRST:
            # this rank's rows for its own experts need no transfer: they are stored locally, and their expert
            # GEMMs run on the other SMs while the rows for the other ranks go out (and theirs come in) on a side
            # stream with comm_sms SMs; the other sources' rows follow once the all-reduce says they landed
            def push_split(to_self, sms, stream):
                _lib.call("ats_moe_ep_push_split", x2.data_ptr(), row_token.data_ptr(), T,
                          *_exchange_args(allv, W, me, El, 1, 0, 1, ps.table("xr"), part_rows, H, dt)[:-1],
                          1 if to_self else 0, sms, stream.cuda_stream)

            bufs = experts_prep(0)
            push_split(True, 0, cur)
            side = state.copy_streams(dev, max(W, 2))[0]
            side.wait_stream(cur)
            with torch.cuda.stream(side):
                push_split(False, comm_sms, side)
                dist.all_reduce(flag, group=group)
            for t in (x2, row_token, allv, flag):
                t.record_stream(side)
            nsm = torch.cuda.get_device_properties(dev).multi_processor_count
            with _lib.gemm_sm_limit(max(1, nsm - comm_sms)):
                experts_run(bufs, (me, me + 1))
            _mark("experts_own")
            cur.wait_stream(side)
            _mark("exchange_out")
            experts_run(bufs, (0, me))
            experts_run(bufs, (me + 1, W))
            _mark("experts")
            dist.all_reduce(flag, group=group)
            _mark("exchange_back_flag")
        else:
            push(0, parts, 0, cur)
            _mark("exchange_push")
            dist.all_reduce(flag, group=group)
            _mark("exchange_out")
            for p in range(parts):
                experts(p)
            _mark("experts")
            dist.all_reduce(flag, group=group)
            _mark("exchange_back_flag")
        out = torch.empty((T, H), dtype=x2.dtype, device=dev)
        if parts > 1 and comm_sms > 0:  # the parts' results were pulled on the side stream
            _lib.call("ats_moe_combine", ys.data_ptr(), out.data_ptr(), dt, T, H, E, k, C, L, ws.data_ptr(), wsb,
                      st)
            _mark("combine")
        elif _FUSED_COMBINE:
            # the combine reads the expert outputs straight from the expert ranks' buffers (and keeps the
            # packed copy the backward needs): the pull and the combine in one pass
            _lib.call("ats_moe_ep_combine", ys.data_ptr(), R, out.data_ptr(), T, k, C, ws.data_ptr(), wsb,
                      allv.data_ptr(), W, me, El, parts, ps.table("yr").data_ptr(), part_rows, H, dt, st)
            _mark("exchange_back_combine")
        else:
            pull(0, parts, 0, cur)
            _mark("exchange_back")
            _lib.call("ats_moe_combine", ys.data_ptr(), out.data_ptr(), dt, T, H, E, k, C, L, ws.data_ptr(), wsb,
                      st)
            _mark("combine")
        ctx.save_for_backward(logits, gates, idx, ws, ys, allv, wgu_stack, wd_stack, x2, w32, rws, *keep)
        ctx.meta = (E, El, k, C, lbw, Fdim, W, group, T, H, wsb, R, segb, gate_w.dtype, parts, part_rows, me,
                    comm_sms)
        ctx.ps, ctx.state = ps, state
        if not will_backward:
            state.release(ps)
        ctx.mark_non_differentiable(util, counts, idx)
        return out, aux, util, counts, idx

    @staticmethod
    def backward(ctx, dout, daux, _dutil, _dcounts, _didx):
        logits, gates, idx, ws, ys, allv, wgu_stack, wd_stack, x2, w32, rws, *keep = ctx.saved_tensors
        E, El, k, C, lbw, Fdim, W, group, T, H, wsb, R, segb, gate_dtype, parts, part_rows, me, comm_sms = ctx.meta
        ps, state = ctx.ps, ctx.state
        L = _lib.ATS_MOE_PACKED
        Ep = El // parts
        dev = x2.device
        dt = _lib.dtype_code(x2.dtype)
        st = _lib.stream_of(x2)
        flag = state.flag(dev)
        if dout is None:
            dout = torch.zeros((T, H), dtype=x2.dtype, device=dev)
        dout = dout.to(x2.dtype).contiguous()
        _mark("bwd_start")
        dys = torch.empty((R, H), dtype=x2.dtype, device=dev)
        dgate_row = torch.empty(R, dtype=torch.float32, device=dev)
        _lib.call("ats_moe_combine_bwd", dout.data_ptr(), ys.data_ptr(), dys.data_ptr(), dgate_row.data_ptr(), dt,
                  T, H, E, k, C, L, ws.data_ptr(), wsb, st)
        dlogits = torch.empty((T, E), dtype=torch.float32, device=dev)
        daux_t = daux.to(torch.float32).contiguous() if daux is not None else None

        def route_bwd():  # the routing gradient needs only the gate-row gradients
            _lib.call("ats_moe_route_bwd", logits.data_ptr(), gates.data_ptr(), idx.data_ptr(),
                      dgate_row.data_ptr(), _lib.ptr(daux_t), dlogits.data_ptr(), T, E, k, C, L, float(lbw),
                      ws.data_ptr(), wsb, st)

        cur = torch.cuda.current_stream(dev)
        nsm = torch.cuda.get_device_properties(dev).multi_processor_count
        dgate_w = None
        early_router = comm_sms > 0 and rws is not None and _ROUTER_BESIDE_PUSH
        if early_router:
            # the output-gradient rows go out on a side stream with comm_sms SMs while the router's weight
            # gradient, which needs only the routing gradient, runs on the other SMs
            route_bwd()
            _mark("combine_bwd")
            side = state.copy_streams(dev, W)[0]
            side.wait_stream(cur)
            with torch.cuda.stream(side):
                _lib.call("ats_moe_ep_zero_padding", ps.local["dyr"].data_ptr(), allv.data_ptr(), W, me, El, parts,
                          0, parts, part_rows, H, dt, side.cuda_stream)
                _lib.call("ats_moe_ep_push", dys.data_ptr(), None, R,
                          *_exchange_args(allv, W, me, El, parts, 0, parts, ps.table("dyr"), part_rows, H, dt,
                                          comm_sms), side.cuda_stream)
                dist.all_reduce(flag, group=group)
            for t in (dys, allv, flag):
                t.record_stream(side)
            with _lib.gemm_sm_limit(max(1, nsm - comm_sms)):
                dgate_w = router_weight_grad(dlogits, x2, w32, rws)
            cur.wait_stream(side)
        else:
            _mark("combine_bwd")
            _lib.call("ats_moe_ep_zero_padding", ps.local["dyr"].data_ptr(), allv.data_ptr(), W, me, El, parts, 0,
                      parts, part_rows, H, dt, st)
            _lib.call("ats_moe_ep_push", dys.data_ptr(), None, R,
                      *_exchange_args(allv, W, me, El, parts, 0, parts, ps.table("dyr"), part_rows, H, dt), st)
            dist.all_reduce(flag, group=group)
        _mark("exchange_out_bwd")
        dwgu = torch.empty_like(wgu_stack)
        dwd = torch.empty_like(wd_stack)
        dhs = []

        def expert_bwd(stages):
            for p in range(parts):
                h, a, seg_ws = keep[3 * p:3 * p + 3]
                sl = slice(p * part_rows, (p + 1) * part_rows)
                xr, dyr, dxr = ps.local["xr"][sl], ps.local["dyr"][sl], ps.local["dxr"][sl]
                if stages & 1:
                    dhs.append(torch.empty((part_rows, 2 * Fdim), dtype=x2.dtype, device=dev))
                _lib.call("ats_moe_ep_experts_bwd_staged", dyr.data_ptr(), xr.data_ptr(), h.data_ptr(),
                          a.data_ptr(), wgu_stack[p * Ep].data_ptr(), wd_stack[p * Ep].data_ptr(), dhs[p].data_ptr(),
                          dxr.data_ptr(), dwgu[p * Ep].data_ptr(), dwd[p * Ep].data_ptr(), dt, W, Ep, C, H, Fdim,
                          seg_ws.data_ptr(), segb, stages, st)

        dxs = torch.empty((R, H), dtype=x2.dtype, device=dev)
        if comm_sms > 0:
            # data gradient, then the return transfer on a side stream with comm_sms SMs while the weight
            # gradients run on the others
            expert_bwd(1)
            _mark("experts_bwd_data")
            side = state.copy_streams(dev, W)[0]
            side.wait_stream(cur)
            with torch.cuda.stream(side):
                dist.all_reduce(flag, group=group)
                _lib.call("ats_moe_ep_pull", dxs.data_ptr(), R,
                          *_exchange_args(allv, W, me, El, parts, 0, parts, ps.table("dxr"), part_rows, H, dt,
                                          comm_sms), side.cuda_stream)
            for t in (dxs, allv, flag):
                t.record_stream(side)
            with _lib.gemm_sm_limit(max(1, nsm - comm_sms)):
                expert_bwd(2)
            if not early_router:
                route_bwd()
            _mark("experts_bwd_weights")
            cur.wait_stream(side)
            _mark("exchange_back_bwd")
        else:
            expert_bwd(3)
            route_bwd()
            _mark("experts_bwd")
            dist.all_reduce(flag, group=group)
            _lib.call("ats_moe_ep_pull", dxs.data_ptr(), R,
                      *_exchange_args(allv, W, me, El, parts, 0, parts, ps.table("dxr"), part_rows, H, dt), st)
            _mark("exchange_back_bwd")
        dx, dgate_w = router_backward(dlogits, x2, w32, rws, dxs, ws, wsb, (T, E, k, C, L), True, dw=dgate_w)
        _mark("router_bwd")
        state.release(ps)
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

    ``exchange`` says how rows cross between ranks: "packed" and "slots" are
    NCCL all-to-alls (see ``_Exchange``); "peer" copies the packed rows with
    the copy engines straight into buffers the peers mapped once (CUDA IPC),
    so the transfers take no SMs and run beside the expert GEMMs.
    ``overlap_parts`` P runs the local experts in P parts so that each part's
    row transfers overlap the expert GEMMs of the others (P must divide the
    local expert count; 1 exchanges everything at once); meanwhile the GEMMs
    leave ``comm_sms`` SMs to the collectives (default: 16 for the NCCL
    exchanges, whose transfers run on SMs, none for "peer").  "device" moves
    the rows with kernels of its own; with ``comm_sms`` > 0 (default 16) its
    backward loads the returning input gradients on that many SMs while the
    weight-gradient GEMMs run on the rest."""

    def __init__(self, hidden_size: int, intermediate_size: int, num_experts: int, num_layers: int,
                 top_k: int = 2, capacity_factor: float = 1.25, load_balancing_weight: float = 0.01,
                 group=None, exchange: str = "packed", overlap_parts: int = 1, comm_sms: int | None = None,
                 ep_size: int | None = None) -> None:
        super().__init__()
        if exchange not in ("packed", "slots", "peer", "device"):
            raise ValueError(f"exchange must be 'packed', 'slots', 'peer' or 'device', got {exchange!r}")
        if comm_sms is None:
            comm_sms = 0 if exchange == "peer" else 16
        self.exchange = exchange
        self.group = group
        if ep_size is None:  # the given group (or the default one), bound now
            self.world = dist.get_world_size(group) if dist.is_available() and dist.is_initialized() else 1
            self.rank = dist.get_rank(group) if self.world > 1 else 0
            self._bound = True
        else:  # ep_size ranks, bound at the first forward (the process group may not exist yet)
            if ep_size < 1:
                raise ValueError(f"ep_size must be >= 1, got {ep_size}")
            self.world, self.rank, self._bound = ep_size, 0, ep_size == 1
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
        self._peer = _PeerState()
        self.top_k = top_k
        self.capacity_factor = capacity_factor
        self.load_balancing_weight = load_balancing_weight
        self.gate = nn.Linear(hidden_size, num_experts, bias=False)
        self.experts = nn.ModuleList([SwiGLU(hidden_size, intermediate_size) for _ in range(self.num_local_experts)])
        for ex in self.experts:
            init_residual_projection(ex.down_proj, num_layers)
        self.last_expert_utilization: dict[int, float] | None = None
        self.last_counts: torch.Tensor | None = None

    def _bind(self) -> None:
        """Resolve the expert-parallel group of an ``ep_size`` layer: the default
        group when its size is ep_size, else groups of ep_size consecutive ranks
        (every rank creates all of them, in the same order, at its first forward)."""
        if self._bound:
            return
        if not (dist.is_available() and dist.is_initialized()):
            raise RuntimeError(f"MoELayer(ep_size={self.world}) needs torch.distributed initialised before its "
                               f"first forward. Fix: launch with torchrun and init the process group, or use "
                               f"ep_size=1.")
        ws, me = dist.get_world_size(), dist.get_rank()
        if ws % self.world != 0:
            raise ValueError(f"ep_size={self.world} must divide the world size {ws}")
        if ws != self.world:
            for i in range(ws // self.world):
                g = dist.new_group(list(range(i * self.world, (i + 1) * self.world)))
                if i == me // self.world:
                    self.group = g
        self.rank = dist.get_rank(self.group)
        self._bound = True

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
        self._bind()
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
        if self.world == 1 or self.comm_sms == 0 or (self.overlap_parts == 1 and self.exchange != "peer"):
            return 0
        return max(1, torch.cuda.get_device_properties(device).multi_processor_count - self.comm_sms)

    def release_peer_buffers(self) -> None:
        """Unmap the peers' exchange buffers (exchange="peer"; every rank, together,
        with no forward waiting for its backward).  The next forward maps new ones."""
        if self.world > 1 and self._peer.sets:
            torch.cuda.synchronize()
            dist.barrier(group=self.group)
        self._peer.close()

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
        self._bind()
        flat = x.reshape(-1, H).contiguous()
        T = flat.shape[0]
        cap = capacity_for(T, self.top_k, self.num_experts, self.capacity_factor)
        wgu = [e.gate_up_proj.weight for e in self.experts]
        wd = [e.down_proj.weight for e in self.experts]
        if wgu[0].dtype != flat.dtype:
            raise TypeError(f"MoE: token dtype {flat.dtype} does not match expert weight dtype {wgu[0].dtype}")
        bias = logit_bias.detach().float().contiguous() if logit_bias is not None else None
        head = (self.num_experts, self.num_local_experts, self.top_k, cap, self.load_balancing_weight,
                wgu[0].shape[0] // 2, self.world, self.group)
        if self.exchange == "device" and self.world > 1:
            will_backward = torch.is_grad_enabled() and (flat.requires_grad or any(
                p.requires_grad for p in self.parameters()))
            meta = head + (self.overlap_parts, self.comm_sms, self._peer, self.rank, will_backward)
            fn = _EPDeviceFn
        elif self.exchange == "peer" and self.world > 1:
            will_backward = torch.is_grad_enabled() and (flat.requires_grad or any(
                p.requires_grad for p in self.parameters()))
            meta = head + (self.overlap_parts, self._gemm_sms(flat.device), self._peer, self.rank, will_backward)
            fn = _EPPeerFn
        else:
            mode = "packed" if self.exchange in ("peer", "device") else self.exchange
            meta = head + (mode, self.overlap_parts, self._gemm_sms(flat.device))
            fn = _EPMoEFn
        out, aux, util, counts, _ = fn.apply(flat, self.gate.weight, bias, meta, stacked(wgu), stacked(wd), *wgu, *wd)
        self.last_expert_utilization = LazyUtilization(util)
        self.last_counts = counts
        return out.view(batch, seq, H), aux

"""Expert-parallel exchange on CPU with two gloo ranks (no GPU).

The row and count exchanges of the expert-parallel MoE only move tensors;
here they run on CPU tensors: every row of a send buffer carries its
(source rank, global expert, slot) so the receiver can check where it landed,
a stand-in expert doubles the rows, and the return exchange must bring each
row back to its original slot.  The packed exchange (variable splits of
back-to-back expert segments) gets the same check, and also that only the
kept rows and their padding to 128 travel; so does the exchange in parts
(per-peer sends of each part's row runs, all parts in flight at once).  A last test makes one rank leave before the
collective: its peer must fail within the process group's timeout instead of
waiting for ever."""

from __future__ import annotations

import os
import socket
import traceback
from datetime import timedelta

import pytest
import torch
import torch.distributed as dist
import torch.multiprocessing as mp

import numpy as np

from ats_v2_b200.ep import (ExpertParallelMoE, _Exchange, balanced_placement, exchange_counts, exchange_rows, peer_plan,
                            slot_rows)


def _free_port() -> int:
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _init(rank, world, port, timeout_s=60):
    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    dist.init_process_group("gloo", rank=rank, world_size=world, timeout=timedelta(seconds=timeout_s))


def _exchange_worker(rank, world, port, E_local, cap, H, errq):
    try:
        _init(rank, world, port)
        E = world * E_local
        Cp = slot_rows(cap)
        g = torch.Generator().manual_seed(rank)
        kept = torch.randint(0, cap + 1, (E,), generator=g, dtype=torch.int32)
        send = torch.zeros(E * Cp, H)
        for e in range(E):
            for s in range(int(kept[e])):
                send[e * Cp + s, 0] = rank
                send[e * Cp + s, 1] = e
                send[e * Cp + s, 2] = s
                send[e * Cp + s, 3:] = 1.0
        recv_kept = exchange_counts(kept)
        recv = exchange_rows(send)
        # what every source keeps for my experts, in [source][local expert] order
        all_kept = [torch.empty_like(kept) for _ in range(world)]
        dist.all_gather(all_kept, kept)
        for src in range(world):
            for el in range(E_local):
                e = rank * E_local + el
                assert int(recv_kept[src * E_local + el]) == int(all_kept[src][e])
                for s in range(int(all_kept[src][e])):
                    row = recv[(src * E_local + el) * Cp + s]
                    assert (int(row[0]), int(row[1]), int(row[2])) == (src, e, s)
        back = exchange_rows(recv * 2.0)  # a stand-in expert, then the return trip
        assert torch.equal(back, send * 2.0)
        dist.barrier()
        dist.destroy_process_group()
    except Exception:
        errq.put((rank, traceback.format_exc()))
        raise


def _parts_worker(rank, world, port, mode, parts, E_local, cap, H, errq):
    """Exchange in parts: part p carries the rows of local experts
    [p*E_local/P, (p+1)*E_local/P) of every rank.  Packed: each rank's experts
    are back-to-back segments of align128(kept) rows and only those rows
    travel; slots: the [E][Cp] buffer.  Each part's expert-side buffer must
    hold its (source, expert) segments in that order, and the return trip must
    put every row back where it left from."""
    try:
        _init(rank, world, port)
        E = world * E_local
        Cp = slot_rows(cap)
        Ep = E_local // parts
        g = torch.Generator().manual_seed(10 + rank)
        kept = torch.randint(0, cap + 1, (E,), generator=g, dtype=torch.int32)
        if mode == "packed":
            pad = [(int(c) + 127) // 128 * 128 for c in kept]
        else:
            pad = [Cp] * E
        seg_start = torch.tensor([0] + list(torch.tensor(pad).cumsum(0)), dtype=torch.int32)
        R = int(seg_start[-1])
        send = torch.zeros(max(R, 1), H)
        for e in range(E):
            for s in range(int(kept[e])):
                send[int(seg_start[e]) + s, :3] = torch.tensor([rank, e, s], dtype=torch.float32)
                send[int(seg_start[e]) + s, 3:] = 1.0
        recv_kept = exchange_counts(kept)
        ex = _Exchange(mode, world, E_local, Cp, None, seg_start, recv_kept, parts)
        assert (ex.parts, ex.Ep) == (parts, Ep)
        pending = [ex.out(send, p) for p in range(parts)]  # every part in flight at once
        back = torch.zeros_like(send)
        for p in range(parts):
            recv, arrived = pending[p]
            arrived.wait()
            assert recv.shape[0] == world * Ep * Cp
            row = 0
            for src in range(world):
                for el in range(p * Ep, (p + 1) * Ep):
                    e = rank * E_local + el
                    c = int(recv_kept[src * E_local + el])
                    for s in range(c):
                        got = recv[row + s]
                        assert (int(got[0]), int(got[1]), int(got[2])) == (src, e, s)
                    span = (c + 127) // 128 * 128 if mode == "packed" else Cp
                    assert bool((recv[row + c:row + span] == 0).all())  # padding rows are zero
                    row += span
            if mode == "packed" or parts > 1:
                assert row == sum(n for _, n in ex.recv[p])
            back, returned = ex.back(recv * 2.0, back, p)  # a stand-in expert, then the return trip
            returned.wait()
        assert torch.equal(back[:R], send[:R] * 2.0)
        dist.barrier()
        dist.destroy_process_group()
    except Exception:
        errq.put((rank, traceback.format_exc()))
        raise


def _rebalance_worker(rank, world, port, errq):
    """Every expert's weights carry its label; after rebalance each rank must
    hold exactly the experts the permutation gives it, with their weights and
    gate rows."""
    try:
        _init(rank, world, port)
        E, H, F = 8, 16, 8
        El = E // world
        m = ExpertParallelMoE(H, F, E, num_layers=2, top_k=2)
        with torch.no_grad():
            for e in range(E):
                m.gate.weight[e].fill_(float(e))
            for i, ex in enumerate(m.experts):
                ex.gate_up_proj.weight.fill_(float(rank * El + i))
                ex.down_proj.weight.fill_(100.0 + rank * El + i)
        load = torch.tensor([1.0, 1.0, 9.0, 8.0, 1.0, 1.0, 1.0, 1.0])  # experts 2 and 3 are hot
        perm = m.rebalance(load).tolist()
        assert sorted(perm) == list(range(E))
        assert perm == balanced_placement(load.tolist(), world)
        for j in range(E):
            assert bool((m.gate.weight[j] == float(perm[j])).all())
        for i, ex in enumerate(m.experts):
            old = perm[rank * El + i]
            assert bool((ex.gate_up_proj.weight == float(old)).all())
            assert bool((ex.down_proj.weight == 100.0 + old).all())
        hot = {2, 3}
        assert len(hot & set(perm[:El])) == 1 and len(hot & set(perm[El:])) == 1  # one hot expert per rank
        dist.barrier()
        dist.destroy_process_group()
    except Exception:
        errq.put((rank, traceback.format_exc()))
        raise


def _agree_worker(rank, world, port, errq):
    try:
        _init(rank, world, port)
        from ats_v2_b200.ep import _PeerState
        mine = [[1, 0, 1, 1], [1, 1, 0, 1]][rank]
        assert _PeerState._agree(mine, None, "cpu") == [1, 0, 0, 1]
        dist.barrier()
        dist.destroy_process_group()
    except Exception:
        errq.put((rank, traceback.format_exc()))
        raise


def test_orphan_masks_agree_over_ranks():
    ctx = mp.get_context("spawn")
    errq = ctx.SimpleQueue()
    mp.start_processes(_agree_worker, args=(2, _free_port(), errq), nprocs=2, join=True, start_method="spawn")
    assert errq.empty()


def _leaver_worker(rank, world, port, errq):
    try:
        _init(rank, world, port, timeout_s=3)
        buf = torch.ones(world * 4, 8)
        if rank == 1:
            return  # leaves before the collective: no NCCL/GPU involved
        try:
            exchange_rows(buf)
        except Exception as exc:  # the peer's timeout or lost connection
            errq.put((rank, f"raised: {type(exc).__name__}"))
            return
        errq.put((rank, "no error"))
    except Exception:
        errq.put((rank, traceback.format_exc()))


@pytest.mark.parametrize("E_local,cap,H", [(2, 5, 8), (3, 130, 4)])
def test_row_and_count_exchange_round_trip(E_local, cap, H):
    ctx = mp.get_context("spawn")
    errq = ctx.SimpleQueue()
    mp.start_processes(_exchange_worker, args=(2, _free_port(), E_local, cap, H, errq), nprocs=2, join=True,
                       start_method="spawn")
    assert errq.empty()


@pytest.mark.parametrize("mode,parts,world,E_local,cap,H", [("packed", 1, 2, 2, 5, 8), ("packed", 1, 2, 3, 300, 4),
                                                           ("packed", 2, 2, 4, 300, 4), ("slots", 2, 2, 2, 5, 8),
                                                           ("packed", 3, 3, 3, 130, 4)])
def test_exchange_in_parts_sends_only_kept_segments_and_round_trips(mode, parts, world, E_local, cap, H):
    ctx = mp.get_context("spawn")
    errq = ctx.SimpleQueue()
    mp.start_processes(_parts_worker, args=(world, _free_port(), mode, parts, E_local, cap, H, errq), nprocs=world,
                       join=True, start_method="spawn")
    assert errq.empty()


@pytest.mark.parametrize("W,El,parts,cap", [(2, 4, 2, 300), (3, 2, 1, 5), (4, 2, 2, 130), (8, 8, 4, 257),
                                            (2, 1, 1, 1)])
def test_peer_copy_plan_builds_the_packed_expert_side_layout(W, El, parts, cap):
    """Every rank's copy plan, applied to simulated buffers of all ranks, must
    give each part of each rank's expert side the (source, expert) segments
    in order -- the layout the NCCL packed exchange delivers and the segment
    table reads -- and the return copies must bring every row home."""
    E = W * El
    Cp = slot_rows(cap)
    Ep = El // parts
    part_rows = W * Ep * Cp
    rng = np.random.default_rng(W * 100 + El * 10 + parts)
    kept = rng.integers(0, cap + 1, size=(W, E))
    kept[0, :El] = 0  # a source that keeps nothing for rank 0's experts
    rnd = (np.minimum(kept, Cp) + 127) // 128 * 128
    xs = []
    for s_ in range(W):
        seg0 = np.concatenate([[0], np.cumsum(rnd[s_])])
        buf = np.zeros((max(int(seg0[-1]), 1), 3), dtype=np.int64)
        for e in range(E):
            for r in range(int(kept[s_, e])):
                buf[seg0[e] + r] = (s_ + 1, e + 1, r + 1)
        xs.append(buf)
    plans = [peer_plan(kept.tolist(), Cp, El, parts, me) for me in range(W)]
    xr = [np.full((W * El * Cp, 3), -1, dtype=np.int64) for _ in range(W)]
    for me in range(W):
        seg, out, _ = plans[me]
        assert seg[me] == [0] + np.cumsum(rnd[me]).tolist()
        for p in range(parts):
            for d, src, dst, n in out[p]:
                assert n > 0 and src + n <= xs[me].shape[0] and dst + n <= part_rows
                xr[d][p * part_rows + dst:p * part_rows + dst + n] = xs[me][src:src + n]
    for d in range(W):
        for p in range(parts):
            row = p * part_rows
            for src in range(W):
                for i in range(p * Ep, (p + 1) * Ep):
                    e = d * El + i
                    c = int(kept[src, e])
                    for r in range(c):
                        assert tuple(xr[d][row + r]) == (src + 1, e + 1, r + 1)
                    assert (xr[d][row + c:row + int(rnd[src, e])] == 0).all()  # padding rows arrive as zeros
                    row += int(rnd[src, e])
    ys = [np.full_like(b, -1) for b in xs]
    for me in range(W):
        _, _, back = plans[me]
        for p in range(parts):
            for s_, src, dst, n in back[p]:
                ys[s_][dst:dst + n] = 2 * xr[me][p * part_rows + src:p * part_rows + src + n]
    for s_ in range(W):
        n = int(rnd[s_].sum())
        assert (ys[s_][:n] == 2 * xs[s_][:n]).all()


def test_peer_buffer_pool_reuses_free_sets_and_bounds_waiting_forwards(monkeypatch):
    """The pool behind exchange="peer": a forward takes a free set that fits,
    else maps a new one (dropping free sets that no longer fit); a backward
    gives its set back; forwards waiting for their backward are bounded."""
    from ats_v2_b200 import ep as epm

    made, closed = [], []

    class FakeSet:
        def __init__(self, rows_x, rows_t, H, dtype, device, group, W, me, names=None, expert_side=None):
            self.rows_x, self.rows_t, self.H, self.dtype = rows_x, rows_t, H, dtype
            self.busy = False
            self.owner = None
            made.append(self)

        def fits(self, rows_x, rows_t, H, dtype):
            return rows_x <= self.rows_x and rows_t <= self.rows_t and H == self.H and dtype == self.dtype

        def close(self):
            closed.append(self)

    monkeypatch.setattr(epm, "_PeerSet", FakeSet)
    st = epm._PeerState()
    monkeypatch.setattr(st, "_agree", lambda mask, group, device: mask)  # one rank: its own mask
    args = (None, None, 2, 0)
    a = st.acquire(1024, 512, 64, torch.bfloat16, *args)
    assert a.busy and made == [a]
    st.release(a)
    assert st.acquire(1000, 500, 64, torch.bfloat16, *args) is a  # smaller sizes fit the free set
    b = st.acquire(1024, 512, 64, torch.bfloat16, *args)  # a is busy: a second set
    assert b is not a and len(made) == 2
    st.release(a)
    st.release(b)
    c = st.acquire(4096, 512, 64, torch.bfloat16, *args)  # grown: free sets that no longer fit are unmapped
    assert closed == [a, b] and st.sets == [c]
    for _ in range(epm._PeerState.MAX_SETS - 1):
        st.acquire(4096, 512, 64, torch.bfloat16, *args)
    with pytest.raises(RuntimeError, match="waiting for their backward"):
        st.acquire(4096, 512, 64, torch.bfloat16, *args)
    st.close()
    assert st.sets == [] and len(closed) == 2 + epm._PeerState.MAX_SETS


def test_peer_buffer_sets_of_dropped_graphs_come_back_only_when_every_rank_agrees(monkeypatch):
    """Activation checkpointing recomputes a forward inside the backward and
    drops that graph, so its set is never released by a backward.  When no
    free set fits, sets whose forward's context is gone are taken back --
    only those orphaned on every rank (a minimum over the ranks' masks)."""
    import gc
    import weakref

    from ats_v2_b200 import ep as epm

    class FakeSet:
        def __init__(self, rows_x, rows_t, H, dtype, device, group, W, me, names=None, expert_side=None):
            self.rows_x, self.rows_t, self.H, self.dtype = rows_x, rows_t, H, dtype
            self.busy = False
            self.owner = None

        def fits(self, rows_x, rows_t, H, dtype):
            return rows_x <= self.rows_x and rows_t <= self.rows_t and H == self.H and dtype == self.dtype

        def close(self):
            pass

    class Ctx:  # stands in for an autograd context
        pass

    monkeypatch.setattr(epm, "_PeerSet", FakeSet)
    st = epm._PeerState()
    other_rank = {"mask": None}
    seen = []

    def agree(mask, group, device):
        seen.append(list(mask))
        peer = other_rank["mask"] if other_rank["mask"] is not None else mask
        return [min(a, b) for a, b in zip(mask, peer)]

    monkeypatch.setattr(st, "_agree", agree)
    shape = (1024, 512, 64, torch.bfloat16, None, None, 2, 0)
    kept, dropped = Ctx(), Ctx()
    a = st.acquire(*shape)
    a.owner = weakref.ref(kept)       # the original forward: its backward will run
    b = st.acquire(*shape)
    b.owner = weakref.ref(dropped)    # the recomputed forward: its graph is dropped
    assert seen == [[0]]              # b's acquire asked, but a's context is alive
    del dropped
    gc.collect()
    other_rank["mask"] = [0, 0]       # another rank still holds b's graph: nothing comes back
    c = st.acquire(*shape)
    assert c is not b and len(st.sets) == 3 and b.busy
    other_rank["mask"] = None         # every rank has dropped it
    d = st.acquire(*shape)
    assert d is b and seen[-1] == [0, 1, 0]
    st.release(a)
    assert st.acquire(*shape) is a    # a free set is taken without asking the other ranks
    assert len(seen) == 3


def test_balanced_placement_spreads_the_load():
    load = [float(2 ** (-i)) for i in range(16)]  # one expert far hotter than the rest
    for world in (1, 2, 4, 8):
        perm = balanced_placement(load, world)
        el = 16 // world
        assert sorted(perm) == list(range(16))
        ranks = [perm[r * el:(r + 1) * el] for r in range(world)]
        assert all(b == sorted(b) for b in ranks)
        per = [sum(load[e] for e in b) for b in ranks]
        contiguous = [sum(load[r * el:(r + 1) * el]) for r in range(world)]
        assert max(per) <= max(contiguous) + 1e-12
    assert balanced_placement(load, 1) == list(range(16))  # one rank: nothing moves
    with pytest.raises(ValueError):
        balanced_placement(load, 3)


def test_rebalance_moves_gate_rows_and_expert_weights_between_ranks():
    ctx = mp.get_context("spawn")
    errq = ctx.SimpleQueue()
    mp.start_processes(_rebalance_worker, args=(2, _free_port(), errq), nprocs=2, join=True, start_method="spawn")
    assert errq.empty()


def test_peer_that_leaves_makes_the_collective_fail_not_hang():
    ctx = mp.get_context("spawn")
    errq = ctx.SimpleQueue()
    port = _free_port()
    procs = [ctx.Process(target=_leaver_worker, args=(r, 2, port, errq)) for r in range(2)]
    for p in procs:
        p.start()
    for p in procs:
        p.join(timeout=60)
    alive = [p for p in procs if p.is_alive()]
    for p in alive:
        p.kill()
    assert not alive, "a rank hung past the timeout"
    results = []
    while not errq.empty():
        results.append(errq.get())
    assert any(r == 0 and msg.startswith("raised") for r, msg in results), results


def test_peer_copy_plan_invariants_over_random_layouts():
    """Property check of ``peer_plan`` (it decides where the copy engines write
    into other GPUs' memory): over random world sizes, parts and kept counts,
    every rank's token rows leave exactly once, every part buffer of every
    rank is tiled by the incoming runs without gaps or overlaps and stays
    within W*Ep*Cp rows, and the return runs mirror the outgoing ones."""
    from hypothesis import given, settings
    from hypothesis import strategies as st

    @settings(max_examples=200, deadline=None)
    @given(st.data())
    def check(data):
        W = data.draw(st.sampled_from([1, 2, 3, 4, 8]))
        El = data.draw(st.sampled_from([1, 2, 4, 6, 8]))
        parts = data.draw(st.sampled_from([p for p in (1, 2, 3, 4) if El % p == 0]))
        cap = data.draw(st.integers(1, 700))
        Cp = slot_rows(cap)
        E = W * El
        kept = [[data.draw(st.integers(0, cap)) for _ in range(E)] for _ in range(W)]
        Ep = El // parts
        part_rows = W * Ep * Cp
        plans = [peer_plan(kept, Cp, El, parts, me) for me in range(W)]
        incoming = {(d, p): [] for d in range(W) for p in range(parts)}
        for me, (seg, out, back) in enumerate(plans):
            sent = []
            for p in range(parts):
                for d, src, dst, n in out[p]:
                    assert n > 0 and 0 <= dst and dst + n <= part_rows
                    sent.append((src, src + n))
                    incoming[(d, p)].append((dst, dst + n, me, src))
            sent.sort()
            covered = 0
            for a, b in sent:  # the runs cover [0, seg[me][E]) exactly once
                assert a == covered
                covered = b
            assert covered == seg[me][E]
        for (d, p), runs in incoming.items():
            runs.sort()
            pos = 0
            for a, b, src_rank, _ in runs:  # sources in rank order, back to back from row 0
                assert a == pos
                pos = b
            assert pos <= part_rows
            back = sorted(plans[d][2][p])
            mirror = sorted((s_, a, src, b - a) for a, b, s_, src in runs)
            assert [(s_, srow, drow, n) for s_, srow, drow, n in back] == \
                   [(s_, a, src, n) for s_, a, src, n in mirror]

    check()

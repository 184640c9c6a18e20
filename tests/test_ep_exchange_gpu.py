"""The device-driven row exchange kernels (``ats_moe_ep_push``, ``_push_split``,
``_pull``, ``_zero_padding``, ``_combine``) on one GPU, with W ranks emulated by
W buffers.

Each emulated rank holds kept rows in the packed layout (segment sizes its
kept counts rounded up to 128) and an expert-side buffer.  Every rank pushes
into the buffers (the address table names all of them, as the IPC mappings
do across processes), and afterwards every buffer must equal the layout the
copy plan ``peer_plan`` describes -- the layout ``ats_moe_ep_segments``
reads -- with zero padding rows; pulling back must return each rank's kept
rows.  No kernel waits on another: the emulated ranks run one after another
on one stream.
"""

from __future__ import annotations

import ctypes

import numpy as np
import pytest
import torch

from ats_v2_b200 import _lib
from ats_v2_b200.ep import peer_plan

pytestmark = pytest.mark.gpu


def _counts(W, E, C, seed):
    rng = np.random.default_rng(seed)
    Cp = (C + 127) // 128 * 128
    kept = rng.integers(0, C + 1, size=(W, E))
    kept[rng.random((W, E)) < 0.2] = 0  # empty segments
    rows = []
    for s in range(W):
        rnd = [(int(c) + 127) // 128 * 128 for c in kept[s]]
        seg = np.concatenate([[0], np.cumsum(rnd)]).astype(np.int64)
        R = int(seg[-1]) + 128  # a few rows to spare, as the plan's upper bound has
        rows.append(np.concatenate([kept[s], [Cp, R], seg]).astype(np.int32))
    return kept, Cp, np.stack(rows)


@pytest.mark.parametrize("W,El,parts,C,H,tokens", [(2, 4, 1, 300, 256, False), (4, 2, 2, 200, 512, True),
                                                   (8, 8, 2, 130, 128, False), (3, 3, 3, 64, 256, True)])
def test_push_pull_and_padding_match_the_copy_plan(W, El, parts, C, H, tokens):
    E = W * El
    Ep = El // parts
    kept, Cp, allv = _counts(W, E, C, seed=W * 100 + El)
    part_rows = W * Ep * Cp
    dev = torch.device("cuda")
    g = torch.Generator(device=dev).manual_seed(0)
    counts = torch.from_numpy(allv).to(dev)
    bufs = [torch.full((parts * part_rows, H), float("nan"), device=dev).bfloat16() for _ in range(W)]
    table = torch.tensor([b.data_ptr() for b in bufs], dtype=torch.int64, device=dev)
    st = torch.cuda.current_stream().cuda_stream
    srcs, toks, row_tok = [], [], []
    for s in range(W):
        R = int(allv[s, E + 1])
        if tokens:  # rows come from token rows through row_token (-1 on padding rows)
            T = 1000
            x = torch.randn(T, H, device=dev, generator=g).bfloat16()
            rt = torch.full((R,), -1, dtype=torch.int32)
            seg = allv[s, E + 2:]
            for e in range(E):
                n = int(min(kept[s, e], C))
                rt[int(seg[e]):int(seg[e]) + n] = torch.randint(0, T, (n,), dtype=torch.int32)
            rt = rt.to(dev)
            src = x[rt.clamp(min=0).long()]
            toks.append(x)
            row_tok.append(rt)
        else:
            src = torch.randn(R, H, device=dev, generator=g).bfloat16()
        srcs.append(src)
    for d in range(W):
        _lib.call("ats_moe_ep_zero_padding", bufs[d].data_ptr(), counts.data_ptr(), W, d, El, parts, 0, parts,
                  part_rows, H, _lib.ATS_BF16, st)
    for s in range(W):
        if tokens:
            src_args = (toks[s].data_ptr(), row_tok[s].data_ptr(), toks[s].shape[0])
        else:
            src_args = (srcs[s].data_ptr(), None, srcs[s].shape[0])
        xargs = (counts.data_ptr(), W, s, El, parts, 0, parts, table.data_ptr(), part_rows, H, _lib.ATS_BF16)
        if s % 2:  # the rows for the rank itself, then the others' (ats_moe_ep_push_split): one push together
            for to_self in (1, 0):
                _lib.call("ats_moe_ep_push_split", *src_args, *xargs, to_self, 0, st)
        else:
            _lib.call("ats_moe_ep_push", *src_args, *xargs, 0, st)
    torch.cuda.synchronize()
    code = ctypes.c_int(0)
    assert _lib.query("ats_device_status", ctypes.byref(code)) == 0 and code.value == 0
    kl = [[int(v) for v in row] for row in kept]
    for d in range(W):
        _, _, back = peer_plan(kl, Cp, El, parts, d)
        got = bufs[d].float().cpu()
        for p in range(parts):
            filled = torch.zeros(part_rows, dtype=torch.bool)
            for s, off, src_row, n in back[p]:
                # the segments of source s for d's part p, in expert order: kept rows then zero padding
                seg = allv[s, E + 2:]
                for j in range(Ep):
                    e = d * El + p * Ep + j
                    rows = int(seg[e + 1] - seg[e])
                    nk = int(min(kept[s, e], C))
                    a = p * part_rows + off + int(seg[e]) - src_row
                    assert torch.equal(got[a:a + nk], srcs[s][int(seg[e]):int(seg[e]) + nk].float().cpu())
                    assert torch.count_nonzero(got[a + nk:a + rows]) == 0
                    filled[a - p * part_rows:a - p * part_rows + rows] = True
            assert int(filled.sum()) == sum(n for _, _, _, n in back[p])
    # pull every rank's kept rows back
    for s in range(W):
        R = int(allv[s, E + 1])
        out = torch.zeros(R, H, device=dev).bfloat16()
        _lib.call("ats_moe_ep_pull", out.data_ptr(), R, counts.data_ptr(), W, s, El, parts, 0, parts,
                  table.data_ptr(), part_rows, H, _lib.ATS_BF16, 16 if s % 2 else 0, st)
        torch.cuda.synchronize()
        seg = allv[s, E + 2:]
        for e in range(E):
            nk = int(min(kept[s, e], C))
            a = int(seg[e])
            assert torch.equal(out[a:a + nk], srcs[s][a:a + nk])
    assert _lib.query("ats_device_status", ctypes.byref(code)) == 0


def test_unequal_capacities_are_refused_on_the_device():
    W, El, H = 2, 2, 128
    E = W * El
    kept, Cp, allv = _counts(W, E, 100, seed=7)
    allv[1, E] = Cp + 128  # rank 1 claims another slot size
    dev = torch.device("cuda")
    counts = torch.from_numpy(allv).to(dev)
    part_rows = W * El * Cp
    bufs = [torch.zeros(part_rows + 256, H, device=dev).bfloat16() for _ in range(W)]
    table = torch.tensor([b.data_ptr() for b in bufs], dtype=torch.int64, device=dev)
    src = torch.randn(int(allv[0, E + 1]), H, device=dev).bfloat16()
    _lib.call("ats_moe_ep_push", src.data_ptr(), None, src.shape[0], counts.data_ptr(), W, 0, El, 1, 0, 1,
              table.data_ptr(), part_rows, H, _lib.ATS_BF16, 0, torch.cuda.current_stream().cuda_stream)
    torch.cuda.synchronize()
    assert all(torch.count_nonzero(b) == 0 for b in bufs)  # nothing moved
    code = ctypes.c_int(0)
    assert _lib.query("ats_device_status", ctypes.byref(code)) == _lib.ATS_EBADARG and code.value == 1
    assert _lib.query("ats_device_status", ctypes.byref(code)) == 0


@pytest.mark.parametrize("W,El,parts,T,H,k,cf", [(2, 4, 1, 700, 256, 2, 1.25), (4, 2, 2, 500, 128, 2, 1.0),
                                                 (3, 2, 1, 300, 512, 3, 2.0)])
def test_fused_combine_equals_pull_then_combine(W, El, parts, T, H, k, cf):
    """``ats_moe_ep_combine`` (the combine reading the expert outputs straight from
    the expert ranks' buffers) against ``ats_moe_ep_pull`` followed by
    ``ats_moe_combine``: the same output bit for bit, and the same packed copy of
    every kept row.  W ranks emulated by W routing plans and W expert-side
    buffers of random expert outputs on one GPU."""
    from ats_v2_b200.ep import _route, _row_tokens
    from ats_v2_b200.moe import capacity_for

    E = W * El
    Ep = El // parts
    L = _lib.ATS_MOE_PACKED
    C = capacity_for(T, k, E, cf)
    Cp = (C + 127) // 128 * 128
    part_rows = W * Ep * Cp
    dev = torch.device("cuda")
    g = torch.Generator(device=dev).manual_seed(W * 10 + El)
    st = torch.cuda.current_stream().cuda_stream
    ranks = []
    for s in range(W):
        x = torch.randn(T, H, device=dev, generator=g).bfloat16()
        gate_w = 0.05 * torch.randn(E, H, device=dev, generator=g)
        (_, _, _, ws, wsb, R, _, _, _, _, _, kept, seg_start) = _route(x, gate_w, None, E, k, C, L, 0.01)
        mine = torch.cat([kept, torch.tensor([Cp, R], dtype=torch.int32, device=dev), seg_start])
        ranks.append((ws, wsb, R, mine, _row_tokens(ws, wsb, T, E, k, C, L, R, dev)))
    allv = torch.stack([r[3] for r in ranks]).contiguous()
    yr = [torch.randn(parts * part_rows, H, device=dev, generator=g).bfloat16() for _ in range(W)]
    table = torch.tensor([b.data_ptr() for b in yr], dtype=torch.int64, device=dev)
    for me, (ws, wsb, R, _, row_token) in enumerate(ranks):
        ys1 = torch.zeros(R, H, device=dev).bfloat16()
        _lib.call("ats_moe_ep_pull", ys1.data_ptr(), R, allv.data_ptr(), W, me, El, parts, 0, parts,
                  table.data_ptr(), part_rows, H, _lib.ATS_BF16, 0, st)
        out1 = torch.empty(T, H, device=dev).bfloat16()
        _lib.call("ats_moe_combine", ys1.data_ptr(), out1.data_ptr(), _lib.ATS_BF16, T, H, E, k, C, L,
                  ws.data_ptr(), wsb, st)
        ys2 = torch.zeros(R, H, device=dev).bfloat16()
        out2 = torch.empty(T, H, device=dev).bfloat16()
        _lib.call("ats_moe_ep_combine", ys2.data_ptr(), R, out2.data_ptr(), T, k, C, ws.data_ptr(), wsb,
                  allv.data_ptr(), W, me, El, parts, table.data_ptr(), part_rows, H, _lib.ATS_BF16, st)
        torch.cuda.synchronize()
        assert torch.equal(out1, out2), f"rank {me}: fused combine differs"
        kept_rows = row_token >= 0
        assert int(kept_rows.sum()) > 0
        assert torch.equal(ys1[kept_rows], ys2[kept_rows]), f"rank {me}: packed copy differs"
    code = ctypes.c_int(0)
    assert _lib.query("ats_device_status", ctypes.byref(code)) == _lib.ATS_OK and code.value == 0

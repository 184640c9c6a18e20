"""Oracle for the MoE layer: router, permutation, SwiGLU experts, combine,
auxiliary loss, forward and backward (test-only).

Reference (``ats/model/moe.py``, the single-process _PyTorchMoEFallback):
  * ``:76-90``   compute_routing: softmax(logits) -> topk(k) -> renormalise.
  * ``:103-105`` capacity = max(1, int(capacity_factor * T * k / E)).
  * ``:109-116`` per expert e in ascending order: tokens t (ascending) with
                 e in idx[t]; the first `capacity` are kept, the rest dropped.
  * ``:117-122`` expert FFN on the kept rows, gate weight of that slot,
                 ``output.index_add_(0, tokens, expert_output * weight)``.
  * ``:138-144`` Switch aux loss E * sum(mean(probs) * dispatch_fraction) * lbw.
  * ``:157-162`` utilization = dispatch_fraction / max(sum, 1e-8).
  * ``ats/model/ffn.py:37-45`` SwiGLU: [gate, up] = chunk(x Wgu^T, 2);
                 down(silu(gate) * up).
  * ``ats/model/moe_triton.py:121-127`` _pytorch_moe_routing (same routing math).

Numerics.  The router runs in float32 (router weights and logits are
float32).  Experts run in ``compute`` dtype ("bf16" or "f32"): every torch op
of the reference rounds its result to that dtype, and so does the oracle
(gate_up, silu, the product, down_proj).  The combine casts
``expert_output * weight`` to the output dtype before ``index_add_`` (a
bfloat16 buffer cannot take a float32 source) and accumulates in that dtype
in ascending expert order.

Top-k tie rule.  Softmax is monotone in the logits, so ranking by probability
equals ranking by logit; the oracle ranks by logit, descending, and breaks
exact ties by the lower expert index (a stable sort).
"""

from __future__ import annotations

import numpy as np

from oracle.bf16 import round_to


def softmax_f32(logits) -> np.ndarray:
    """Row softmax in float32: exp(l - max) / sum (moe.py:87)."""
    l32 = np.asarray(logits, dtype=np.float32)
    m = np.max(l32, axis=-1, keepdims=True)
    e = np.exp((l32 - m).astype(np.float64)).astype(np.float32)
    return (e / np.sum(e, axis=-1, keepdims=True, dtype=np.float32)).astype(np.float32)


def topk_order(logits, k: int) -> np.ndarray:
    """Indices of the k largest logits per row, descending, ties -> lower index."""
    l32 = np.asarray(logits, dtype=np.float32)
    return np.argsort(-l32, axis=-1, kind="stable")[:, :k].astype(np.int64)


def route(logits, k: int):
    """(gates[T,k] f32, idx[T,k] int64, probs[T,E] f32)  -- moe.py:86-90."""
    if k < 1:
        raise ValueError(f"top_k must be >= 1, got {k}")
    probs = softmax_f32(logits)
    idx = topk_order(logits, k)
    top = np.take_along_axis(probs, idx, axis=-1)
    s = np.zeros(top.shape[0], dtype=np.float32)
    for j in range(k):  # left-to-right sum of the k selected probabilities
        s = (s + top[:, j]).astype(np.float32)
    gates = (top / s[:, None]).astype(np.float32)
    return gates, idx, probs


def capacity(num_tokens: int, k: int, num_experts: int, capacity_factor: float) -> int:
    """moe.py:103-105."""
    return max(1, int(capacity_factor * num_tokens * k / num_experts))


def permutation(idx: np.ndarray, num_experts: int, cap: int):
    """Per expert (ascending) the ascending token list, truncated to `cap`.

    Returns (kept: list[np.ndarray], counts: np.ndarray[E]) where counts are
    the pre-capacity dispatch counts (moe.py:109-116, :139-142)."""
    kept, counts = [], np.zeros(num_experts, dtype=np.int64)
    for e in range(num_experts):
        toks = np.nonzero((idx == e).any(axis=-1))[0]
        counts[e] = toks.size
        kept.append(toks[:cap].astype(np.int64))
    return kept, counts


def _silu(g32: np.ndarray) -> np.ndarray:
    return (g32 / (1.0 + np.exp(-g32.astype(np.float64)))).astype(np.float32)


def _dsilu(g32: np.ndarray) -> np.ndarray:
    sg = 1.0 / (1.0 + np.exp(-g32.astype(np.float64)))
    return (sg * (1.0 + g32 * (1.0 - sg))).astype(np.float32)


def expert_fwd(xe, wgu, wd, compute: str):
    """SwiGLU expert (ffn.py:42-44).  Returns (y, g, u, s, a) with roundings."""
    F = wgu.shape[0] // 2
    h = round_to(np.asarray(xe, np.float32) @ np.asarray(wgu, np.float32).T, compute)
    g, u = h[:, :F], h[:, F:]
    s = round_to(_silu(g), compute)
    a = round_to(s * u, compute)
    y = round_to(a @ np.asarray(wd, np.float32).T, compute)
    return y, g, u, s, a


def expert_bwd(dy, xe, wgu, wd, g, u, s, a, compute: str, acc=np.float32):
    """Backward of expert_fwd for the expert-output gradient dy (ffn.py:42-44
    under autograd): (dxe, dwgu, dwd), each rounded to `compute`.  `acc` is the
    accumulation type of the two weight-gradient sums over the rows (float32 as
    torch's GEMM; float64 for a reference of a float32-accumulated kernel)."""
    da = round_to(dy @ np.asarray(wd, np.float32), compute)
    dwd = round_to((dy.T.astype(acc) @ np.asarray(a, acc)).astype(np.float32), compute)
    ds = round_to(da * u, compute)
    du = round_to(da * s, compute)
    dg = round_to(ds * _dsilu(g), compute)
    dh = np.concatenate([dg, du], axis=-1)
    dxe = round_to(dh @ np.asarray(wgu, np.float32), compute)
    dwgu = round_to((dh.T.astype(acc) @ np.asarray(xe, acc)).astype(np.float32), compute)
    return dxe, dwgu, dwd


def moe_forward(x, logits, wgu, wd, top_k: int, capacity_factor: float,
                lbw: float, compute: str = "f32"):
    """Full MoE layer forward on flattened tokens x [T,H].

    wgu [E, 2F, H], wd [E, H, F].  Returns a dict with out [T,H], aux (float),
    utilization [E], and the routing/permutation state used by moe_backward."""
    x32 = np.asarray(x, np.float32)
    T, H = x32.shape
    E = wgu.shape[0]
    gates, idx, probs = route(logits, top_k)
    cap = capacity(T, top_k, E, capacity_factor)
    kept, counts = permutation(idx, E, cap)
    out = np.zeros_like(x32)
    saved = []
    for e in range(E):
        toks = kept[e]
        if toks.size == 0:
            saved.append(None)
            continue
        y, g, u, s, a = expert_fwd(x32[toks], wgu[e], wd[e], compute)
        wgt = np.sum(gates[toks] * (idx[toks] == e), axis=-1, dtype=np.float32)
        contrib = round_to(y * wgt[:, None], compute)
        out[toks] = round_to(out[toks] + contrib, compute)
        saved.append((toks, y, g, u, s, a, wgt))
    frac = (counts.astype(np.float64) / T).astype(np.float32)
    pmean = np.mean(probs, axis=0, dtype=np.float64).astype(np.float32)
    aux = float(E * np.sum(pmean.astype(np.float64) * frac) * lbw)
    util = frac / max(float(frac.sum()), 1e-8)
    return {
        "out": out, "aux": aux, "util": util.astype(np.float32), "gates": gates,
        "idx": idx, "probs": probs, "counts": counts, "kept": kept, "cap": cap,
        "saved": saved, "frac": frac,
    }


def moe_backward(dout, fwd: dict, x, wgu, wd, lbw: float, compute: str = "f32"):
    """Gradients of moe_forward for upstream dout [T,H] and d(aux)=1.

    Returns dict: dx_experts [T,H] (float32, unrounded sum of the per-expert
    gather gradients), dlogits [T,E], dwgu [E,2F,H], dwd [E,H,F]."""
    x32 = np.asarray(x, np.float32)
    d32 = np.asarray(dout, np.float32)
    T, H = x32.shape
    E, F2, _ = wgu.shape
    F = F2 // 2
    gates, idx, probs = fwd["gates"], fwd["idx"], fwd["probs"]
    k = idx.shape[1]
    dgates = np.zeros_like(gates)
    dx = np.zeros((T, H), dtype=np.float64)
    dwgu = np.zeros(wgu.shape, dtype=np.float32)
    dwd = np.zeros(wd.shape, dtype=np.float32)
    for e in range(E):
        sv = fwd["saved"][e]
        if sv is None:
            continue
        toks, y, g, u, s, a, wgt = sv
        dcontrib = d32[toks]
        dy = round_to(dcontrib * wgt[:, None], compute)
        dw_tok = np.sum(dcontrib.astype(np.float64) * y, axis=-1).astype(np.float32)
        slot = np.argmax(idx[toks] == e, axis=-1)
        dgates[toks, slot] += dw_tok
        dxe, dwgu[e], dwd[e] = expert_bwd(dy, x32[toks], wgu[e], wd[e], g, u, s, a, compute)
        dx[toks] += dxe
    # renormalisation backward: gates_i = p_i / S over the selected slots
    top = np.take_along_axis(probs, idx, axis=-1)
    S = np.sum(top, axis=-1, keepdims=True, dtype=np.float32)
    dtop = (dgates - np.sum(dgates * gates, axis=-1, keepdims=True)) / S
    dprobs = np.zeros_like(probs)
    np.put_along_axis(dprobs, idx, dtop.astype(np.float32), axis=-1)
    # aux loss: d/dprobs[t,e] of E*lbw*sum_e mean_t(p)*frac_e
    dprobs += (np.float32(E * lbw) * fwd["frac"] / np.float32(T))[None, :]
    # softmax backward
    dl = probs * (dprobs - np.sum(probs * dprobs, axis=-1, keepdims=True))
    del k
    return {"dx_experts": dx.astype(np.float32), "dlogits": dl.astype(np.float32),
            "dwgu": dwgu, "dwd": dwd, "dgates": dgates}


def router_logits(x, wg) -> np.ndarray:
    """gate Linear in float32: x @ Wg^T (moe.py:86)."""
    return (np.asarray(x, np.float32) @ np.asarray(wg, np.float32).T).astype(np.float32)


def moe_layer_backward_full(dout, fwd, x, wg, wgu, wd, lbw, compute="f32"):
    """Adds the router Linear's gradients: dx = dx_experts + dlogits @ Wg,
    dWg = dlogits^T @ x.  dx is rounded to the token dtype."""
    b = moe_backward(dout, fwd, x, wgu, wd, lbw, compute)
    dl = b["dlogits"]
    dx = b["dx_experts"] + dl @ np.asarray(wg, np.float32)
    b["dx"] = round_to(dx, compute)
    b["dwg"] = (dl.T @ np.asarray(x, np.float32)).astype(np.float32)
    return b

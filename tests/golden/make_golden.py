"""Generate the golden vectors that pin the oracle to the reference.

Run it with an ats-v2 source tree, named by the first argument or by
ATS_REFERENCE_DIR:

    python tests/golden/make_golden.py <ats-v2 checkout>

It imports the reference's own modules (``ats.model.norm``, ``rope``,
``norm_triton``, ``rope_triton``, ``moe_triton``, ``moe``, ``ffn``,
``mla_triton``) with their
Triton paths disabled, runs them forward and backward (torch autograd) on
seeded CPU inputs, and writes ``tests/golden/*.npz``.  bfloat16 tensors are
stored as uint16 bit patterns (key suffix ``_bf16``).

The fixtures are small (a few hundred KB in total) so they can be committed;
the tests never import the reference.

One case needs a note: the north-star MoE runs a float32 router on bfloat16
tokens and experts.  The reference fallback cannot run that combination
as-is (``index_add_`` refuses a float32 source into a bfloat16 buffer,
moe.py:122), so the bf16 MoE case below drives the reference's own pieces
(compute_routing with a float32 gate, the reference SwiGLU experts, the
moe.py:109-122 loop) with the single added cast of ``expert_output * weight``
to the buffer dtype.
"""

from __future__ import annotations

import json
import os
import sys
from pathlib import Path

import numpy as np
import torch

REF = sys.argv[1] if len(sys.argv) > 1 else os.environ.get("ATS_REFERENCE_DIR", "")
OUT = Path(__file__).resolve().parent


def _import_reference():
    if not REF or not Path(REF, "ats", "model").is_dir():
        raise SystemExit("name an ats-v2 source tree: make_golden.py <checkout> (or set ATS_REFERENCE_DIR); "
                         f"got {REF!r}")
    sys.path.insert(0, REF)
    import ats.model.mla_triton as mla_triton
    import ats.model.moe as moe
    import ats.model.moe_triton as moe_triton
    import ats.model.norm as norm
    import ats.model.norm_triton as norm_triton
    import ats.model.rope as rope
    import ats.model.rope_triton as rope_triton
    # never take the unverified Triton kernels: the PyTorch path is the reference
    for m in (norm_triton, rope_triton, moe_triton, mla_triton):
        m.HAS_TRITON = False
    return norm, norm_triton, rope, rope_triton, moe, moe_triton, mla_triton


def _np(t: torch.Tensor, key: str, store: dict) -> None:
    t = t.detach().cpu()
    if t.dtype == torch.bfloat16:
        store[key + "_bf16"] = t.contiguous().view(torch.int16).numpy().view(np.uint16)
    elif t.dtype in (torch.int64, torch.int32):
        store[key] = t.numpy().astype(np.int64)
    else:
        store[key] = t.float().numpy()


def gen_rmsnorm(norm, norm_triton) -> dict:
    s: dict = {}
    torch.manual_seed(0)
    # fp32, the CPU parity workload's shape family (hidden 512, eps 1e-6)
    x = torch.randn(1, 40, 512)
    w = 1.0 + 0.02 * torch.randn(512)
    dy = torch.randn(1, 40, 512)
    m = norm.RMSNorm(512, eps=1e-6)
    with torch.no_grad():
        m.weight.copy_(w)
    xr = x.clone().requires_grad_(True)
    y = m(xr)
    y.backward(dy)
    for k, v in dict(f32_x=x, f32_w=w, f32_dy=dy, f32_y=y, f32_dx=xr.grad, f32_dw=m.weight.grad).items():
        _np(v, k, s)
    # bf16 activations, fp32 weight, eps 1e-5 (the 7B RMSNorm config's dtypes)
    x = torch.randn(24, 1024).bfloat16()
    w = 1.0 + 0.02 * torch.randn(1024)
    dy = torch.randn(24, 1024).bfloat16()
    m = norm.RMSNorm(1024, eps=1e-5)
    with torch.no_grad():
        m.weight.copy_(w)
    xr = x.clone().requires_grad_(True)
    import warnings
    with warnings.catch_warnings():
        warnings.simplefilter("ignore")
        y = m(xr)
        y.backward(dy)
    for k, v in dict(b_x=x, b_w=w, b_dy=dy, b_y=y, b_dx=xr.grad, b_dw=m.weight.grad).items():
        _np(v, k, s)
    # fused residual: the reference test's shapes, then a bf16 case
    torch.manual_seed(0)
    x = torch.randn(2, 5, 16)
    res = torch.randn(2, 5, 16)
    w = torch.randn(16)
    xr, rr, wr = (t.clone().requires_grad_(True) for t in (x, res, w))
    out = norm_triton._pytorch_rmsnorm_residual(xr, rr, wr, 1e-6)
    g = torch.randn_like(out)
    out.backward(g)
    for k, v in dict(r32_x=x, r32_res=res, r32_w=w, r32_out=out, r32_g=g, r32_dx=xr.grad,
                     r32_dres=rr.grad, r32_dw=wr.grad).items():
        _np(v, k, s)
    x = torch.randn(8, 256).bfloat16()
    res = torch.randn(8, 256).bfloat16()
    w = (1.0 + 0.1 * torch.randn(256)).bfloat16()
    xr, rr, wr = (t.clone().requires_grad_(True) for t in (x, res, w))
    out = norm_triton._pytorch_rmsnorm_residual(xr, rr, wr, 1e-6)
    g = torch.randn_like(out)
    out.backward(g)
    for k, v in dict(rb_x=x, rb_res=res, rb_w=w, rb_out=out, rb_g=g, rb_dx=xr.grad,
                     rb_dres=rr.grad, rb_dw=wr.grad).items():
        _np(v, k, s)
    return s


def gen_rope(rope, rope_triton) -> dict:
    s: dict = {}
    # cache of the 7B config: D=128, theta=5e5, up to 4096 positions
    r = rope.RotaryEmbedding(128, max_seq_len=4096, theta=500000.0)
    cos, sin = r(4096, torch.device("cpu"), torch.float32)
    sel = torch.cat([torch.arange(0, 32), torch.arange(4064, 4096)])
    _np(r.inv_freq, "inv_freq_128_5e5", s)
    _np(cos[sel], "cos_128_5e5_rows", s)
    _np(sin[sel], "sin_128_5e5_rows", s)
    s["rows_128_5e5"] = sel.numpy()
    cb, sb = r(4096, torch.device("cpu"), torch.bfloat16)
    _np(cb[sel], "cosb_128_5e5_rows", s)
    _np(sb[sel], "sinb_128_5e5_rows", s)
    # cache doubling (rope.py:50-59): a 16-entry cache asked for 20 rows grows to 32
    r2 = rope.RotaryEmbedding(8, max_seq_len=16, theta=10000.0)
    r2(20, torch.device("cpu"), torch.float32)
    s["grow_16_to_20"] = np.array([r2._cached_seq_len], dtype=np.int64)
    # fp32 q/k, the CPU parity workload's RoPE family: BSHD memory viewed as BHSD
    torch.manual_seed(0)
    q = torch.randn(1, 32, 8, 64)
    k = torch.randn(1, 32, 4, 64)
    r1 = rope.RotaryEmbedding(64, max_seq_len=256, theta=10000.0)
    c, sn = r1(32, torch.device("cpu"), torch.float32)
    qv = q.clone().transpose(1, 2).requires_grad_(True)
    kv = k.clone().transpose(1, 2).requires_grad_(True)
    qo, ko = rope.apply_rotary_pos_emb(qv, kv, c, sn)
    gq, gk = torch.randn_like(qo), torch.randn_like(ko)
    torch.autograd.backward([qo, ko], [gq, gk])
    for kk, v in dict(f_q=q, f_k=k, f_cos=c, f_sin=sn, f_qo=qo, f_ko=ko, f_gq=gq, f_gk=gk,
                      f_dq=qv.grad, f_dk=kv.grad).items():
        _np(v.contiguous(), kk, s)
    # bf16 q/k with theta 5e5, D=128 (the 7B RoPE config's dtypes)
    q = torch.randn(1, 32, 8, 128).bfloat16()
    k = torch.randn(1, 32, 2, 128).bfloat16()
    c, sn = r(32, torch.device("cpu"), torch.bfloat16)
    qv = q.clone().transpose(1, 2).requires_grad_(True)
    kv = k.clone().transpose(1, 2).requires_grad_(True)
    qo, ko = rope.apply_rotary_pos_emb(qv, kv, c, sn)
    gq, gk = torch.randn_like(qo), torch.randn_like(ko)
    torch.autograd.backward([qo, ko], [gq, gk])
    for kk, v in dict(b_q=q, b_k=k, b_cos=c, b_sin=sn, b_qo=qo, b_ko=ko, b_gq=gq, b_gk=gk,
                      b_dq=qv.grad, b_dk=kv.grad).items():
        _np(v.contiguous(), kk, s)
    # the single-tensor entry point on the reference test's shape
    torch.manual_seed(0)
    x = torch.randn(1, 2, 6, 8)
    r3 = rope.RotaryEmbedding(8, max_seq_len=16, theta=10000.0)
    c, sn = r3(6, torch.device("cpu"), torch.float32)
    y = rope_triton._pytorch_apply_rope(x, c, sn)
    for kk, v in dict(t_x=x, t_cos=c, t_sin=sn, t_y=y).items():
        _np(v, kk, s)
    return s


def _zipf_bias(E: int, s_exp: float = 1.1, seed: int = 1) -> torch.Tensor:
    p = torch.arange(1, E + 1, dtype=torch.float64) ** (-s_exp)
    p = p / p.sum()
    perm = torch.randperm(E, generator=torch.Generator().manual_seed(seed))
    b = torch.log(p[perm])
    return (b - b.mean()).float()


def gen_routing(moe_triton) -> dict:
    s: dict = {}
    cases = []
    torch.manual_seed(0)
    cases.append(("r5x4", torch.randn(5, 4), 2))
    torch.manual_seed(0)
    cases.append(("r32x8", torch.randn(32, 8), 2))
    torch.manual_seed(3)
    cases.append(("r64x8k1", torch.randn(64, 8), 1))
    cases.append(("r64x16k4", torch.randn(64, 16), 4))
    cases.append(("r512x64z", torch.randn(512, 64) + _zipf_bias(64)[None, :], 2))
    cases.append(("r200x256k8", torch.randn(200, 256), 8))
    for name, logits, k in cases:
        p, i = moe_triton._pytorch_moe_routing(logits, k)
        _np(logits, name + "_logits", s)
        _np(p, name + "_probs", s)
        _np(i, name + "_idx", s)
        s[name + "_k"] = np.array([k], dtype=np.int64)
    s["zipf64"] = _zipf_bias(64).numpy()
    return s


def _moe_case_fp32(moe, T_b, T_s, H, F, E, k, cf, lbw, seed) -> dict:
    s: dict = {}
    torch.manual_seed(seed)
    layer = moe.MoELayer(hidden_size=H, intermediate_size=F, num_experts=E, num_layers=2,
                         top_k=k, capacity_factor=cf, load_balancing_weight=lbw)
    assert not layer.uses_deepspeed
    fb = layer.moe
    with torch.no_grad():
        fb.gate.weight.normal_(0.0, 0.02)
        for ex in fb.experts:
            ex.gate_up_proj.weight.normal_(0.0, 0.02)
            ex.down_proj.weight.normal_(0.0, 0.02)
    x = torch.randn(T_b, T_s, H)
    xr = x.clone().requires_grad_(True)
    out, aux = layer(xr)
    g = torch.randn_like(out)
    (out * g).sum().add(aux).backward()
    flat = x.reshape(-1, H)
    with torch.no_grad():
        logits = fb.gate(flat)
    _np(x.reshape(-1, H), "x", s)
    _np(fb.gate.weight, "wg", s)
    _np(torch.stack([e.gate_up_proj.weight for e in fb.experts]), "wgu", s)
    _np(torch.stack([e.down_proj.weight for e in fb.experts]), "wd", s)
    _np(logits, "logits", s)
    _np(out.reshape(-1, H), "out", s)
    s["aux"] = np.array([aux.item()], dtype=np.float64)
    s["util"] = np.array([layer.last_expert_utilization[i] for i in range(E)], dtype=np.float64)
    _np(g.reshape(-1, H), "g", s)
    _np(xr.grad.reshape(-1, H), "dx", s)
    _np(fb.gate.weight.grad, "dwg", s)
    _np(torch.stack([e.gate_up_proj.weight.grad for e in fb.experts]), "dwgu", s)
    _np(torch.stack([e.down_proj.weight.grad for e in fb.experts]), "dwd", s)
    s["cfg"] = np.array([H, F, E, k], dtype=np.int64)
    s["cf_lbw"] = np.array([cf, lbw], dtype=np.float64)
    return s


def _moe_case_bf16(moe, T, H, F, E, k, cf, lbw, seed) -> dict:
    """bf16 tokens/experts with a float32 router, driven through the
    reference's own modules (see the module docstring)."""
    import torch.nn.functional as Fn
    s: dict = {}
    torch.manual_seed(seed)
    fb = moe._PyTorchMoEFallback(H, F, E, k, cf, lbw, num_layers=2)
    with torch.no_grad():
        fb.gate.weight.normal_(0.0, 0.02)
        for ex in fb.experts:
            ex.gate_up_proj.weight.normal_(0.0, 0.02)
            ex.down_proj.weight.normal_(0.0, 0.02)
    for ex in fb.experts:
        ex.to(torch.bfloat16)
    x = torch.randn(T, H).bfloat16()
    xr = x.clone().requires_grad_(True)
    wg = fb.gate.weight  # float32 router weight

    class _F32Gate(torch.nn.Module):
        def forward(self, inp):
            return Fn.linear(inp.float(), wg)

    gate_mod = fb.gate
    fb.gate = _F32Gate()
    top_p, top_i, router_probs = fb.compute_routing(xr)
    fb.gate = gate_mod
    cap = max(1, int(cf * T * k / E))
    output = torch.zeros_like(xr)
    for e in range(E):  # moe.py:109-122 with the dtype cast added before index_add_
        tok = (top_i == e).any(dim=-1).nonzero(as_tuple=True)[0]
        if tok.numel() == 0:
            continue
        tok = tok[:cap]
        y = fb.experts[e](xr[tok])
        wgt = (top_p[tok] * (top_i[tok] == e)).sum(dim=-1, keepdim=True)
        output = output.index_add(0, tok, (y * wgt).to(output.dtype))
    pm = router_probs.mean(dim=0)
    frac = Fn.one_hot(top_i, E).float().sum(dim=1).mean(dim=0)
    aux = E * torch.sum(pm * frac) * lbw
    g = torch.randn_like(output)
    (output.float() * g.float()).sum().add(aux).backward()
    with torch.no_grad():
        logits = Fn.linear(x.float(), wg)
    _np(x, "x", s)
    _np(wg, "wg", s)
    _np(torch.stack([e.gate_up_proj.weight for e in fb.experts]), "wgu", s)
    _np(torch.stack([e.down_proj.weight for e in fb.experts]), "wd", s)
    _np(logits, "logits", s)
    _np(output, "out", s)
    s["aux"] = np.array([aux.item()], dtype=np.float64)
    util = frac / frac.sum().clamp(min=1e-8)
    s["util"] = util.double().numpy()
    _np(g, "g", s)
    _np(xr.grad, "dx", s)
    _np(wg.grad, "dwg", s)
    _np(torch.stack([e.gate_up_proj.weight.grad for e in fb.experts]), "dwgu", s)
    _np(torch.stack([e.down_proj.weight.grad for e in fb.experts]), "dwd", s)
    s["cfg"] = np.array([H, F, E, k], dtype=np.int64)
    s["cf_lbw"] = np.array([cf, lbw], dtype=np.float64)
    return s


def gen_mla(mla_triton) -> dict:
    """fused_mla_kv_decompress (mla_triton.py:122-151) forward and autograd
    backward, float32 and bfloat16, on seeded [2, 24, latent] latents."""
    s = {}
    for tag, dt, (B, S, L, O), seed in (("f32", torch.float32, (2, 24, 64, 96), 21),
                                          ("bf16", torch.bfloat16, (2, 24, 128, 64), 22)):
        g = torch.Generator().manual_seed(seed)
        c = torch.randn(B, S, L, generator=g).to(dt).requires_grad_()
        w_uk = (0.1 * torch.randn(O, L, generator=g)).to(dt).requires_grad_()
        w_uv = (0.1 * torch.randn(O, L, generator=g)).to(dt).requires_grad_()
        dk = torch.randn(B, S, O, generator=g).to(dt)
        dv = torch.randn(B, S, O, generator=g).to(dt)
        k, v = mla_triton.fused_mla_kv_decompress(c, w_uk, w_uv)
        torch.autograd.backward([k, v], [dk, dv])
        for name, t in (("c", c), ("w_uk", w_uk), ("w_uv", w_uv), ("dk", dk), ("dv", dv), ("k", k), ("v", v),
                        ("dc", c.grad), ("dw_uk", w_uk.grad), ("dw_uv", w_uv.grad)):
            _np(t, f"{tag}_{name}", s)
    return s


def main() -> None:
    torch.set_num_threads(min(8, os.cpu_count() or 1))
    torch.backends.cuda.matmul.allow_tf32 = False
    norm, norm_triton, rope, rope_triton, moe, moe_triton, mla_triton = _import_reference()
    files = {
        "rmsnorm.npz": gen_rmsnorm(norm, norm_triton),
        "rope.npz": gen_rope(rope, rope_triton),
        "routing.npz": gen_routing(moe_triton),
        # cf 1.25 with 64 tokens: capacity 40 < demand for popular experts -> drops
        "moe_f32_drop.npz": _moe_case_fp32(moe, 2, 32, 64, 128, 4, 2, 1.25, 0.01, 11),
        # cf = E/k: no capacity drop (the single-GPU MoE config's setting)
        "moe_f32_nodrop.npz": _moe_case_fp32(moe, 1, 48, 32, 96, 8, 2, 4.0, 0.01, 12),
        "moe_bf16.npz": _moe_case_bf16(moe, 96, 64, 128, 8, 2, 4.0, 0.01, 13),
        "moe_bf16_drop.npz": _moe_case_bf16(moe, 80, 64, 64, 4, 2, 1.0, 0.01, 14),
        "mla.npz": gen_mla(mla_triton),
    }
    manifest = {}
    for name, d in files.items():
        np.savez_compressed(OUT / name, **d)
        manifest[name] = sorted(d.keys())
    (OUT / "MANIFEST.json").write_text(json.dumps(
        {"torch": torch.__version__, "files": manifest}, indent=1, sort_keys=True) + "\n")
    print("wrote", ", ".join(files))


if __name__ == "__main__":
    main()

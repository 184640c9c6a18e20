"""Pin the numpy oracle against golden vectors produced by the reference's
own PyTorch modules (tests/golden/make_golden.py).  CPU only.

Tolerances: float32 results within 1e-5 relative (with a small absolute
floor for values near zero); bfloat16 results within 2e-2 relative /
1e-2 absolute, and additionally at least 99% bit-identical; router indices
and permutations exactly equal.
"""

from __future__ import annotations

import numpy as np
import pytest

from oracle import mla as omla
from oracle import moe as omoe
from oracle import norm as onorm
from oracle import rope as orope
from tests.conftest import load_golden

F32 = dict(rtol=1e-5, atol=1e-6)
BF16 = dict(rtol=2e-2, atol=1e-2)


def _bf16_close(a, b, min_exact=0.99):
    np.testing.assert_allclose(a, b, **BF16)
    exact = float(np.mean(a.view(np.uint32) == b.view(np.uint32)))
    assert exact >= min_exact, f"only {exact:.4f} of bf16 values bit-identical"


def test_rmsnorm_f32_matches_reference():
    g = load_golden("rmsnorm")
    y, _ = onorm.rmsnorm_fwd(g["f32_x"], g["f32_w"], 1e-6, "f32")
    np.testing.assert_allclose(y, g["f32_y"], **F32)
    dx, dw = onorm.rmsnorm_bwd(g["f32_dy"], g["f32_x"], g["f32_w"], 1e-6, "f32", "f32")
    np.testing.assert_allclose(dx, g["f32_dx"], rtol=1e-5, atol=1e-5)
    np.testing.assert_allclose(dw, g["f32_dw"], rtol=1e-5, atol=1e-5)


def test_rmsnorm_bf16_fp32_weight_matches_reference():
    g = load_golden("rmsnorm")
    y, _ = onorm.rmsnorm_fwd(g["b_x"], g["b_w"], 1e-5, "bf16")
    _bf16_close(y, g["b_y"])
    dx, dw = onorm.rmsnorm_bwd(g["b_dy"], g["b_x"], g["b_w"], 1e-5, "bf16", "f32")
    _bf16_close(dx, g["b_dx"], min_exact=0.97)
    np.testing.assert_allclose(dw, g["b_dw"], rtol=1e-4, atol=1e-4)


def test_rmsnorm_residual_matches_reference():
    g = load_golden("rmsnorm")
    out, _ = onorm.rmsnorm_residual_fwd(g["r32_x"], g["r32_res"], g["r32_w"], 1e-6)
    np.testing.assert_allclose(out, g["r32_out"], **F32)
    dx, dres, dw = onorm.rmsnorm_residual_bwd(g["r32_g"], g["r32_x"], g["r32_w"], 1e-6)
    np.testing.assert_allclose(dx, g["r32_dx"], rtol=1e-5, atol=1e-5)
    np.testing.assert_allclose(dres, g["r32_dres"], **F32)
    np.testing.assert_allclose(dw, g["r32_dw"], rtol=1e-5, atol=1e-5)
    out, _ = onorm.rmsnorm_residual_fwd(g["rb_x"], g["rb_res"], g["rb_w"], 1e-6,
                                        "bf16", "bf16", "bf16")
    _bf16_close(out, g["rb_out"])
    dx, dres, dw = onorm.rmsnorm_residual_bwd(g["rb_g"], g["rb_x"], g["rb_w"], 1e-6,
                                              "bf16", "bf16", "bf16")
    _bf16_close(dx, g["rb_dx"], min_exact=0.97)
    _bf16_close(dres, g["rb_dres"], min_exact=1.0)
    np.testing.assert_allclose(dw, g["rb_dw"], **BF16)


def test_rope_cache_matches_reference():
    g = load_golden("rope")
    assert np.array_equal(orope.inv_freq(128, 500000.0), g["inv_freq_128_5e5"])
    cos, sin = orope.cos_sin_cache(4096, 128, 500000.0, "f32")
    rows = g["rows_128_5e5"]
    np.testing.assert_allclose(cos[rows], g["cos_128_5e5_rows"], rtol=0, atol=1e-6)
    np.testing.assert_allclose(sin[rows], g["sin_128_5e5_rows"], rtol=0, atol=1e-6)
    cb, sb = orope.cos_sin_cache(4096, 128, 500000.0, "bf16")
    _bf16_close(cb[rows], g["cosb_128_5e5_rows"])
    _bf16_close(sb[rows], g["sinb_128_5e5_rows"])


def test_rope_apply_f32_matches_reference():
    g = load_golden("rope")
    q = g["f_q"].transpose(0, 2, 1, 3)
    k = g["f_k"].transpose(0, 2, 1, 3)
    np.testing.assert_allclose(orope.rope_fwd(q, g["f_cos"], g["f_sin"]), g["f_qo"], **F32)
    np.testing.assert_allclose(orope.rope_fwd(k, g["f_cos"], g["f_sin"]), g["f_ko"], **F32)
    np.testing.assert_allclose(orope.rope_bwd(g["f_gq"], g["f_cos"], g["f_sin"]), g["f_dq"], **F32)
    np.testing.assert_allclose(orope.rope_bwd(g["f_gk"], g["f_cos"], g["f_sin"]), g["f_dk"], **F32)


def test_rope_apply_bf16_matches_reference():
    g = load_golden("rope")
    q = g["b_q"].transpose(0, 2, 1, 3)
    k = g["b_k"].transpose(0, 2, 1, 3)
    _bf16_close(orope.rope_fwd(q, g["b_cos"], g["b_sin"], "bf16"), g["b_qo"], min_exact=1.0)
    _bf16_close(orope.rope_fwd(k, g["b_cos"], g["b_sin"], "bf16"), g["b_ko"], min_exact=1.0)
    _bf16_close(orope.rope_bwd(g["b_gq"], g["b_cos"], g["b_sin"], "bf16"), g["b_dq"], min_exact=1.0)
    _bf16_close(orope.rope_bwd(g["b_gk"], g["b_cos"], g["b_sin"], "bf16"), g["b_dk"], min_exact=1.0)


def test_rope_single_tensor_entry_matches_reference():
    g = load_golden("rope")
    np.testing.assert_allclose(orope.rope_fwd(g["t_x"], g["t_cos"], g["t_sin"]), g["t_y"], **F32)


@pytest.mark.parametrize("case", ["r5x4", "r32x8", "r64x8k1", "r64x16k4", "r512x64z", "r200x256k8"])
def test_routing_matches_reference(case):
    g = load_golden("routing")
    k = int(g[case + "_k"][0])
    gates, idx, _ = omoe.route(g[case + "_logits"], k)
    assert np.array_equal(idx, g[case + "_idx"]), "router indices must be bit-exact"
    np.testing.assert_allclose(gates, g[case + "_probs"], rtol=1e-6, atol=1e-7)


@pytest.mark.parametrize("case", ["moe_f32_drop", "moe_f32_nodrop"])
def test_moe_f32_layer_matches_reference(case):
    g = load_golden(case)
    H, F, E, k = (int(v) for v in g["cfg"])
    cf, lbw = (float(v) for v in g["cf_lbw"])
    logits = omoe.router_logits(g["x"], g["wg"])
    np.testing.assert_allclose(logits, g["logits"], rtol=1e-5, atol=1e-6)
    # route on the reference's own logits (the bit-exactness contract)
    fwd = omoe.moe_forward(g["x"], g["logits"], g["wgu"], g["wd"], k, cf, lbw, "f32")
    np.testing.assert_allclose(fwd["out"], g["out"], rtol=1e-5, atol=1e-6)
    assert fwd["aux"] == pytest.approx(float(g["aux"][0]), rel=1e-5)
    np.testing.assert_allclose(fwd["util"], g["util"], rtol=1e-6, atol=1e-7)
    b = omoe.moe_layer_backward_full(g["g"], fwd, g["x"], g["wg"], g["wgu"], g["wd"], lbw, "f32")
    np.testing.assert_allclose(b["dx"], g["dx"], rtol=1e-4, atol=1e-6)
    np.testing.assert_allclose(b["dwg"], g["dwg"], rtol=1e-4, atol=1e-6)
    np.testing.assert_allclose(b["dwgu"], g["dwgu"], rtol=1e-4, atol=1e-6)
    np.testing.assert_allclose(b["dwd"], g["dwd"], rtol=1e-4, atol=1e-6)


def test_moe_f32_drop_case_really_drops():
    g = load_golden("moe_f32_drop")
    H, F, E, k = (int(v) for v in g["cfg"])
    cf, _ = (float(v) for v in g["cf_lbw"])
    T = g["x"].shape[0]
    _, idx, _ = omoe.route(g["logits"], k)
    cap = omoe.capacity(T, k, E, cf)
    _, counts = omoe.permutation(idx, E, cap)
    assert counts.max() > cap


@pytest.mark.parametrize("case", ["moe_bf16", "moe_bf16_drop"])
def test_moe_bf16_layer_matches_reference(case):
    g = load_golden(case)
    H, F, E, k = (int(v) for v in g["cfg"])
    cf, lbw = (float(v) for v in g["cf_lbw"])
    fwd = omoe.moe_forward(g["x"], g["logits"], g["wgu"], g["wd"], k, cf, lbw, "bf16")
    _bf16_close(fwd["out"], g["out"], min_exact=0.95)
    assert fwd["aux"] == pytest.approx(float(g["aux"][0]), rel=1e-5)
    np.testing.assert_allclose(fwd["util"], g["util"], rtol=1e-6, atol=1e-7)
    b = omoe.moe_layer_backward_full(g["g"], fwd, g["x"], g["wg"], g["wgu"], g["wd"], lbw, "bf16")
    np.testing.assert_allclose(b["dx"], g["dx"], **BF16)
    np.testing.assert_allclose(b["dwg"], g["dwg"], rtol=1e-3, atol=1e-5)
    np.testing.assert_allclose(b["dwgu"], g["dwgu"], **BF16)
    np.testing.assert_allclose(b["dwd"], g["dwd"], **BF16)


def test_capacity_formula():
    assert omoe.capacity(32768, 2, 64, 1.25) == 1280
    assert omoe.capacity(8192, 2, 8, 4.0) == 8192
    assert omoe.capacity(1, 1, 64, 0.01) == 1


@pytest.mark.parametrize("tag", ["f32", "bf16"])
def test_mla_kv_decompress_matches_reference(tag):
    g = load_golden("mla")
    c, w_uk, w_uv = g[f"{tag}_c"], g[f"{tag}_w_uk"], g[f"{tag}_w_uv"]
    k, v = omla.kv_decompress(c, w_uk, w_uv, tag)
    dc, dwk, dwv = omla.kv_decompress_bwd(g[f"{tag}_dk"], g[f"{tag}_dv"], c, w_uk, w_uv, tag)
    pairs = ((k, "k"), (v, "v"), (dc, "dc"), (dwk, "dw_uk"), (dwv, "dw_uv"))
    for got, name in pairs:
        if tag == "f32":
            np.testing.assert_allclose(got, g[f"f32_{name}"], rtol=1e-5, atol=1e-5, err_msg=name)
        else:
            _bf16_close(got, g[f"bf16_{name}"], min_exact=0.97)


"""The CPU oracle against the reference's golden vectors (tests/golden/*.npz).

Bit-exact where the reference's arithmetic is integer or a chain of single
bf16 roundings (MXFP8 codes/scales, the gated residual); within one bf16 ulp
where the golden came from an eager CPU op whose reduction order or
transcendental implementation differs from the CUDA order the oracle follows.
"""
from pathlib import Path

import numpy as np
import pytest
import torch

import oracle

GOLD = Path(__file__).resolve().parent / "golden"


def load(name):
    return np.load(GOLD / name)


def close_bf16(a_bits, b_bits, atol=1e-6):
    """Within one bf16 ulp, or within atol absolutely (transcendental tails
    such as GELU at x < -5, where tanh implementations round 1 + tanh(x)
    to 0 or to one fp32 ulp)."""
    fa, fb = oracle.bf16_bits_to_f32(a_bits), oracle.bf16_bits_to_f32(b_bits)
    return (ulp_diff(a_bits, b_bits) <= 1) | (np.abs(fa - fb) <= atol)


def ulp_diff(a_bits, b_bits):
    """Distance in bf16 ulps between two bf16 bit arrays of the same sign."""
    a = a_bits.astype(np.int32)
    b = b_bits.astype(np.int32)
    a = np.where(a & 0x8000, -(a & 0x7FFF), a)
    b = np.where(b & 0x8000, -(b & 0x7FFF), b)
    return np.abs(a - b)


@pytest.mark.parametrize("shape", [(1, 128), (77, 256), (130, 256), (200, 384)])
def test_mxfp8_oracles_match_reference(shape):
    g = load("mxfp8_quantize.npz")
    m, k = shape
    x = g[f"x_{m}_{k}"]
    codes, scales = g[f"codes_{m}_{k}"], g[f"scales_{m}_{k}"]
    cq, cs = oracle.mx_quantize(x)
    nq, ns = oracle.mx_quantize_numpy(x)
    assert np.array_equal(cq, codes) and np.array_equal(cs, scales)
    assert np.array_equal(nq, codes) and np.array_equal(ns, scales)


def test_e4m3_encoder_matches_torch_cast():
    rng = np.random.default_rng(0)
    v = np.concatenate([rng.standard_normal(20000).astype(np.float32) * s for s in (1e-3, 0.05, 1.0, 30.0, 150.0)])
    v = np.concatenate([v, np.float32([0.0, -0.0, 448.0, -448.0, 2.0 ** -10, 3 * 2.0 ** -10, -(2.0 ** -10)])])
    v = v[np.abs(v) <= 448]
    ref = torch.from_numpy(v).to(torch.float8_e4m3fn).view(torch.uint8).numpy()
    assert np.array_equal(oracle._encode_e4m3(v), ref)
    assert all(oracle.e4m3(float(x)) == int(r) for x, r in zip(v[::50], ref[::50]))


@pytest.mark.parametrize("key", ["1_49_256", "2_9_512"])
def test_gated_residual_oracle_bit_exact(key):
    g = load("residual.npz")
    h, x, gate, out = g[f"h_{key}"], g[f"x_{key}"], g[f"g_{key}"], g[f"out_{key}"]
    b, s, d = h.shape
    got = oracle.gated_residual(h.reshape(b * s, d), x.reshape(b * s, d), gate.reshape(b, d), s)
    assert np.array_equal(got, out.reshape(b * s, d))


@pytest.mark.parametrize("key", ["1_7_512", "2_3_1536", "1_2_3072"])
def test_ln_mod_oracle_within_one_ulp(key):
    g = load("ln_mod.npz")
    x, sc, sh = g[f"x_{key}"], g[f"scale_{key}"], g[f"shift_{key}"]
    b, s, d = x.shape
    got = oracle.ln_mod(x.reshape(b * s, d), sc.reshape(b, d), sh.reshape(b, d), s)
    assert ulp_diff(got, g[f"out_{key}"].reshape(b * s, d)).max() <= 1
    got = oracle.ln_mod(x.reshape(b * s, d), sc.reshape(b, d), None, s)
    d1 = ulp_diff(got, g[f"noshift_{key}"].reshape(b * s, d))
    assert d1.max() <= 1 and (d1 == 0).mean() > 0.98


def test_ln_stats_close_to_float64():
    rng = np.random.default_rng(1)
    for d in (512, 3072, 4096):
        x = oracle.f32_to_bf16_bits(rng.standard_normal(d).astype(np.float32) * 3 + 0.5)
        m, v = oracle.ln_stats(x)
        xf = oracle.bf16_bits_to_f32(x).astype(np.float64)
        assert abs(m - xf.mean()) < 1e-5 and abs(v - xf.var()) / xf.var() < 1e-5


def test_rms_norm_and_rope_oracle_vs_diffusers():
    g = load("rope_rms.npz")
    q, w = g["q"], g["w"]
    b, s, h, d = q.shape
    normed = oracle.rms_norm(q.reshape(-1, 128), w).reshape(q.shape)
    dn = ulp_diff(normed, g["normed"])
    assert dn.max() <= 1 and (dn == 0).mean() > 0.99
    rq, _ = oracle.rope_qk(g["normed"], g["normed"], g["img_freqs"])
    dr = ulp_diff(rq, g["rotated"])
    assert dr.max() <= 1 and (dr == 0).mean() > 0.99


def test_activation_oracles_vs_eager():
    g = load("activations.npz")
    ds = ulp_diff(oracle.swiglu(g["g"], g["v"]), g["swiglu"])
    assert ds.max() <= 1 and (ds == 0).mean() > 0.99
    got = oracle.gelu_tanh(g["x"])
    assert close_bf16(got, g["gelu"]).all() and (got == g["gelu"]).mean() > 0.99


def test_qknorm_rope_pack_oracle_is_composition():
    g = load("rope_rms.npz")
    q = g["q"]
    b, s, h, d = q.shape
    k = q[:, ::-1].copy()
    v = (q ^ np.uint16(0x8000)).copy()
    ck = q[:, :3].copy()
    cv = k[:, :3].copy()
    oq, ok, ov = oracle.qknorm_rope_pack(q, k, v, ck, cv, g["w"], g["w"], g["img_freqs"])
    nq = oracle.rms_norm(q.reshape(-1, 128), g["w"]).reshape(q.shape)
    nk = oracle.rms_norm(k.reshape(-1, 128), g["w"]).reshape(q.shape)
    rq, rk = oracle.rope_qk(nq, nk, g["img_freqs"])
    assert np.array_equal(oq, rq)
    assert np.array_equal(ok, np.concatenate([ck, rk], 1)) and np.array_equal(ov, np.concatenate([cv, v], 1))


def test_mxfp8_gemm_oracle_close_to_bf16():
    rng = np.random.default_rng(2)
    a = oracle.f32_to_bf16_bits(rng.standard_normal((64, 256)).astype(np.float32))
    w = oracle.f32_to_bf16_bits((0.02 * rng.standard_normal((128, 256))).astype(np.float32))
    aq, asc = oracle.mx_quantize(a)
    wq, wsc = oracle.mx_quantize(w)
    y = oracle.mxfp8_gemm(aq, asc, wq, wsc, 64, 128)
    ref = oracle.bf16_bits_to_f32(a).astype(np.float64) @ oracle.bf16_bits_to_f32(w).astype(np.float64).T
    rel = np.linalg.norm(y - ref) / np.linalg.norm(ref)
    assert rel < 0.06  # E4M3 (3 mantissa bits) per operand


def test_sage_oracle_close_to_exact_attention():
    rng = np.random.default_rng(3)
    q, k, v = (rng.standard_normal((1, 96, 2, 128)).astype(np.float32) for _ in range(3))
    o = oracle.sage_attention(q, k, v)
    ref = oracle.attention_fp32(q, k, v)
    cos = (o * ref).sum() / np.sqrt((o * o).sum() * (ref * ref).sum())
    assert cos > 0.999

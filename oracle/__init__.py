"""CPU oracle for the qia_* kernels -- TEST INFRASTRUCTURE, never the product.

Only tests/, __graft_entry__.smoke() and bench.py's cpu_baseline leg import
this package, and only as the checker. It restates the reference's arithmetic
on the CPU:

* qia_oracle.c (ctypes): LayerNorm in PyTorch's CUDA Welford order + AdaLN
  modulation, gated residual, RMSNorm/RoPE/K-V pack, SwiGLU, GELU-tanh, and the
  MXFP8 quantizer (reference src/qwen_image_accel/kernels/*.py, cited per
  function in the C file).
* numpy (this file): an independent MXFP8 restatement that follows the
  reference's own known-answer test (tests/gpu/check_mxfp8.py:41-55), the
  block-scaled GEMM as dequantize -> fp32 matmul, and the Sage-style
  quantized attention (SAGE:sageattention/core.py:725-828 with the kernels it
  calls).

Pins: the MXFP8 quantizer and gated residual are checked against golden
vectors produced by the reference's own Triton kernels (tests/golden/); the
LayerNorm order is pinned on the GPU against torch's CUDA LayerNorm, which is
the reference's own check (tests/gpu/check_layernorm_ops.py:23).
"""
from __future__ import annotations

import ctypes
import os
import subprocess
from pathlib import Path

import numpy as np

HERE = Path(__file__).resolve().parent
SRC = HERE / "qia_oracle.c"
BUILD = HERE / "_build"
LIB = BUILD / "libqia_oracle.so"

_lib = None


def build(force: bool = False) -> Path:
    """Compile the C oracle with gcc (no FMA contraction)."""
    BUILD.mkdir(parents=True, exist_ok=True)
    if force or not LIB.exists() or LIB.stat().st_mtime < SRC.stat().st_mtime:
        tmp = LIB.with_suffix(f".{os.getpid()}.tmp")
        cmd = ["gcc", "-O2", "-std=c11", "-fPIC", "-shared", "-ffp-contract=off", "-fno-fast-math",
               "-D_GNU_SOURCE", str(SRC), "-o", str(tmp), "-lm"]
        subprocess.run(cmd, check=True, capture_output=True, text=True)
        os.replace(tmp, LIB)
    return LIB


def lib() -> ctypes.CDLL:
    global _lib
    if _lib is None:
        _lib = ctypes.CDLL(str(build()))
        P, I, F = ctypes.c_void_p, ctypes.c_int64, ctypes.c_float
        sig = {
            "oracle_mx_quantize": [P, I, P, P, I, I],
            "oracle_ln_mod": [P, P, P, P, I, ctypes.c_int, I, F],
            "oracle_ln_mod_quant": [P, P, P, P, P, I, ctypes.c_int, I, F],
            "oracle_adaln_residual": [P, P, P, P, P, P, I, ctypes.c_int, I, F],
            "oracle_gated_residual": [P, P, P, P, I, I, I],
            "oracle_rms_norm": [P, P, P, I, F],
            "oracle_rope_qk": [P, P, P, P, P, I, I, I],
            "oracle_qknorm_rope_pack": [P, P, P, P, P, P, P, P, P, P, P, I, I, I, I, F, F],
            "oracle_qknorm_rope_segment": [P, I, P, P, P, P, P, P, I, I, I, I, I, F, F],
            "oracle_swiglu": [P, P, P, I],
            "oracle_swiglu_quant": [P, P, P, P, I, I],
            "oracle_gelu_tanh": [P, P, I],
        }
        for name, args in sig.items():
            fn = getattr(_lib, name)
            fn.argtypes = args
            fn.restype = None
        _lib.oracle_e4m3.argtypes = [ctypes.c_float]
        _lib.oracle_e4m3.restype = ctypes.c_uint8
        _lib.oracle_ln_stats.argtypes = [P, ctypes.c_int, P, P]
        _lib.oracle_ln_stats.restype = None
    return _lib


# ----------------------------------------------------------------- bf16 helpers
def f32_to_bf16_bits(x: np.ndarray) -> np.ndarray:
    """Round fp32 -> bf16 (nearest even), returned as uint16 bit patterns."""
    u = np.ascontiguousarray(x, dtype=np.float32).view(np.uint32).astype(np.uint64)
    r = ((u + 0x7FFF + ((u >> 16) & 1)) >> 16).astype(np.uint16)
    nan = np.isnan(np.asarray(x, dtype=np.float32))
    if nan.any():
        r[nan] = 0x7FC0
    return r


def bf16_bits_to_f32(b: np.ndarray) -> np.ndarray:
    return (np.asarray(b, dtype=np.uint16).astype(np.uint32) << 16).view(np.float32)


def _p(a: np.ndarray | None):
    return None if a is None else a.ctypes.data_as(ctypes.c_void_p)


def _c(a, dtype):
    return np.ascontiguousarray(a, dtype=dtype)


# ----------------------------------------------------------------- C-backed ops
def mx_quantize(x_bits: np.ndarray):
    """bf16 [rows, k] -> (codes uint8 [padded, k], scales uint8 [padded*k/32])."""
    x = _c(x_bits, np.uint16)
    rows, k = x.shape
    padded = (rows + 127) // 128 * 128
    qv = np.zeros((padded, k), np.uint8)
    qs = np.zeros(padded * k // 32, np.uint8)
    lib().oracle_mx_quantize(_p(x), k, _p(qv), _p(qs), rows, k)
    return qv, qs


def ln_mod(x_bits, scale_bits, shift_bits, rows_per_batch, eps=1e-6):
    x = _c(x_bits, np.uint16)
    rows, dim = x.shape
    out = np.empty_like(x)
    sc = _c(scale_bits, np.uint16)
    sh = None if shift_bits is None else _c(shift_bits, np.uint16)
    lib().oracle_ln_mod(_p(x), _p(sc), _p(sh), _p(out), rows, dim, rows_per_batch, eps)
    return out


def ln_mod_quant(x_bits, scale_bits, shift_bits, rows_per_batch, eps=1e-6):
    x = _c(x_bits, np.uint16)
    rows, dim = x.shape
    padded = (rows + 127) // 128 * 128
    qv = np.zeros((padded, dim), np.uint8)
    qs = np.zeros(padded * dim // 32, np.uint8)
    sc = _c(scale_bits, np.uint16)
    sh = None if shift_bits is None else _c(shift_bits, np.uint16)
    lib().oracle_ln_mod_quant(_p(x), _p(sc), _p(sh), _p(qv), _p(qs), rows, dim, rows_per_batch, eps)
    return qv, qs


def adaln_residual(x_bits, r_bits, scale_bits, shift_bits, gate_bits, rows_per_batch, eps=1e-6):
    x = _c(x_bits, np.uint16)
    rows, dim = x.shape
    out = np.empty_like(x)
    args = [_c(a, np.uint16) for a in (r_bits, scale_bits, shift_bits, gate_bits)]
    lib().oracle_adaln_residual(_p(x), *map(_p, args), _p(out), rows, dim, rows_per_batch, eps)
    return out


def ln_stats(x_row_bits):
    x = _c(x_row_bits, np.uint16)
    m, v = np.zeros(1, np.float32), np.zeros(1, np.float32)
    lib().oracle_ln_stats(_p(x), x.shape[-1], _p(m), _p(v))
    return float(m[0]), float(v[0])


def gated_residual(h_bits, x_bits, gate_bits, rows_per_batch):
    h = _c(h_bits, np.uint16)
    rows, dim = h.shape
    out = np.empty_like(h)
    x, g = _c(x_bits, np.uint16), _c(gate_bits, np.uint16)
    lib().oracle_gated_residual(_p(h), _p(x), _p(g), _p(out), rows, dim, rows_per_batch)
    return out


def rms_norm(x_bits, w_bits, eps=1e-6):
    x = _c(x_bits, np.uint16)
    out = np.empty_like(x)
    lib().oracle_rms_norm(_p(x), _p(_c(w_bits, np.uint16)), _p(out), x.size // 128, eps)
    return out


def rope_qk(q_bits, k_bits, freqs):
    q, k = _c(q_bits, np.uint16), _c(k_bits, np.uint16)
    b, s, h, d = q.shape
    oq, ok = np.empty_like(q), np.empty_like(k)
    lib().oracle_rope_qk(_p(q), _p(k), _p(_c(freqs, np.float32)), _p(oq), _p(ok), b, s, h)
    return oq, ok


def qknorm_rope_pack(q, k, v, ck, cv, wq, wk, freqs, eps_q=1e-6, eps_k=1e-6):
    q, k, v = (_c(a, np.uint16) for a in (q, k, v))
    b, s, h, d = q.shape
    p = 0 if ck is None else ck.shape[1]
    ck = None if ck is None else _c(ck, np.uint16)
    cv = None if cv is None else _c(cv, np.uint16)
    oq = np.empty_like(q)
    ok = np.empty((b, p + s, h, d), np.uint16)
    ov = np.empty_like(ok)
    lib().oracle_qknorm_rope_pack(_p(q), _p(k), _p(v), _p(ck), _p(cv), _p(_c(wq, np.uint16)),
                                  _p(_c(wk, np.uint16)), _p(_c(freqs, np.float32)), _p(oq), _p(ok), _p(ov),
                                  b, s, p, h, eps_q, eps_k)
    return oq, ok, ov


def qknorm_rope_segment(qkv, wq, wk, freqs, oq, ok, ov, batch, seg_len, seq_offset, heads, eps_q=1e-6, eps_k=1e-6):
    """Writes one segment into the preallocated joint outputs oq/ok/ov (uint16)."""
    x = _c(qkv, np.uint16)
    seq_total = oq.shape[1]
    lib().oracle_qknorm_rope_segment(_p(x), x.shape[-1], _p(_c(wq, np.uint16)), _p(_c(wk, np.uint16)),
                                     _p(_c(freqs, np.float32)), _p(oq), _p(ok), _p(ov), batch, seg_len,
                                     seq_offset, seq_total, heads, eps_q, eps_k)


def swiglu(g_bits, v_bits):
    g, v = _c(g_bits, np.uint16), _c(v_bits, np.uint16)
    out = np.empty_like(g)
    lib().oracle_swiglu(_p(g), _p(v), _p(out), g.size)
    return out


def swiglu_quant(g_bits, v_bits):
    g, v = _c(g_bits, np.uint16), _c(v_bits, np.uint16)
    rows, width = g.shape
    padded = (rows + 127) // 128 * 128
    qv = np.zeros((padded, width), np.uint8)
    qs = np.zeros(padded * width // 32, np.uint8)
    lib().oracle_swiglu_quant(_p(g), _p(v), _p(qv), _p(qs), rows, width)
    return qv, qs


def gelu_tanh(x_bits):
    x = _c(x_bits, np.uint16)
    out = np.empty_like(x)
    lib().oracle_gelu_tanh(_p(x), _p(out), x.size)
    return out


def e4m3(x: float) -> int:
    return int(lib().oracle_e4m3(ctypes.c_float(x)))


# ----------------------------------------------------------------- numpy MXFP8
_E4M3_TABLE = None


def e4m3_decode_table() -> np.ndarray:
    """fp32 value of each E4M3 (fn) code."""
    global _E4M3_TABLE
    if _E4M3_TABLE is None:
        t = np.zeros(256, np.float32)
        for c in range(256):
            s = -1.0 if c & 0x80 else 1.0
            e = (c >> 3) & 0xF
            m = c & 7
            if e == 0xF and m == 7:
                t[c] = np.nan
            elif e == 0:
                t[c] = s * m * 2.0 ** -9
            else:
                t[c] = s * (1 + m / 8.0) * 2.0 ** (e - 7)
        _E4M3_TABLE = t
    return _E4M3_TABLE


def mx_quantize_numpy(x_bits: np.ndarray):
    """Independent restatement of the reference's known-answer test
    (tests/gpu/check_mxfp8.py:41-55): exponent from the amax bits, codes of
    x * 2^(127-e), scales swizzled (m/128, 4, 32, kb/4, 4) -> (0, 3, 2, 1, 4)."""
    x = bf16_bits_to_f32(_c(x_bits, np.uint16))
    m, k = x.shape
    padded = (m + 127) // 128 * 128
    xp = np.zeros((padded, k), np.float32)
    xp[:m] = x
    blocks = xp.reshape(padded, k // 32, 32)
    amax = np.abs(blocks).max(-1)
    bits = amax.view(np.uint32).astype(np.int64)
    e = ((bits >> 23) & 0xFF) - 8 + ((bits & 0x7FFFFF) > 6291456).astype(np.int64)
    e = np.where(amax == 0, 0, np.clip(e, 0, 254))
    inv = ((254 - e).astype(np.uint32) << 23).view(np.float32)
    scaled = (blocks * inv[..., None]).reshape(padded, k)
    codes = _encode_e4m3(scaled)
    sw = e.astype(np.uint8).reshape(padded // 128, 4, 32, k // 128, 4).transpose(0, 3, 2, 1, 4).reshape(-1)
    return codes, sw


def _encode_e4m3(v: np.ndarray) -> np.ndarray:
    """Vectorised RNE satfinite fp32 -> E4M3 through the exact code table."""
    table = e4m3_decode_table()
    pos = table[:127]                      # codes 0..126, increasing, all finite
    a = np.minimum(np.abs(v).astype(np.float64), 448.0)
    idx = np.searchsorted(pos, a, side="left")
    idx = np.clip(idx, 1, 126)
    lo, hi = pos[idx - 1].astype(np.float64), pos[idx].astype(np.float64)
    pick_hi = (a - lo > hi - a) | ((a - lo == hi - a) & (idx % 2 == 0))
    code = np.where(pick_hi, idx, idx - 1)
    code = np.where(a == 0, 0, code).astype(np.uint8)
    # negative inputs keep their sign bit, including those rounding to zero (0x80)
    return np.where(np.signbit(v), code | 0x80, code).astype(np.uint8)


def mx_dequantize(codes: np.ndarray, scales: np.ndarray, rows: int) -> np.ndarray:
    """MXFP8 -> fp32 [rows, k]: code value * 2^(e-127)."""
    padded, k = codes.shape
    vals = e4m3_decode_table()[codes]
    e = scales.reshape(padded // 128, k // 128, 32, 4, 4).transpose(0, 3, 2, 1, 4).reshape(padded, k // 32)
    mult = np.ldexp(np.float32(1.0), e.astype(np.int32) - 127).astype(np.float32)
    return (vals.reshape(padded, k // 32, 32) * mult[..., None]).reshape(padded, k)[:rows]


def mxfp8_gemm(a_codes, a_scales, b_codes, b_scales, m: int, n: int, bias=None) -> np.ndarray:
    """Block-scaled GEMM restated as dequantize -> fp64 matmul -> fp32 [m, n]
    (reference src/qwen_image_accel/optimizations/mxfp8.py:32-36, torch._scaled_mm)."""
    a = mx_dequantize(a_codes, a_scales, m).astype(np.float64)
    b = mx_dequantize(b_codes, b_scales, n).astype(np.float64)
    y = a @ b.T
    if bias is not None:
        y = y + bias.astype(np.float64)[None, :]
    return y.astype(np.float32)


# ----------------------------------------------------------------- Sage attention
def sage_quant_q(q: np.ndarray, blk: int = 32):
    """Per-(32-token warp block, head) INT8 of Q (SAGE:csrc/fused/fused.cu:64-198
    with BLKQ=128, WARPQ=32): scale = amax/127 (amax floor 1e-7), codes =
    rint(x * 127/amax) saturated to [-127, 127]. q: fp32 [B, S, H, D].

    The divides here are IEEE; the reference's extension is built with
    --use_fast_math, whose approximate divide can land an ulp away, so a code
    whose x * 127/amax sits within that of a rounding boundary can differ by
    one (and a scale by an ulp or two). The kernels use the reference's
    divide and are pinned bit for bit against the built reference on the GPU
    (tests/test_sage_ref_gpu.py); against this restatement the tests count
    and bound those differences."""
    b, s, h, d = q.shape
    nblk = (s + blk - 1) // blk
    qp = np.zeros((b, nblk * blk, h, d), np.float32)
    qp[:, :s] = q
    blocks = qp.reshape(b, nblk, blk, h, d)
    amax = np.maximum(np.abs(blocks).max(axis=(2, 4)), np.float32(1e-7))   # [b, nblk, h]
    inv = (np.float32(127.0) / amax).astype(np.float32)
    codes = np.clip(np.rint(blocks * inv[:, :, None, :, None]), -128, 127).astype(np.int8)
    scale = (amax / np.float32(127.0)).astype(np.float32).transpose(0, 2, 1)   # [b, h, nblk]
    return codes.reshape(b, nblk * blk, h, d)[:, :s], scale


def sage_k_mean(k: np.ndarray) -> np.ndarray:
    """Per-(batch, head, channel) mean of K over the sequence, rounded to bf16
    (SAGE:sageattention/core.py:773, k.mean(dim=seq) on a bf16 tensor). The
    reference sums in torch's reduction order; this restates the kernels' own
    fp32 order (pinned against torch's k.mean on the GPU, where at most 1 in
    500 elements may land one bf16 ulp apart: tests/test_sage_ref_gpu.py): per 32-row tile, sixteen fp32 row-group sums (rows g and
    g+16 of the tile, in order, added to 0.0); the groups paired (g + (g+1)
    for even g); the eight pair sums added in order to 0.0 (the tile sum);
    the tile sums as eight interleaved sub-sums (tiles j, j+8, j+16, ... in
    order, from 0.0), added in sub order to 0.0; times fp32(1/S)."""
    b, s, h, d = k.shape
    parts = []
    for t0 in range(0, s, 32):
        grp = []
        for g in range(16):
            acc = np.zeros((b, h, d), np.float32)
            for i in range(t0 + g, min(s, t0 + 32), 16):
                acc += k[:, i].astype(np.float32)
            grp.append(acc)
        part = np.zeros((b, h, d), np.float32)
        for w in range(8):
            part += (grp[2 * w] + grp[2 * w + 1]).astype(np.float32)
        parts.append(part)
    subs = []
    for j in range(8):
        acc = np.zeros((b, h, d), np.float32)
        for part in parts[j::8]:
            acc += part
        subs.append(acc)
    total = np.zeros((b, h, d), np.float32)
    for acc in subs:
        total += acc
    mean = (total * np.float32(1.0 / s)).astype(np.float32)
    return bf16_bits_to_f32(f32_to_bf16_bits(mean))


def sage_quant_k(k: np.ndarray, blk: int = 64):
    """K smoothing (minus the bf16-rounded sequence mean) then
    per-(64-token block, head) INT8 (SAGE:csrc/fused/fused.cu:594-683)."""
    km = sage_k_mean(k)                                  # [b, h, d]
    ks = (k - km[:, None]).astype(np.float32)
    codes, scale = sage_quant_q(ks, blk)
    return codes, scale, km


def sage_quant_v(v: np.ndarray, scale_max: float = 448.0):
    """Per-(batch, head, channel) FP8: scale = amax/448 over the sequence,
    codes = E4M3(x * 448/amax) (SAGE:csrc/fused/fused.cu:316-427, no smoothing)."""
    amax = np.abs(v).max(axis=1).astype(np.float32)              # [b, h, d]
    scale = (amax / np.float32(scale_max)).astype(np.float32)
    with np.errstate(divide="ignore"):
        recp = np.where(amax > 0, np.float32(scale_max) / amax, np.float32(0)).astype(np.float32)
    codes = _encode_e4m3((v * recp[:, None]).astype(np.float32))
    return codes, scale


def block_causal_mask(image_ids: np.ndarray, key_valid: np.ndarray | None = None) -> np.ndarray:
    """The Qwen-Image 2.1 prefill mask, densely: query q may see key kv when
    kv <= q or both are tokens of the same image block, and kv is a valid key
    (WHL:diffusers/models/transformers/transformer_qwenimage21.py:291-296,
    `mask_mod` of build_qwenimage21_block_causal_mask). image_ids: int [S],
    -1 at text tokens; key_valid: bool [B, S] or None. Returns bool [B, S, S]
    (B = 1 without key_valid)."""
    ids = np.asarray(image_ids, np.int64)
    s = ids.shape[0]
    q = np.arange(s)[:, None]
    kv = np.arange(s)[None, :]
    same = (ids[:, None] == ids[None, :]) & (ids[:, None] >= 0)
    allowed = (q >= kv) | same
    if key_valid is None:
        return allowed[None]
    return allowed[None] & np.asarray(key_valid, bool)[:, None, :]


def block_causal_kv_limits(image_ids: np.ndarray) -> np.ndarray:
    """One key limit per query that reproduces block_causal_mask without a key
    mask when every image block is one contiguous run (as
    QwenImage21Transformer2DModel.build_token_metadata assigns them,
    transformer_qwenimage21.py:808-844): q + 1 for a text token, the end of
    its run for an image token -- the `[0, end)` keys each prefix segment sees
    in QwenImage21AttnProcessor (transformer_qwenimage21.py:502-541). Plain
    loop restatement; int32 [S]."""
    ids = [int(x) for x in np.asarray(image_ids).ravel()]
    s = len(ids)
    out = np.zeros(s, np.int32)
    end = s
    for i in range(s - 1, -1, -1):
        if i == s - 1 or ids[i + 1] != ids[i]:
            end = i + 1
        out[i] = i + 1 if ids[i] < 0 else end
    return out


def sage_attention(q: np.ndarray, k: np.ndarray, v: np.ndarray, sm_scale: float | None = None,
                   kv_limit: np.ndarray | None = None) -> np.ndarray:
    """Sage-style attention (SAGE:sageattention/core.py:725-828): INT8 Q/K with
    K smoothing, fp32 softmax in base 2 with the +log2(448) offset so that P
    lands in [0, 448], P rounded to E4M3, FP8 V with per-channel scales, output
    divided by the row sum of the unrounded P. Inputs fp32 [B, S, H, D];
    returns fp32 [B, Sq, H, D]. kv_limit (int [B, Sq] or [Sq]): query t sees
    keys [0, limit) only -- the row max and the row sum run over those keys,
    the others get P = 0; the quantization is unchanged (K's mean still runs
    over all keys). A row with no visible key is zero."""
    b, sq, h, d = q.shape
    if sm_scale is None:
        sm_scale = d ** -0.5
    qc, qs = sage_quant_q(q, 32)
    kc, ks, _ = sage_quant_k(k, 64)
    vc, vs = sage_quant_v(v)
    table = e4m3_decode_table()
    out = np.zeros((b, sq, h, d), np.float32)
    log2e = np.float32(1.4426950408889634)
    for bi in range(b):
        for hi in range(h):
            s_int = qc[bi, :, hi, :].astype(np.int32) @ kc[bi, :, hi, :].astype(np.int32).T   # [sq, skv]
            qscale = np.repeat(qs[bi, hi], 32)[:sq]
            kscale = np.repeat(ks[bi, hi], 64)[: k.shape[1]]
            sc = s_int.astype(np.float32) * (qscale[:, None] * kscale[None, :]) * np.float32(sm_scale * log2e)
            if kv_limit is None:
                m = sc.max(axis=1, keepdims=True) - np.float32(8.807)
                p = np.exp2(sc - m).astype(np.float32)
            else:
                lim = np.asarray(kv_limit).reshape(-1, sq)[bi if np.asarray(kv_limit).ndim > 1 else 0]
                seen = np.arange(k.shape[1])[None, :] < np.clip(lim, 0, k.shape[1])[:, None]
                m = np.where(seen, sc, -np.inf).max(axis=1, keepdims=True) - np.float32(8.807)
                m = np.where(np.isfinite(m), m, 0.0).astype(np.float32)
                p = np.where(seen, np.exp2(sc - m), 0.0).astype(np.float32)
            denom = p.sum(axis=1, keepdims=True)
            p8 = table[_encode_e4m3(p)]
            vv = table[vc[bi, :, hi, :]]
            o = (p8.astype(np.float64) @ vv.astype(np.float64)).astype(np.float32)
            safe = np.where(denom > 0, denom, 1.0)
            out[bi, :, hi, :] = np.where(denom > 0, o / safe, 0.0) * vs[bi, hi][None, :]
    return out


def attention_fp32(q, k, v, sm_scale=None, mask=None):
    """Exact softmax attention in fp64 (reference for cosine checks). mask:
    bool [B, Sq, Skv] (or [1, Sq, Skv]) of visible keys, or None; a row with
    no visible key is zero."""
    b, sq, h, d = q.shape
    if sm_scale is None:
        sm_scale = d ** -0.5
    out = np.zeros((b, sq, h, d), np.float32)
    for bi in range(b):
        for hi in range(h):
            s = q[bi, :, hi, :].astype(np.float64) @ k[bi, :, hi, :].astype(np.float64).T * sm_scale
            if mask is not None:
                s = np.where(mask[bi if mask.shape[0] > 1 else 0], s, -np.inf)
            mx = s.max(axis=1, keepdims=True)
            p = np.exp(s - np.where(np.isfinite(mx), mx, 0.0))
            den = p.sum(axis=1, keepdims=True)
            p = np.where(den > 0, p / np.where(den > 0, den, 1.0), 0.0)
            out[bi, :, hi, :] = (p @ v[bi, :, hi, :].astype(np.float64)).astype(np.float32)
    return out

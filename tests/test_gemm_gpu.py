"""GPU parity of the tcgen05 block-scaled MXFP8 GEMM and its epilogues.

Contract: within 1e-2 relative Frobenius error of a BF16
reference GEMM of the same (dequantized) operands. We also check against the
fp32 product of the dequantized operands (the exact algorithm; only the
accumulation order and the final bf16 rounding differ) and, on a small case,
against the CPU oracle (oracle.mxfp8_gemm: dequantize -> fp64 matmul).
"""
import numpy as np
import pytest
import torch
import torch.nn.functional as F

import oracle

pytestmark = pytest.mark.gpu
DEV = "cuda"


@pytest.fixture(autouse=True)
def _cuda():
    if not torch.cuda.is_available():
        pytest.skip("needs a CUDA device")


def dequant(q):
    """fp32 (rows, K) value of a Quantized activation/weight."""
    vals = q.values.float()
    padded, k = vals.shape
    e = q.scales.view(torch.uint8).view(padded // 128, k // 128, 32, 4, 4).permute(0, 3, 2, 1, 4).reshape(padded,
                                                                                                           k // 32)
    return (vals.view(padded, k // 32, 32) * torch.exp2(e.float() - 127)[..., None]).view(padded, k)[: q.rows]


def rel_fro(a, b):
    a, b = a.double(), b.double()
    return ((a - b).norm() / b.norm()).item()


def make_linear(n, k, seed, bias=True):
    g = torch.Generator(device=DEV).manual_seed(seed)
    lin = torch.nn.Linear(k, n, bias=bias, device=DEV, dtype=torch.bfloat16)
    with torch.no_grad():
        lin.weight.copy_(0.02 * torch.randn(n, k, device=DEV, generator=g))
        if bias:
            lin.bias.copy_(0.01 * torch.randn(n, device=DEV, generator=g))
    return lin


def make_x(m, k, seed):
    g = torch.Generator(device=DEV).manual_seed(seed)
    return torch.randn(m, k, device=DEV, dtype=torch.bfloat16, generator=g)


@pytest.mark.parametrize("bn", ["128", "192", "256"])
@pytest.mark.parametrize("m,n,k", [(128, 768, 256), (77, 384, 512), (300, 1536, 384), (4352, 3072, 3072),
                                   (4352, 9216, 3072), (512, 12288, 3072), (200, 3072, 12288)])
def test_gemm_matches_references(monkeypatch, bn, m, n, k):
    from qwen_image_accel_b200.kernels.mxfp8 import quantize
    from qwen_image_accel_b200.optimizations.mxfp8 import MXFP8Linear
    if n % int(bn):
        pytest.skip("tile width does not divide N")
    monkeypatch.setenv("QIA_GEMM_BN", bn)
    lin = make_linear(n, k, 1)
    mx = MXFP8Linear(lin)
    x = make_x(m, k, 2)
    a = quantize(x)
    y = mx.matmul(a)
    torch.cuda.synchronize()
    from qwen_image_accel_b200 import _lib
    assert _lib.device_error() == 0
    wq = type(a)(mx.weight_fp8.t(), mx.weight_scale, n, torch.Size((n, k)))
    da, dw = dequant(a), dequant(wq)
    exact = da @ dw.T + lin.bias.float()
    assert rel_fro(y.float(), exact) < 4e-3            # only accumulation order + bf16 output rounding
    bf16_ref = F.linear(da.to(torch.bfloat16), dw.to(torch.bfloat16), lin.bias)
    assert rel_fro(y.float(), bf16_ref.float()) < 1e-2  # north_star contract
    # element-wise: within 2 bf16 ulps of the exact product almost everywhere
    tol = exact.abs() * 2 ** -7 + 1e-4
    assert ((y.float() - exact).abs() <= tol).float().mean().item() > 0.999


def test_gemm_vs_cpu_oracle():
    from qwen_image_accel_b200.kernels.mxfp8 import quantize
    from qwen_image_accel_b200.optimizations.mxfp8 import MXFP8Linear
    m, n, k = 77, 384, 256
    lin = make_linear(n, k, 3)
    mx = MXFP8Linear(lin)
    x = make_x(m, k, 4)
    a = quantize(x)
    y = mx.matmul(a)
    xb = x.cpu().view(torch.int16).numpy().view(np.uint16)
    wb = lin.weight.detach().cpu().view(torch.int16).numpy().view(np.uint16)
    aq, asc = oracle.mx_quantize(xb)
    wq, wsc = oracle.mx_quantize(wb)
    assert np.array_equal(a.values.cpu().view(torch.uint8).numpy(), aq)
    bias = lin.bias.detach().float().cpu().numpy()
    ref = oracle.mxfp8_gemm(aq, asc, wq, wsc, m, n, bias)
    got = y.float().cpu().numpy()
    assert np.linalg.norm(got - ref) / np.linalg.norm(ref) < 4e-3


def test_quantization_error_vs_bf16_linear_is_reported():
    """Information: MXFP8 (both operands E4M3) vs the unquantized BF16 linear."""
    from qwen_image_accel_b200.optimizations.mxfp8 import MXFP8Linear
    lin = make_linear(3072, 3072, 5)
    x = make_x(4352, 3072, 6)
    y = MXFP8Linear(lin)(x)
    ref = x.float() @ lin.weight.float().T + lin.bias.float()
    err = rel_fro(y.float(), ref)
    print(f"MXFP8 vs unquantized BF16 linear: rel Frobenius {err:.4f}")
    assert err < 0.08


@pytest.mark.parametrize("m", [77, 300, 4352])
def test_gelu_epilogues(m):
    from qwen_image_accel_b200.kernels.mxfp8 import quantize
    from qwen_image_accel_b200.optimizations.mxfp8 import MXFP8Linear
    n, k = 12288, 3072
    lin = make_linear(n, k, 7)
    mx = MXFP8Linear(lin)
    a = quantize(make_x(m, k, 8))
    h = mx.matmul(a)                       # bf16(acc + bias)
    g = mx.matmul_gelu(a)
    ref_g = F.gelu(h, approximate="tanh")
    assert ((g.float() - ref_g.float()).abs() <= ref_g.float().abs() * 2 ** -7 + 1e-5).float().mean().item() > 0.999
    q = mx.matmul_gelu_quantize(a)
    sep = quantize(g)
    same = (q.values.view(torch.uint8) == sep.values.view(torch.uint8)).float().mean().item()
    assert same > 0.999
    assert rel_fro(dequant(q), dequant(sep)) < 5e-3
    padded = q.values.shape[0]
    if padded > m:
        assert int(q.values.view(torch.uint8)[m:].abs().sum()) == 0


@pytest.mark.parametrize("inplace", [False, True])
def test_gate_residual_epilogue(inplace):
    from qwen_image_accel_b200.kernels.mxfp8 import quantize
    from qwen_image_accel_b200.optimizations.mxfp8 import MXFP8Linear
    b, s, n, k = 2, 4096, 3072, 12288
    lin = make_linear(n, k, 9)
    mx = MXFP8Linear(lin)
    a = quantize(make_x(b * s, k, 10))
    g = torch.Generator(device=DEV).manual_seed(11)
    resid = torch.randn(b, s, n, device=DEV, dtype=torch.bfloat16, generator=g)
    gate = 0.1 * torch.randn(b, 1, n, device=DEV, dtype=torch.bfloat16, generator=g)
    y = mx.matmul(a).view(b, s, n)
    ref = resid + gate * y
    r0 = resid.clone()
    out = mx.matmul_gate_residual(a, gate, resid, out=resid if inplace else None)
    assert rel_fro(out.float(), ref.float()) < 1e-3
    assert ((out.float() - ref.float()).abs() <= ref.float().abs() * 2 ** -7 + 1e-4).float().mean().item() > 0.999
    if not inplace:
        assert torch.equal(resid, r0)


def test_full_size_bf16_contract():
    """Full BASELINE size (M=16640, FFN up 3072->12288): the north_star bound
    against cuBLAS BF16 on the dequantized operands."""
    from qwen_image_accel_b200.kernels.mxfp8 import quantize
    from qwen_image_accel_b200.optimizations.mxfp8 import MXFP8Linear
    m, n, k = 16640, 12288, 3072
    lin = make_linear(n, k, 12)
    mx = MXFP8Linear(lin)
    a = quantize(make_x(m, k, 13))
    y = mx.matmul(a)
    wq = type(a)(mx.weight_fp8.t(), mx.weight_scale, n, torch.Size((n, k)))
    ref = F.linear(dequant(a).to(torch.bfloat16), dequant(wq).to(torch.bfloat16), lin.bias)
    assert rel_fro(y.float(), ref.float()) < 1e-2


# BASELINE config 2, every shape of the sweep: M in {4352, 16640} x (QKV
# 3072->9216, out 3072->3072, FFN up 3072->12288 with the GELU-tanh epilogue,
# FFN down 12288->3072), activations ~N(0, 1), weights ~N(0, 0.02), bias
# ~N(0, 0.01), seed 1; the launch picks its tile width as in the model.
@pytest.mark.parametrize("m", [4352, 16640])
@pytest.mark.parametrize("n,k,gelu", [(9216, 3072, False), (3072, 3072, False), (12288, 3072, True),
                                      (3072, 12288, False)])
def test_config2_sweep_shapes(m, n, k, gelu):
    from qwen_image_accel_b200 import _lib
    from qwen_image_accel_b200.kernels.mxfp8 import quantize
    from qwen_image_accel_b200.optimizations.mxfp8 import MXFP8Linear
    lin = make_linear(n, k, 1)
    mx = MXFP8Linear(lin)
    a = quantize(make_x(m, k, 1))
    y = mx.matmul_gelu(a) if gelu else mx.matmul(a)
    torch.cuda.synchronize()
    assert _lib.device_error() == 0
    assert y.shape == (m, n)
    wq = type(a)(mx.weight_fp8.t(), mx.weight_scale, n, torch.Size((n, k)))
    da, dw = dequant(a), dequant(wq)
    bf16_ref = F.linear(da.to(torch.bfloat16), dw.to(torch.bfloat16), lin.bias)
    exact = da @ dw.T + lin.bias.float()
    if gelu:
        bf16_ref = F.gelu(bf16_ref, approximate="tanh")
        exact = F.gelu(exact, approximate="tanh")
    del da, dw
    assert rel_fro(y.float(), bf16_ref.float()) < 1e-2   # north_star contract
    assert rel_fro(y.float(), exact) < 4e-3              # accumulation order + bf16 roundings only


@pytest.mark.parametrize("bn", ["192", "256"])
@pytest.mark.parametrize("pad", [0, 8, 16])
def test_gemm_output_row_stride(monkeypatch, bn, pad):
    """Outputs with a row stride ldo = N + pad + 8 and a start offset of `pad`
    elements: rows whose start is 32-byte aligned take 32-byte stores, the
    others 16-byte stores. Every path must write exactly the [M, N] window,
    including the partial last row block (M = 300), at both tile widths."""
    from qwen_image_accel_b200.kernels.mxfp8 import quantize
    from qwen_image_accel_b200.optimizations.mxfp8 import MXFP8Linear
    monkeypatch.setenv("QIA_GEMM_BN", bn)
    m, n, k = 300, 1536, 384
    lin = make_linear(n, k, 16)
    mx = MXFP8Linear(lin)
    a = quantize(make_x(m, k, 17))
    monkeypatch.setenv("QIA_GEMM_BN", "128")
    ref = mx.matmul(a)
    monkeypatch.setenv("QIA_GEMM_BN", bn)
    buf = torch.full((m, n + pad + 8), -7.0, device=DEV, dtype=torch.bfloat16)
    out = buf[:, pad:pad + n]
    mx.matmul(a, out=out)
    torch.cuda.synchronize()
    assert torch.equal(out, ref)
    assert bool((buf[:, :pad] == -7.0).all()) and bool((buf[:, pad + n:] == -7.0).all())
    from qwen_image_accel_b200 import _lib
    assert _lib.device_error() == 0


@pytest.mark.parametrize("bn", ["128", "192", "256", None])
@pytest.mark.parametrize("m0,m1,n,k", [(8192, 512, 768, 256), (300, 77, 384, 384), (128, 1000, 1536, 256)])
def test_grouped_launch_matches_single_gemms(monkeypatch, bn, m0, m1, n, k):
    """Two GEMMs in one grouped launch (each epilogue) give byte-identical
    outputs to the single-GEMM entry points, including a group whose first
    problem is the small one and rows that are not multiples of 128."""
    from qwen_image_accel_b200.kernels.mxfp8 import quantize
    from qwen_image_accel_b200.optimizations.mxfp8 import (MXFP8Linear, matmul_gate_residual_grouped,
                                                            matmul_gelu_quantize_grouped, matmul_grouped)
    if bn is not None:
        monkeypatch.setenv("QIA_GEMM_BN", bn)
    lins = [MXFP8Linear(make_linear(n, k, 40 + i)) for i in range(2)]
    acts = [quantize(make_x(m, k, 50 + i)) for i, m in enumerate((m0, m1))]
    got = matmul_grouped(list(zip(lins, acts)))
    for lin, act, out in zip(lins, acts, got):
        assert torch.equal(out, lin.matmul(act))
    got_q = matmul_gelu_quantize_grouped(list(zip(lins, acts)))
    for lin, act, q in zip(lins, acts, got_q):
        ref = lin.matmul_gelu_quantize(act)
        assert torch.equal(q.values.view(torch.uint8)[: q.rows], ref.values.view(torch.uint8)[: ref.rows])
        assert torch.equal(q.scales.view(torch.uint8), ref.scales.view(torch.uint8))
    g = torch.Generator(device=DEV).manual_seed(60)
    items, refs = [], []
    for lin, act, m in zip(lins, acts, (m0, m1)):
        batch = 2 if m % 2 == 0 else 1
        gate = torch.randn(batch, 1, n, device=DEV, dtype=torch.bfloat16, generator=g)
        resid = torch.randn(m, n, device=DEV, dtype=torch.bfloat16, generator=g)
        refs.append(lin.matmul_gate_residual(act, gate, resid.clone()))
        items.append((lin, act, gate, resid))
    matmul_gate_residual_grouped(items)
    for (_, _, _, resid), ref in zip(items, refs):
        assert torch.equal(resid, ref)
    torch.cuda.synchronize()
    from qwen_image_accel_b200 import _lib
    assert _lib.device_error() == 0


@pytest.mark.parametrize("bn", ["128", "256", None])
@pytest.mark.parametrize("m,f,k", [(300, 384, 256), (4096, 1536, 512), (130, 128, 384)])
def test_swiglu_epilogue_matches_gemm_pair_then_swiglu_quantize(monkeypatch, bn, m, f, k):
    """qia_mxfp8_gemm_swiglu_quant over the interleaved [W_gate; W_value]
    stack is byte-identical to the two bf16 GEMMs followed by
    swiglu_quantize (codes, scales and the zero padding rows)."""
    import torch.nn as nn
    from qwen_image_accel_b200.kernels.epilogue import swiglu_quantize
    from qwen_image_accel_b200.kernels.mxfp8 import quantize
    from qwen_image_accel_b200.optimizations.mxfp8 import MXFP8Linear, interleaved_gate_value
    if bn:
        monkeypatch.setenv("QIA_GEMM_BN", bn)
    else:
        monkeypatch.delenv("QIA_GEMM_BN", raising=False)
    gate, value = make_linear(f, k, 5, bias=False), make_linear(f, k, 6, bias=False)
    stacked = nn.Linear(k, 2 * f, bias=False, device="cuda", dtype=torch.bfloat16)
    with torch.no_grad():
        stacked.weight.copy_(interleaved_gate_value(gate.weight, value.weight))
    mg, mv, ms = MXFP8Linear(gate), MXFP8Linear(value), MXFP8Linear(stacked)
    a = quantize(make_x(m, k, 7))
    want = swiglu_quantize(mg.matmul(a), mv.matmul(a))
    got = ms.matmul_swiglu_quantize(a)
    assert got.rows == want.rows and got.values.shape == want.values.shape
    assert torch.equal(got.values.view(torch.uint8), want.values.view(torch.uint8))
    assert torch.equal(got.scales.view(torch.uint8), want.scales.view(torch.uint8))

"""The Ulysses peer-memory exchange kernels on one GPU (csrc/ulysses_p2p.cu,
qia_sage_attn_quantized_peers): two ranks of a Ulysses group are emulated by
two launches into two local buffer sets, in sequence (no kernel waits on
another launch), so the layouts, the signals and the outputs are checked here;
tests/test_ulysses_gpu.py runs the real exchange between GPUs.

* qia_ulysses_wait gives up after its time limit when nothing signals, and
  reports QIA_ERR_TIMEOUT through the device error word (no GPU fault, the
  context stays usable), and passes rounds whose signals are all present;
* qia_ulysses_scatter_qkv puts every rank's q|k|v rows where the fused
  quantizer of the heads' owner reads them, and signals each rank once per
  launch;
* qia_sage_attn_quantized_peers writes each image row to the token's owner and
  the text rows to every rank, byte-identical to the single-GPU split
  attention of the same heads, and signals each rank once per CTA.
"""
import ctypes

import pytest
import torch

pytestmark = pytest.mark.gpu
DEV = "cuda"
TIMEOUT = 5


@pytest.fixture(autouse=True)
def _cuda():
    if not torch.cuda.is_available():
        pytest.skip("needs a CUDA device")


def _lib():
    from qwen_image_accel_b200 import _lib
    return _lib


def test_wait_times_out_without_signals_and_passes_signalled_rounds():
    L = _lib()
    L.device_error()                                    # clear
    counters = torch.zeros(2, dtype=torch.int64, device=DEV)
    rnd = torch.zeros(1, dtype=torch.int64, device=DEV)
    st = L.stream(counters.device)
    # nothing ever signals: the wait gives up after 50 ms
    L.call("qia_ulysses_wait", L.ptr(counters), L.ptr(rnd), 2, 1, 50_000_000, st)
    assert L.device_error() == TIMEOUT
    assert int(rnd.item()) == 1
    # three rounds of one signal per source present: rounds 2..3 pass, round 4 times out
    counters.fill_(3)
    for want_round in (2, 3):
        L.call("qia_ulysses_wait", L.ptr(counters), L.ptr(rnd), 2, 1, 50_000_000, st)
        assert L.device_error() == 0
        assert int(rnd.item()) == want_round
    L.call("qia_ulysses_wait", L.ptr(counters), L.ptr(rnd), 2, 1, 50_000_000, st)
    assert L.device_error() == TIMEOUT
    # the context is still usable
    assert torch.equal(counters + 1, torch.full_like(counters, 4))


def _table(ts):
    return torch.tensor([t.data_ptr() for t in ts], dtype=torch.int64, device=DEV)


@pytest.mark.parametrize("U,s_loc,heads", [(2, 96, 4), (4, 40, 8), (1, 64, 2)])
def test_scatter_layout_and_signals(U, s_loc, heads):
    L = _lib()
    hl = heads // U
    g = torch.Generator(device=DEV).manual_seed(U)
    qkv = torch.randn(U * s_loc, 3 * heads * 128, device=DEV, generator=g).to(torch.bfloat16)
    recv = [torch.zeros(U * s_loc, 3 * hl * 128, device=DEV, dtype=torch.bfloat16) for _ in range(U)]
    sig = [torch.zeros(2 * U + 2, dtype=torch.int64, device=DEV) for _ in range(U)]
    done = torch.zeros(U, dtype=torch.int64, device=DEV)
    rt, sg = _table(recv), _table(sig)
    st = L.stream(qkv.device)
    for u in range(U):                                   # rank u's rows, twice (two rounds)
        rows = qkv[u * s_loc:(u + 1) * s_loc]
        for _ in range(2):
            L.call("qia_ulysses_scatter_qkv", L.ptr(rows), rows.stride(0), s_loc, heads, 128, L.ptr(rt), L.ptr(sg),
                   L.ptr(done[u:]), U, u, st)
    torch.cuda.synchronize()
    assert L.device_error() == 0
    for r in range(U):
        want = qkv.view(U * s_loc, 3, U, hl, 128)[:, :, r].reshape(U * s_loc, 3 * hl * 128)
        assert torch.equal(recv[r], want)
        assert sig[r][:U].tolist() == [2] * U          # one signal per launch
        assert int(sig[r][U:].abs().sum()) == 0


def test_attention_peers_equal_split_attention():
    from qwen_image_accel_b200.kernels.attention import joint_qk_norm_rope
    from qwen_image_accel_b200.mmdit import rope_tables
    from qwen_image_accel_b200.optimizations.sage_attention import sage_attention_split, sage_quantize_joint
    L = _lib()
    U, heads, Lt, grid = 2, 4, 40, (1, 12, 16)
    Li = grid[1] * grid[2]
    s_loc, hl = Li // U, heads // U
    g = torch.Generator(device=DEV).manual_seed(3)
    qkv_t = torch.randn(Lt, 3 * heads * 128, device=DEV, generator=g).to(torch.bfloat16)
    qkv_i = torch.randn(Li, 3 * heads * 128, device=DEV, generator=g).to(torch.bfloat16)
    w = [tuple((1 + 0.1 * torch.randn(128, device=DEV, generator=g)).to(torch.bfloat16) for _ in range(2))
         for _ in range(2)]
    fi, ft = (torch.view_as_real(t).to(DEV).contiguous() for t in rope_tables(*grid, Lt))
    # reference: QK-norm/RoPE into the joint sequence, then the split attention (all heads)
    S = Lt + Li
    q, k, v = (torch.empty(1, S, heads, 128, device=DEV, dtype=torch.bfloat16) for _ in range(3))
    joint_qk_norm_rope(qkv_t[None], w[0][0], w[0][1], ft, q, k, v, 0, 1e-6)
    joint_qk_norm_rope(qkv_i[None], w[1][0], w[1][1], fi, q, k, v, Lt, 1e-6)
    ref_t = torch.empty(1, Lt, heads, 128, device=DEV, dtype=torch.bfloat16)
    ref_i = torch.empty(1, Li, heads, 128, device=DEV, dtype=torch.bfloat16)
    sage_attention_split(q, k, v, Lt, ref_t, ref_i)
    # two emulated ranks, each its heads over every token, output to the owners
    img = [torch.zeros(s_loc, heads, 128, device=DEV, dtype=torch.bfloat16) for _ in range(U)]
    txt = [torch.zeros(Lt, heads, 128, device=DEV, dtype=torch.bfloat16) for _ in range(U)]
    sig = [torch.zeros(2 * U + 2, dtype=torch.int64, device=DEV) for _ in range(U)]
    it, tt = _table(img), _table(txt)
    so = torch.tensor([t.data_ptr() + 8 * U for t in sig], dtype=torch.int64, device=DEV)
    st = L.stream(qkv_t.device)
    for u in range(U):
        heads_u = lambda x: x.view(x.shape[0], 3, U, hl, 128)[:, :, u].reshape(x.shape[0], 3 * hl * 128)  # noqa: E731
        ws = sage_quantize_joint(heads_u(qkv_t)[None], heads_u(qkv_i)[None], w[0], w[1], ft, fi, hl)
        L.call("qia_sage_attn_quantized_peers", L.ptr(ws["_workspace"]), S, hl, 128, Lt, L.ptr(it), L.ptr(tt), s_loc,
               U, u * hl, heads, L.ptr(so), u, 0.0, st)
        torch.cuda.synchronize()
    assert L.device_error() == 0
    for r in range(U):
        assert torch.equal(img[r], ref_i[0, r * s_loc:(r + 1) * s_loc])
        assert torch.equal(txt[r], ref_t[0])
        ctas = L.load().qia_sage_attn_ctas(1, hl, S)
        assert sig[r][U:2 * U].tolist() == [ctas] * U

"""The allocation-free attention entry point, qia_sage_attention_noalloc.

It serves callers that cannot allocate device memory (FFI/plugin hosts without
a device allocator of their own, servers whose memory is a fixed pool owned by
another allocator, loops that must not pay cudaMalloc's device sync): the
library's built-in 16 MiB scratch replaces the caller workspace. These tests
call it through the C ABI and compare its output with qia_sage_attention (the
workspace entry point) on two calls in a row, with different sizes, so a
second call cannot pass on the first call's leftovers; and check that sizes
beyond the built-in scratch are refused with a clear message. This file is
collected last so a failing run has already run every other test.
"""
import ctypes

import pytest
import torch

pytestmark = pytest.mark.gpu
DEV = "cuda"


@pytest.fixture(autouse=True)
def _cuda():
    if not torch.cuda.is_available():
        pytest.skip("needs a CUDA device")


def strides(*ts):
    vals = []
    for t in ts:
        vals += [t.stride(0), t.stride(1), t.stride(2)]
    return (ctypes.c_int64 * len(vals))(*vals)


def noalloc(q, k, v):
    from qwen_image_accel_b200 import _lib
    lib = _lib.load()
    out = torch.empty_like(q)
    b, sq, h, d = q.shape
    rc = lib.qia_sage_attention_noalloc(_lib.ptr(q), _lib.ptr(k), _lib.ptr(v), _lib.ptr(out), b, sq, k.shape[1], h,
                                        d, strides(q, k, v, out), 0.0, _lib.stream(q.device))
    assert rc == 0, lib.qia_last_error_string()
    return out


def with_workspace(q, k, v):
    from qwen_image_accel_b200 import _lib
    from qwen_image_accel_b200.optimizations.sage_attention import workspace_bytes
    lib = _lib.load()
    out = torch.empty_like(q)
    b, sq, h, d = q.shape
    ws = torch.empty(workspace_bytes(b, h, sq, k.shape[1]), device=q.device, dtype=torch.uint8)
    rc = lib.qia_sage_attention(_lib.ptr(q), _lib.ptr(k), _lib.ptr(v), _lib.ptr(out), b, sq, k.shape[1], h, d,
                                strides(q, k, v, out), 0.0, _lib.ptr(ws), ws.numel(), _lib.stream(q.device))
    assert rc == 0, lib.qia_last_error_string()
    return out


def cosine(a, b):
    a, b = a.double().flatten(), b.double().flatten()
    return (a @ b / (a.norm() * b.norm())).item()


def qkv(b, sq, skv, h, seed):
    g = torch.Generator(device=DEV).manual_seed(seed)
    mk = lambda s: torch.randn(b, s, h, 128, device=DEV, dtype=torch.bfloat16, generator=g)  # noqa: E731
    return mk(sq), mk(skv), mk(skv)


def test_noalloc_matches_workspace_entry_point_on_two_calls():
    from qwen_image_accel_b200 import _lib
    cases = [qkv(1, 1000, 1000, 4, 11), qkv(2, 300, 777, 2, 12)]
    for q, k, v in cases:
        got = noalloc(q, k, v)
        ref = with_workspace(q, k, v)
        torch.cuda.synchronize()
        assert torch.equal(got, ref)
        assert cosine(got, ref) >= 0.999
    assert _lib.device_error() == 0


def test_noalloc_refuses_sizes_beyond_its_scratch():
    from qwen_image_accel_b200 import _lib
    lib = _lib.load()
    q, k, v = qkv(2, 4352, 4352, 24, 13)
    out = torch.empty_like(q)
    rc = lib.qia_sage_attention_noalloc(_lib.ptr(q), _lib.ptr(k), _lib.ptr(v), _lib.ptr(out), 2, 4352, 4352, 24, 128,
                                        strides(q, k, v, out), 0.0, _lib.stream(q.device))
    assert rc == 2
    assert b"built-in scratch" in lib.qia_last_error_string()

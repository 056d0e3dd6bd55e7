"""The C ABI library: it loads without a GPU, exports every declared symbol and
rejects bad arguments on the host with a status code and a message."""
import ctypes
import re
from pathlib import Path

import pytest

ROOT = Path(__file__).resolve().parents[1]
HEADER = ROOT / "include" / "qia_b200.h"


def declared():
    text = HEADER.read_text()
    return sorted(set(re.findall(r"^(?:int64_t|int|const char\*)\s+(qia_\w+)\(", text, flags=re.M)))


@pytest.fixture(scope="module")
def lib():
    import qwen_image_accel_b200._lib as L
    if not L.LIB_PATH.exists():
        import importlib.util
        spec = importlib.util.spec_from_file_location("qia_build", ROOT / "qwen-image-2.1-accel_b200" / "build.py")
        mod = importlib.util.module_from_spec(spec)
        spec.loader.exec_module(mod)
        mod.build()
    return L.load()


def test_every_declared_symbol_is_exported(lib):
    names = declared()
    assert len(names) >= 14
    for n in names:
        assert hasattr(lib, n), n


def test_python_binding_covers_header():
    import qwen_image_accel_b200._lib as L
    assert set(declared()) == set(L.declared_symbols())


def test_host_validation_returns_status(lib):
    P, I, F = ctypes.c_void_p, ctypes.c_int64, ctypes.c_float
    rc = lib.qia_ln_mod(None, None, None, None, I(1), I(512), I(1), F(1e-6), None)
    assert rc == 1 and b"null" in lib.qia_last_error_string()
    dummy = P(256)
    rc = lib.qia_ln_mod(dummy, dummy, None, dummy, I(4), I(500), I(4), F(1e-6), None)
    assert rc == 2 and b"multiple of 512" in lib.qia_last_error_string()
    rc = lib.qia_mxfp8_quantize(dummy, I(100), dummy, dummy, I(4), I(100), None)
    assert rc == 2
    rc = lib.qia_qknorm_rope_pack(dummy, dummy, dummy, None, None, dummy, dummy, dummy, dummy, dummy, dummy,
                                  I(1), I(4), I(2), I(2), I(128), F(1e-6), F(1e-6), None)
    assert rc == 1 and b"cached" in lib.qia_last_error_string()
    rc = lib.qia_gated_residual(P(258), dummy, dummy, dummy, I(2), I(8), I(2), None)
    assert rc == 3


def test_exchange_entries_reject_bad_arguments_on_the_host(lib):
    """The Ulysses exchange entries check their sizes, ranks and pointers
    before touching the device."""
    P, I, F = ctypes.c_void_p, ctypes.c_int64, ctypes.c_float
    d = P(4096)
    # heads not divisible by the Ulysses degree; rank outside the group; head_dim
    rc = lib.qia_ulysses_scatter_qkv(d, I(3 * 24 * 128), I(64), I(24), I(128), d, d, d, I(5), I(0), None)
    assert rc == 1 and b"U=5" in lib.qia_last_error_string()
    rc = lib.qia_ulysses_scatter_qkv(d, I(3 * 24 * 128), I(64), I(24), I(128), d, d, d, I(2), I(2), None)
    assert rc == 1
    rc = lib.qia_ulysses_scatter_qkv(d, I(3 * 24 * 128), I(64), I(24), I(64), d, d, d, I(2), I(0), None)
    assert rc == 2
    rc = lib.qia_ulysses_scatter_qkv(d, I(3 * 24 * 128), I(64), I(24), I(128), d, d, None, I(2), I(0), None)
    assert rc == 1 and b"null" in lib.qia_last_error_string()
    # a wait with no sources or rounds
    rc = lib.qia_ulysses_wait(d, d, I(0), I(1), I(1000), None)
    assert rc == 1
    # the peer attention: image rows that do not split evenly over the ranks, a slot outside them
    rc = lib.qia_sage_attn_quantized_peers(P(4096 * 256), I(256 + 1000), I(12), I(128), I(256), d, d, I(499), I(2),
                                           I(0), I(24), d, I(0), F(0.0), None)
    assert rc == 1 and b"rows=499" in lib.qia_last_error_string()
    rc = lib.qia_sage_attn_quantized_peers(P(4096 * 256), I(256 + 1000), I(12), I(128), I(256), d, d, I(500), I(2),
                                           I(0), I(24), d, I(2), F(0.0), None)
    assert rc == 1
    rc = lib.qia_sage_attn_quantized_peers(P(4096 * 256), I(256 + 1000), I(12), I(128), I(256), d, d, I(500), I(2),
                                           I(18), I(24), d, I(1), F(0.0), None)
    assert rc == 1 and b"heads 18+12 of 24" in lib.qia_last_error_string()

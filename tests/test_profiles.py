"""Profile registry invariants (mirrors the reference's tests/test_profiles.py)."""
import pytest

from qwen_image_accel_b200 import PROFILES, get_profile


def test_api_profile_names_present():
    for name in ("fused", "fused_sage", "mxfp8_sage", "mxfp8", "baseline", "graph"):
        assert name in PROFILES


def test_flags():
    assert get_profile("mxfp8_sage").quantized and get_profile("mxfp8_sage").sage
    assert get_profile("fused_sage").sage and not get_profile("fused_sage").quantized
    assert get_profile("fused").fused and not get_profile("fused").sage


def test_retired_and_unknown_profiles_raise():
    with pytest.raises(ValueError, match="retired"):
        get_profile("fp8_sage")
    with pytest.raises(ValueError, match="Unknown"):
        get_profile("nope")


def test_import_does_not_load_library():
    import qwen_image_accel_b200._lib as L
    import importlib
    assert importlib.import_module("qwen_image_accel_b200").PROFILES is PROFILES
    assert L.LIB_PATH.name == "libqia_b200.so"

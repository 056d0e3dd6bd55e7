"""The pinned Diffusers wheel as a checker and CPU baseline -- TEST
INFRASTRUCTURE, never the product.

The reference pins diffusers 0.41.0.dev0 as a wheel (third_party/wheels/
diffusers-0.41.0.dev0-py3-none-any.whl, sha256 in third_party/manifest.json:
3-18). `python -m pip install --no-index --no-deps --target baseline/_ref
<that wheel>` puts it under baseline/_ref/ (git-ignored; shipped to the GPU box
with the tree). This module imports it from there, after giving the installed
huggingface_hub the three attributes the wheel imports but hub 1.14 lacks
(`resolve_revision`, `errors.RevisionResolutionError`, `utils.httpx`; the
wheel never calls them on these paths).

Only tests/ and bench.py's reference arm import this module.
"""
from __future__ import annotations

import sys
import types
from pathlib import Path

REF = Path(__file__).resolve().parents[1] / "baseline" / "_ref"


def available() -> bool:
    return (REF / "diffusers" / "__init__.py").exists()


def load():
    """Import and return the pinned `diffusers` package (raises when missing)."""
    if not available():
        raise RuntimeError(f"{REF} holds no diffusers: install the reference's pinned wheel there")
    if str(REF) not in sys.path:
        sys.path.insert(0, str(REF))
    import huggingface_hub
    import huggingface_hub.errors
    import huggingface_hub.utils
    for mod, name, val in [(huggingface_hub, "resolve_revision", lambda *a, **k: None),
                           (huggingface_hub.errors, "RevisionResolutionError",
                            type("RevisionResolutionError", (Exception,), {})),
                           (huggingface_hub.utils, "httpx", types.SimpleNamespace())]:
        if not hasattr(mod, name):
            setattr(mod, name, val)
    import diffusers
    if not str(Path(diffusers.__file__)).startswith(str(REF)):
        raise RuntimeError(f"diffusers was imported from {diffusers.__file__}, not the pinned copy under {REF}")
    return diffusers


def qwen21():
    """The Qwen-Image 2.1 transformer module of the pinned wheel."""
    load()
    from diffusers.models.transformers import transformer_qwenimage21
    return transformer_qwenimage21


def qwen_v1():
    """The Qwen-Image (v1) MMDiT transformer module of the pinned wheel."""
    load()
    from diffusers.models.transformers import transformer_qwenimage
    return transformer_qwenimage

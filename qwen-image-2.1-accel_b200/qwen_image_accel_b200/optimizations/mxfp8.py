"""Block-scaled MXFP8 linears on the tcgen05 GEMM.

Mirrors src/qwen_image_accel/optimizations/mxfp8.py: MXFP8Linear (weight
stored as E4M3 + swizzled E8M0, `.matmul(activation)` on an already-quantized
activation, `.forward(x)`), LAYER_GROUPS, selected_layers and
quantize_transformer. Extensions for the dual-stream (v1) block: linears with
a bias, and the fused epilogues of qia_mxfp8_gemm_* (GELU-tanh, GELU-tanh +
MXFP8 requantization, gate + residual).
"""
from __future__ import annotations

import ctypes
import os

import torch
from torch import nn

from .. import _lib
from ..kernels.mxfp8 import Quantized, empty_quantized, quantize


def _supported(k, n):
    return k % 128 == 0 and n % 128 == 0


class MXFP8Linear(nn.Module):
    """Linear whose weight is stored as MXFP8 and multiplied as MXFP8."""

    def __init__(self, linear: nn.Linear):
        super().__init__()
        self.in_features, self.out_features = linear.in_features, linear.out_features
        if not _supported(self.in_features, self.out_features):
            raise ValueError("MXFP8Linear needs in/out features that are multiples of 128")
        weight = linear.weight.detach().to(torch.bfloat16).contiguous()
        q = quantize(weight)
        self.register_buffer("weight_fp8", q.values.t())     # (K, N) column-major, as in the reference
        self.register_buffer("weight_scale", q.scales)
        b = linear.bias
        self.register_buffer("bias", None if b is None else b.detach().to(torch.bfloat16).contiguous())

    @classmethod
    def from_parts(cls, values: torch.Tensor, scales: torch.Tensor, bias: torch.Tensor | None = None):
        """An MXFP8Linear over already quantized weights: values E4M3 [N, K]
        row-major, scales the E8M0 128x4 layout of N rows (no copy)."""
        self = cls.__new__(cls)
        nn.Module.__init__(self)
        self.out_features, self.in_features = values.shape
        if not _supported(self.in_features, self.out_features):
            raise ValueError("MXFP8Linear needs in/out features that are multiples of 128")
        if scales.numel() != values.numel() // 32:
            raise ValueError("scales must hold one E8M0 per 32 weights")
        self.register_buffer("weight_fp8", values.t())
        self.register_buffer("weight_scale", scales)
        self.register_buffer("bias", bias)
        return self

    # the [N, K] row-major view the kernels consume
    def _w(self):
        return self.weight_fp8.t()

    def _args(self, activation: Quantized):
        if activation.values.shape[1] != self.in_features:
            raise ValueError(f"activation K={activation.values.shape[1]} != in_features={self.in_features}")
        w = self._w()
        return (_lib.ptr(activation.values), _lib.ptr(activation.scales), _lib.ptr(w), _lib.ptr(self.weight_scale),
                _lib.ptr(self.bias))

    def matmul(self, activation: Quantized, dtype=torch.bfloat16, out: torch.Tensor | None = None) -> torch.Tensor:
        """bf16 (rows, N) = activation @ W^T (+ bias); several weights can share one activation."""
        if dtype != torch.bfloat16:
            raise NotImplementedError("MXFP8Linear.matmul produces bf16")
        m, n = activation.rows, self.out_features
        if out is None:
            out = torch.empty((m, n), device=activation.values.device, dtype=torch.bfloat16)
        _lib.call("qia_mxfp8_gemm", *self._args(activation), _lib.ptr(out), m, n, self.in_features, out.stride(0),
                  _lib.stream(out.device))
        return out

    def matmul_gelu(self, activation: Quantized) -> torch.Tensor:
        """bf16 gelu_tanh(activation @ W^T + bias)."""
        m, n = activation.rows, self.out_features
        out = torch.empty((m, n), device=activation.values.device, dtype=torch.bfloat16)
        _lib.call("qia_mxfp8_gemm_gelu", *self._args(activation), _lib.ptr(out), m, n, self.in_features, n,
                  _lib.stream(out.device))
        return out

    def matmul_gelu_quantize(self, activation: Quantized) -> Quantized:
        """gelu_tanh(activation @ W^T + bias) quantized to MXFP8 in the GEMM epilogue."""
        m, n = activation.rows, self.out_features
        q = empty_quantized(m, n, activation.values.device)
        _lib.call("qia_mxfp8_gemm_gelu_quant", *self._args(activation), _lib.ptr(q.values), _lib.ptr(q.scales), m, n,
                  self.in_features, _lib.stream(q.values.device))
        return q

    def matmul_swiglu_quantize(self, activation: Quantized) -> Quantized:
        """MXFP8 SwiGLU activation bf16(silu(g) * v) of the gate/value pair
        this linear stacks (interleaved_gate_value), quantized in the GEMM
        epilogue: [rows, out_features / 2]."""
        if self.bias is not None:
            raise NotImplementedError("the SwiGLU epilogue takes no bias")
        m, n = activation.rows, self.out_features
        q = empty_quantized(m, n // 2, activation.values.device)
        _lib.call("qia_mxfp8_gemm_swiglu_quant", *self._args(activation)[:4], _lib.ptr(q.values), _lib.ptr(q.scales),
                  m, n, self.in_features, _lib.stream(q.values.device))
        return q

    def matmul_gate_residual(self, activation: Quantized, gate: torch.Tensor, residual: torch.Tensor,
                             out: torch.Tensor | None = None) -> torch.Tensor:
        """residual + gate * (activation @ W^T + bias), each step rounded to bf16.

        residual/out: (B, S, N) or (B*S, N) bf16; gate: (B, 1, N) or (B, N).
        out may be residual itself (in-place update)."""
        m, n = activation.rows, self.out_features
        res2 = residual.reshape(-1, n)
        if res2.shape[0] != m or not res2.is_contiguous():
            raise ValueError("residual must be contiguous with the activation's rows")
        rows_per_batch = m // gate.reshape(-1, n).shape[0]
        if out is None:
            out = torch.empty_like(residual)
        _lib.call("qia_mxfp8_gemm_gate_residual", *self._args(activation), _lib.ptr(gate), _lib.ptr(res2),
                  _lib.ptr(out), m, n, self.in_features, n, rows_per_batch, _lib.stream(out.device))
        return out

    def forward(self, x: torch.Tensor) -> torch.Tensor:
        flat = x.reshape(-1, x.shape[-1])
        activation = quantize(flat if flat.stride(-1) == 1 else flat.contiguous())
        return self.matmul(activation, x.dtype).reshape(*x.shape[:-1], self.out_features)


def interleaved_gate_value(gate_weight: torch.Tensor, value_weight: torch.Tensor) -> torch.Tensor:
    """[2F, K] stack of the SwiGLU gate and value weights ([F, K] each),
    interleaved every 32 rows -- the B operand of matmul_swiglu_quantize."""
    f, k = gate_weight.shape
    if value_weight.shape != (f, k) or f % 32:
        raise ValueError("gate and value weights must be [F, K] with F a multiple of 32")
    return torch.stack([gate_weight.reshape(f // 32, 32, k), value_weight.reshape(f // 32, 32, k)], dim=1).reshape(2 * f, k)


def _grouped(epilogue: int, problems: list) -> None:
    """One qia_mxfp8_gemm_grouped launch over one or two (linear, activation,
    fields) problems sharing N, K and the epilogue."""
    lins = [p[0] for p in problems]
    n, k = lins[0].out_features, lins[0].in_features
    if any(l.out_features != n or l.in_features != k for l in lins):
        raise ValueError("grouped GEMMs must share N and K")
    arr = (_lib.GemmProblem * len(problems))()
    for slot, (lin, act, fields) in zip(arr, problems):
        a_v, a_s, b_v, b_s, bias = lin._args(act)
        slot.a_values, slot.a_scales, slot.b_values, slot.b_scales, slot.bias = a_v, a_s, b_v, b_s, bias
        slot.m = act.rows
        for name, value in fields.items():
            setattr(slot, name, value)
    device = problems[0][1].values.device
    _lib.call("qia_mxfp8_gemm_grouped", epilogue, ctypes.addressof(arr), len(problems), n, k, _lib.stream(device))


def matmul_grouped(pairs) -> list:
    """[(linear, activation), ...] (one or two, same N and K) -> their bf16
    matmuls (+ bias) in one launch."""
    outs, problems = [], []
    for lin, act in pairs:
        out = torch.empty((act.rows, lin.out_features), device=act.values.device, dtype=torch.bfloat16)
        outs.append(out)
        problems.append((lin, act, {"out": _lib.ptr(out), "ldo": out.stride(0)}))
    _grouped(_lib.EPI_BF16, problems)
    return outs


def matmul_gelu_quantize_grouped(pairs) -> list:
    """[(linear, activation), ...] -> MXFP8 gelu_tanh(activation @ W^T + bias)
    per problem, in one launch."""
    outs, problems = [], []
    for lin, act in pairs:
        q = empty_quantized(act.rows, lin.out_features, act.values.device)
        outs.append(q)
        problems.append((lin, act, {"q_values": _lib.ptr(q.values), "q_scales": _lib.ptr(q.scales)}))
    _grouped(_lib.EPI_GELU_QUANT, problems)
    return outs


def matmul_gate_residual_grouped(items) -> None:
    """[(linear, activation, gate, residual), ...]: residual += gate * (activation
    @ W^T + bias) in place for each, in one launch (the rules of
    MXFP8Linear.matmul_gate_residual)."""
    problems = []
    for lin, act, gate, residual in items:
        n = lin.out_features
        res2 = residual.reshape(-1, n)
        if res2.shape[0] != act.rows or not res2.is_contiguous():
            raise ValueError("residual must be contiguous with the activation's rows")
        rows_per_batch = act.rows // gate.reshape(-1, n).shape[0]
        problems.append((lin, act, {"gate": _lib.ptr(gate), "resid": _lib.ptr(res2), "out": _lib.ptr(res2),
                                    "ldo": n, "rows_per_batch": rows_per_batch}))
    _grouped(_lib.EPI_GATE_RESIDUAL, problems)


# The linears a layer selection names, per group, over both block layouts this
# package serves (the 2.1 single-stream block and the v1 dual-stream block); a
# name a block does not have is passed over. The group and environment names
# are the reference's interface (src/qwen_image_accel/optimizations/mxfp8.py:
# 46-50); the v1 names are additions.
_ATTENTION_LINEARS = ("attn.to_q", "attn.to_k", "attn.to_v", "attn.to_out.0",
                      "attn.add_q_proj", "attn.add_k_proj", "attn.add_v_proj", "attn.to_add_out")
_MLP_LINEARS = ("img_mlp.gate_layer", "img_mlp.proj", "img_mlp.out",
                "img_mlp.net.0.proj", "img_mlp.net.2", "txt_mlp.net.0.proj", "txt_mlp.net.2")
LAYER_GROUPS = {"attention": _ATTENTION_LINEARS, "mlp": _MLP_LINEARS, "all": _ATTENTION_LINEARS + _MLP_LINEARS}


def selected_layers(selection: str | None = None) -> set:
    """The linear names a selection converts. `selection` (default: the
    QW21_MXFP8_LAYERS environment variable, else "all") is a group name of
    LAYER_GROUPS or a comma-separated list of linear names; an unknown name is
    a ValueError."""
    spec = (os.environ.get("QW21_MXFP8_LAYERS", "all") if selection is None else selection).strip()
    if spec in LAYER_GROUPS:
        return set(LAYER_GROUPS[spec])
    chosen = {part.strip() for part in spec.split(",")} - {""}
    unknown = chosen.difference(LAYER_GROUPS["all"])
    if unknown:
        raise ValueError(f"QW21_MXFP8_LAYERS: {sorted(unknown)} are not block linears; give a group "
                         f"({', '.join(LAYER_GROUPS)}) or names from {sorted(LAYER_GROUPS['all'])}")
    return chosen


def skip_block_indices(skip_blocks=None, profile_default: str | None = None) -> set:
    """Block indices that keep every linear in bf16: `skip_blocks` (a
    comma-separated string or an iterable of ints), else the
    QW21_MXFP8_SKIP_BLOCKS environment variable, else the profile's own list
    (`profile_default`, e.g. the balanced profiles' "0,1,2,29,30,31"), else
    "0,31" -- the reference's default (src/qwen_image_accel/pipeline.py:133),
    taken literally whatever the depth of the stack."""
    if skip_blocks is None:
        skip_blocks = os.environ.get("QW21_MXFP8_SKIP_BLOCKS", profile_default or "0,31")
    if isinstance(skip_blocks, str):
        return {int(tok) for tok in skip_blocks.split(",") if tok.strip()}
    return {int(i) for i in skip_blocks}


def _owner(module: nn.Module, dotted: str):
    """(parent module, attribute name) of a dotted child path, or None."""
    parent_path, _, leaf = dotted.rpartition(".")
    try:
        parent = module.get_submodule(parent_path) if parent_path else module
    except AttributeError:
        return None
    return (parent, leaf) if isinstance(getattr(parent, leaf, None), nn.Module) else None


def quantize_transformer(transformer, skip_blocks=None, layers=None) -> list:
    """Swap the selected bf16 linears of every block outside skip_blocks for
    MXFP8Linear (weights quantized once, here); norms, modulation,
    embeddings, the output projection and every non-block module stay as
    they are. Returns the converted modules' names
    ("transformer_blocks.<i>.<linear>")."""
    keep_bf16 = skip_block_indices(skip_blocks)
    names = sorted(selected_layers(layers))
    converted = []
    with torch.no_grad():
        for index, block in enumerate(transformer.transformer_blocks):
            if index in keep_bf16:
                continue
            for name in names:
                found = _owner(block, name)
                if found is None:
                    continue
                parent, leaf = found
                lin = getattr(parent, leaf)
                if type(lin) is not nn.Linear or not _supported(lin.in_features, lin.out_features):
                    continue
                setattr(parent, leaf, MXFP8Linear(lin))
                converted.append(f"transformer_blocks.{index}.{name}")
    return converted


def stack_linears(linears) -> nn.Module:
    """One linear whose output rows are those of `linears` in order (all
    MXFP8Linear or all bias-free bf16 nn.Linear, same in_features), whose
    storage the given modules then share: each of them is left holding views
    into the stacked weight, so nothing is duplicated and each still computes
    its own rows. (MXFP8 scales stack by concatenation: the 128x4 layout
    orders whole 128-row tiles, and every out_features is a multiple of 128.)"""
    linears = list(linears)
    k = linears[0].in_features
    if any(l.in_features != k for l in linears):
        raise ValueError("stacked linears must share in_features")
    if all(isinstance(l, MXFP8Linear) for l in linears):
        values = torch.cat([l._w() for l in linears])
        scales = torch.cat([l.weight_scale for l in linears])
        has_bias = [l.bias is not None for l in linears]
        if any(has_bias) and not all(has_bias):
            raise ValueError("stacked MXFP8 linears must all have a bias or none")
        bias = torch.cat([l.bias for l in linears]) if all(has_bias) else None
        stacked = MXFP8Linear.from_parts(values, scales, bias)
        r = c = 0
        for l in linears:
            n, ns = l.out_features, l.weight_scale.numel()
            l.weight_fp8 = values[r:r + n].t()
            l.weight_scale = scales[c:c + ns]
            if bias is not None:
                l.bias = bias[r:r + n]
            r, c = r + n, c + ns
        return stacked
    if all(type(l) is nn.Linear and l.bias is None for l in linears):
        weight = torch.cat([l.weight.detach() for l in linears])
        stacked = nn.Linear(k, weight.shape[0], bias=False, device=weight.device, dtype=weight.dtype)
        stacked.weight = nn.Parameter(weight, requires_grad=False)
        r = 0
        for l in linears:
            n = l.out_features
            l.weight = nn.Parameter(weight[r:r + n], requires_grad=False)
            r += n
        return stacked
    raise ValueError("stack_linears takes all-MXFP8 or all bias-free bf16 linears")

"""The whole Qwen-Image 2.1 transformer around Block21, with the prefix KV cache modes.

Mirrors QwenImage21Transformer2DModel.forward (WHL:diffusers/models/
transformers/transformer_qwenimage21.py:847-1018) for causal_condition=True:
the vision-language slot layout (every image slot of `img_mask` stands for 2x2
latent tokens; condition-image and target latents replace those positions of
the text stream), the 3-axis RoPE table (QwenImage21Rope, :652-710), the token
metadata (build_token_metadata, :808-844), the timestep embedder
(QwenImage21TimestepProjEmbeddings, :136-167), the text projection
(QwenImage21TextProjection, :170-200), the shared modulation, the blocks
(qwen21.Block21) and the scale-only output norm (:215-236). kv_cache_mode
"extract" runs the prefill and fills the cache, "cached" decodes the target
tokens from it, None runs the prefill without a cache.

The embedders, the RoPE table and the metadata are prompt-sized torch glue in
the reference's own ops; the per-token work is in the blocks.
"""
from __future__ import annotations

import ctypes
import math

import torch
import torch.nn.functional as F

from . import _lib
from .kernels.layernorm import layer_norm_scale
from .optimizations.mxfp8 import skip_block_indices
from .profiles import get_profile
from .qwen21 import Block21, Block21Config, KVCache, _Norm, block21_parameter_shapes, modulation_values


def model21_parameter_shapes(num_layers: int, cfg: Block21Config, context_in_dim: int, in_channels: int = 64,
                             out_channels: int = 64) -> dict[str, tuple]:
    """Diffusers state-dict names and shapes of QwenImage21Transformer2DModel
    (patch_size 1; no biases)."""
    d = cfg.dim
    shapes = {
        "img_in.weight": (d, in_channels), "modulation.1.weight": (4 * d, d),
        "norm_out.linear.weight": (d, d), "proj_out.weight": (out_channels, d),
        "time_text_embed.timestep_embedder.linear_1.weight": (d, 256),
        "time_text_embed.timestep_embedder.linear_2.weight": (d, d),
        "txt_in.text_norm.weight": (context_in_dim,), "txt_in.in_layer.weight": (d, context_in_dim),
        "txt_in.out_layer.weight": (d, d),
    }
    for i in range(num_layers):
        for n, shp in block21_parameter_shapes(cfg).items():
            shapes[f"transformer_blocks.{i}.{n}"] = shp
    return shapes


def token_metadata(image_pad_mask: torch.Tensor, img_shapes) -> tuple[torch.Tensor, torch.Tensor]:
    """image_ids (-1 at text tokens, one id per image block, blocks taken from
    the token counts of img_shapes) and the target image's token mask
    (build_token_metadata, transformer_qwenimage21.py:808-844)."""
    positions = image_pad_mask.nonzero(as_tuple=True)[0]
    lengths = [math.prod(shape) for shape in img_shapes]
    if sum(lengths) != positions.numel():
        raise ValueError(f"img_shapes accounts for {sum(lengths)} image tokens but image_pad_mask marks "
                         f"{positions.numel()}.")
    image_ids = torch.full_like(image_pad_mask, -1, dtype=torch.long)
    image_ids[positions] = torch.repeat_interleave(torch.arange(len(lengths), device=image_pad_mask.device),
                                                   torch.tensor(lengths, device=image_pad_mask.device))
    target = torch.zeros_like(image_pad_mask)
    target[positions[-lengths[-1]:]] = True
    return image_ids, target


_ROPE_CACHE: dict = {}


def _axis_table(dim: int, theta: int) -> torch.Tensor:
    """complex64 [8192 + 1024, dim/2]: positions 0..8191, then -1024..-1, so a
    negative position indexes from the end (QwenImage21Rope.__init__)."""
    key = (dim, theta)
    if key not in _ROPE_CACHE:
        index = torch.cat([torch.arange(8192), torch.arange(1024).flip(0) * -1 - 1])
        inv = 1.0 / torch.pow(theta, torch.arange(0, dim, 2).to(torch.float32).div(dim))
        ang = torch.outer(index, inv)
        _ROPE_CACHE[key] = torch.polar(torch.ones_like(ang), ang)
    return _ROPE_CACHE[key]


def rope_table(img_shapes, image_pad_mask: torch.Tensor, axes_dim=(16, 56, 56), theta: int = 10000) -> torch.Tensor:
    """complex64 [S, sum(axes_dim)/2] RoPE table of the joint sequence, on the
    CPU (QwenImage21Rope.forward, :677-710): text tokens advance one shared
    position on all three axes; an image block freezes the frame axis at the
    position the preceding text reached and lays its tokens out on a
    height/width grid centred on zero, then advances the position by
    max(height, width)."""
    is_image = image_pad_mask.cpu().tolist()
    total = len(is_image)
    frame, img_h, img_w = [], [], []
    cursor, position = 0, 0
    for _, height, width in img_shapes:
        start = is_image.index(True, cursor)
        frame.extend(range(position, position + start - cursor))
        position += start - cursor
        cursor = start + height * width
        frame.extend([position] * (height * width))
        position += max(height, width)
        img_h.extend(h for h in range(-(height - height // 2), height // 2) for _ in range(width))
        img_w.extend(w for _ in range(height) for w in range(-(width - width // 2), width // 2))
    if cursor < total:
        frame.extend(range(position, position + total - cursor))
    frame_index = torch.tensor(frame, dtype=torch.long)
    mask = image_pad_mask.cpu()
    h_index, w_index = frame_index.clone(), frame_index.clone()
    h_index[mask] = torch.tensor(img_h, dtype=torch.long)
    w_index[mask] = torch.tensor(img_w, dtype=torch.long)
    tabs = [_axis_table(d, theta) for d in axes_dim]
    return torch.cat([tabs[0][frame_index], tabs[1][h_index], tabs[2][w_index]], dim=-1)


_DEVICE_AXES: dict = {}


def rope_table_device(img_shapes, image_pad_mask: torch.Tensor, axes_dim=(16, 56, 56),
                      theta: int = 10000) -> torch.Tensor:
    """rope_table built on the device (qia_rope21_table): the same integer
    positions, taken with prefix sums over the image mask instead of the
    reference's host loop, and the same per-axis complex64 rows gathered --
    bit-identical to rope_table. image_pad_mask: bool [S] on the GPU; the
    result is complex64 [S, sum(axes_dim)/2] on the same device."""
    dev = image_pad_mask.device
    _lib.require_cuda(image_pad_mask)
    key = (tuple(axes_dim), theta, str(dev))
    tabs = _DEVICE_AXES.get(key)
    if tabs is None:
        tabs = _DEVICE_AXES[key] = [torch.view_as_real(_axis_table(d, theta)).to(dev).contiguous()
                                    for d in axes_dim]
    hw = (ctypes.c_int32 * (2 * max(1, len(img_shapes))))()
    for i, (_, h, w) in enumerate(img_shapes):
        hw[2 * i], hw[2 * i + 1] = int(h), int(w)
    mask = image_pad_mask.to(torch.uint8).contiguous()
    s = mask.shape[0]
    out = torch.empty(s, sum(axes_dim) // 2, 2, device=dev, dtype=torch.float32)
    _lib.call("qia_rope21_table", _lib.ptr(mask), s, ctypes.cast(hw, ctypes.c_void_p), len(img_shapes),
              _lib.ptr(tabs[0]), _lib.ptr(tabs[1]), _lib.ptr(tabs[2]), axes_dim[0] // 2, axes_dim[1] // 2,
              axes_dim[2] // 2, 8192, 1024, _lib.ptr(out), _lib.stream(dev))
    return torch.view_as_complex(out)


class Qwen21Transformer:
    """QwenImage21Transformer2DModel on the sm_100a kernels (causal_condition,
    patch size 1). params: name -> tensor mapping or callable with the
    Diffusers names of model21_parameter_shapes."""

    def __init__(self, params, num_layers: int = 32, cfg: Block21Config = Block21Config(),
                 context_in_dim: int = 4096, device="cuda", profile: str = "mxfp8_sage", sage_prefill: bool = False,
                 axes_dims_rope=(16, 56, 56), skip_blocks=None):
        get = params if callable(params) else params.__getitem__
        dev = torch.device(device)
        prof = get_profile(profile)
        # blocks that keep bf16 linears in the MXFP8 profiles (default: the
        # QW21_MXFP8_SKIP_BLOCKS environment variable, else the profile's list,
        # else "0,31", as configure_pipeline / quantize_transformer)
        self.skip_blocks = skip_block_indices(skip_blocks, prof.skip_blocks) if prof.quantized else set()
        self.cfg, self.axes = cfg, tuple(axes_dims_rope)
        w = lambda n: get(n).to(dev, torch.bfloat16).contiguous()
        self.w = {n: w(n) for n in ("img_in.weight", "modulation.1.weight", "norm_out.linear.weight",
                                    "proj_out.weight", "time_text_embed.timestep_embedder.linear_1.weight",
                                    "time_text_embed.timestep_embedder.linear_2.weight", "txt_in.text_norm.weight",
                                    "txt_in.in_layer.weight", "txt_in.out_layer.weight")}
        self.blocks = [Block21(lambda n, i=i: get(f"transformer_blocks.{i}.{n}"), cfg, device=dev, profile=profile,
                               sage_prefill=sage_prefill, quantized=prof.quantized and i not in self.skip_blocks)
                       for i in range(num_layers)]
        self.ln = _Norm(None, cfg.eps, (cfg.dim,))
        self._layouts: dict = {}
        # QwenImage21TemporalTimesteps(256): frequencies built once in fp32 on the CPU
        self.t_freqs = torch.exp(-math.log(10000) * torch.arange(0, 128, dtype=torch.float32) / 128).to(dev)

    # ---------------------------------------------------------------- embedders
    def time_embed(self, t: torch.Tensor) -> torch.Tensor:
        """QwenImage21TimestepProjEmbeddings: [cos | sin](1000 t * freqs) in
        fp32 -> bf16 -> linear_1 -> SiLU -> linear_2 (no biases)."""
        args = (1000.0 * t.float())[:, None] * self.t_freqs[None]
        e = torch.cat([torch.cos(args), torch.sin(args)], dim=-1).to(torch.bfloat16)
        e = F.silu(F.linear(e, self.w["time_text_embed.timestep_embedder.linear_1.weight"]))
        return F.linear(e, self.w["time_text_embed.timestep_embedder.linear_2.weight"])

    def text_projection(self, x: torch.Tensor) -> torch.Tensor:
        """QwenImage21TextProjection: zero-centred RMSNorm (fp32, weight + 1)
        -> Linear -> GELU-tanh -> Linear."""
        xf = x.float()
        rrms = torch.rsqrt(torch.mean(xf ** 2, dim=-1, keepdim=True) + self.cfg.eps)
        y = (xf * rrms * (self.w["txt_in.text_norm.weight"].float() + 1)).to(x.dtype)
        y = F.gelu(F.linear(y, self.w["txt_in.in_layer.weight"]), approximate="tanh")
        return F.linear(y, self.w["txt_in.out_layer.weight"])

    def layout(self, img_shapes, img_mask: torch.Tensor, device) -> dict:
        """The layout-only tensors of a forward -- per-slot repeats, the image
        token mask, the RoPE table, the token metadata and the prefix length
        -- memoised per (image shapes, slot mask): every denoising step of a
        generation shares them, and the reference rebuilds them each forward
        (the RoPE table alone is a host loop over the sequence). The key reads
        the slot mask on the host, where the reference's RoPE already syncs."""
        key = (tuple(tuple(int(v) for v in s) for s in img_shapes[0]), bytes(img_mask[0].cpu().numpy().tobytes()),
               str(device))
        hit = self._layouts.get(key)
        if hit is not None:
            return hit
        repeats = torch.where(img_mask, 4, 1)[0]
        image_pad_mask = torch.repeat_interleave(img_mask[0], repeats)
        image_ids, target = token_metadata(image_pad_mask.to(device), img_shapes[0])
        lay = {"repeats": repeats.to(device), "pad": image_pad_mask.to(device), "pad_cpu": image_pad_mask.cpu(),
               "rope": rope_table_device(img_shapes[0], image_pad_mask.to(device), self.axes), "image_ids": image_ids,
               "target": target, "prefix_len": int((~target).sum())}
        if len(self._layouts) >= 8:
            self._layouts.pop(next(iter(self._layouts)))
        self._layouts[key] = lay
        return lay

    # ---------------------------------------------------------------- forward
    def forward(self, hidden_states: torch.Tensor, encoder_hidden_states: torch.Tensor, timestep: torch.Tensor,
                img_shapes, img_mask: torch.Tensor, encoder_hidden_states_mask: torch.Tensor | None = None,
                kv_cache: KVCache | None = None, kv_cache_mode: str | None = None) -> torch.Tensor:
        """Same arguments and result as QwenImage21Transformer2DModel.forward
        (return_dict=False, first element): the prefill returns the whole
        joint sequence's output, the cached decode the target tokens'."""
        _lib.require_cuda(hidden_states, encoder_hidden_states)
        if kv_cache is not None and kv_cache_mode not in ("extract", "cached"):
            raise ValueError(f"kv_cache_mode must be 'extract' or 'cached' when kv_cache is provided, "
                             f"got {kv_cache_mode!r}.")
        if kv_cache is None and kv_cache_mode is not None:
            raise ValueError(f"kv_cache_mode is {kv_cache_mode!r} but no kv_cache was passed to hold the prefix.")
        dev = hidden_states.device
        b = hidden_states.shape[0]
        x = F.linear(hidden_states, self.w["img_in.weight"])
        c = self.text_projection(encoder_hidden_states)
        # every image slot stands for 2x2 latent tokens; samples share a layout
        lay = self.layout(img_shapes, img_mask, dev)
        image_pad_mask, rope, image_ids = lay["pad"], lay["rope"], lay["image_ids"]
        target_tokens = math.prod(img_shapes[0][-1])
        joint = torch.cat([c, c.new_zeros(b, target_tokens // 4, c.shape[2])], dim=1)
        joint = joint.repeat_interleave(lay["repeats"], dim=1)
        joint[:, image_pad_mask] = x
        t = timestep.to(torch.bfloat16)
        temb = self.time_embed(torch.cat([t, t.new_zeros(1)]))          # [sampled rows, t = 0]
        modulation = F.linear(F.silu(temb), self.w["modulation.1.weight"])
        key_valid = None
        if encoder_hidden_states_mask is not None:
            key_valid = torch.ones(b, image_pad_mask.shape[0], dtype=torch.bool, device=dev)
            text_pos = (~lay["pad_cpu"]).nonzero(as_tuple=True)[0].to(dev)
            vlm_text = ~img_mask[0][: encoder_hidden_states_mask.shape[1]]
            key_valid[:, text_pos] = encoder_hidden_states_mask.bool()[:, vlm_text.to(encoder_hidden_states_mask.device)].to(dev)
        prefix_len = lay["prefix_len"]
        scale = F.linear(F.silu(temb), self.w["norm_out.linear.weight"])   # [B + 1, D]
        if kv_cache_mode == "cached":
            h = joint[:, prefix_len:].contiguous()
            vals = modulation_values(modulation)
            freqs = rope[prefix_len:].contiguous()
            for i, blk in enumerate(self.blocks):
                h = blk.forward_cached(h, vals, freqs, kv_cache.get_layer(i), key_valid=key_valid)
            y = layer_norm_scale(h, (1 + scale[:-1])[:, None].contiguous(), self.ln)
        else:
            h = joint.contiguous()
            for i, blk in enumerate(self.blocks):
                cache = kv_cache.get_layer(i) if kv_cache_mode == "extract" else None
                h = blk.forward_prefill(h, modulation, rope, image_ids, prefix_len, layer_cache=cache,
                                        key_valid=key_valid)
            # prefix rows scale from the t = 0 row, target rows from their sample's row
            y = self.blocks[0]._rows("ln", h, (1 + scale).contiguous(), prefix_len)
        return F.linear(y, self.w["proj_out.weight"])

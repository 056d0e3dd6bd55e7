"""CUDA-graph replay of a whole decode step (the `graph` profile).

Same name and contract as the reference's `install_cuda_graph(transformer,
max_graphs=1)` (src/qwen_image_accel/optimizations/cuda_graph.py:14-87): on a
Diffusers Qwen-Image 2.1 transformer whose decode is routed to the kernels
(install_fused_decode / install_mx_fused_decode), the cached-decode pass over
all blocks becomes one CUDA graph replay; the prefill stays eager.

Mechanics: block 0's forward, in cached mode, replays a graph of every
block's Block21.forward_cached and returns the last block's output; the other
blocks pass their input through in cached mode. A graph is keyed by the
shapes of the step's inputs and the prefix cache; up to `max_graphs` stay
resident (least recently used dropped). Each graph owns static copies of its
inputs: the target hidden states, the modulation and the RoPE rows and
padding mask are copied in before every replay; the per-layer prefix K/V are
copied in whenever a different KV cache object (a new request) arrives. The
modulation vectors are computed inside the graph, so each replay sees the new
timestep. The returned tensor is the graph's static output: it is overwritten
by the next replay. Serial use only (one request at a time), as for the
reference.
"""
from __future__ import annotations

from collections import OrderedDict

import torch

from ..qwen21 import KVLayerCache, modulation_values
from .decode import _key_valid, bound_blocks


class _StepGraph:
    def __init__(self, blocks, h, modulation, rope, mask, kv_cache):
        self.blocks = blocks
        self.h, self.mod, self.rope = h.clone(), modulation.clone(), rope.clone()
        self.mask = None if mask is None else mask.clone()
        self.caches = []
        for layer in kv_cache.layer_caches:
            c = KVLayerCache()
            c.store(layer.k.clone(), layer.v.clone())
            self.caches.append(c)
        self.source = kv_cache
        side = torch.cuda.Stream()
        side.wait_stream(torch.cuda.current_stream())
        with torch.cuda.stream(side):
            for _ in range(2):           # warm-up: allocator pools, kernel attributes, workspaces
                self._body()
        torch.cuda.current_stream().wait_stream(side)
        torch.cuda.synchronize()
        self.graph = torch.cuda.CUDAGraph()
        with torch.cuda.graph(self.graph):
            self.out = self._body()

    def _body(self):
        values = modulation_values(self.mod)
        key_valid = _key_valid(self.mask)
        x = self.h
        for blk, cache in zip(self.blocks, self.caches):
            x = blk.forward_cached(x, values, self.rope, cache, key_valid=key_valid)
        return x

    def run(self, h, modulation, rope, mask, kv_cache):
        self.h.copy_(h)
        self.mod.copy_(modulation)
        self.rope.copy_(rope)
        if mask is not None:
            self.mask.copy_(mask)
        if kv_cache is not self.source:
            for dst, src in zip(self.caches, kv_cache.layer_caches):
                dst.k.copy_(src.k)
                dst.v.copy_(src.v)
            self.source = kv_cache
        self.graph.replay()
        return self.out


def install_cuda_graph(transformer, max_graphs: int = 1) -> None:
    """Replay the decode blocks of `transformer` from CUDA graphs (see the
    module docstring). Needs install_fused_decode or install_mx_fused_decode
    first."""
    blocks = bound_blocks(transformer)
    graphs: OrderedDict = OrderedDict()
    transformer._qw_graphs = graphs
    step = {}

    def remember_cache(module, args, kwargs):
        step["kv_cache"] = kwargs.get("kv_cache")

    transformer.register_forward_pre_hook(remember_cache, with_kwargs=True)
    routed = [b.forward for b in transformer.transformer_blocks]

    def first(*args, **kwargs):
        if kwargs.get("kv_cache_mode") != "cached" or args:
            return routed[0](*args, **kwargs)
        kv_cache = step.get("kv_cache")
        if kv_cache is None:
            raise RuntimeError("the graph replay needs the model's kv_cache argument")
        h, mod, rope = kwargs["hidden_states"], kwargs["modulation"], kwargs["rotary_emb"]
        mask = kwargs.get("attention_mask")
        key = (tuple(h.shape), tuple(mod.shape), tuple(rope.shape), h.dtype, tuple(kv_cache.get_layer(0).k.shape),
               None if mask is None else tuple(mask.shape))
        graph = graphs.get(key)
        if graph is None:
            while len(graphs) >= max_graphs:
                graphs.popitem(last=False)
            graph = graphs[key] = _StepGraph(blocks, h, mod, rope, mask, kv_cache)
        graphs.move_to_end(key)
        return graph.run(h, mod, rope, mask, kv_cache)

    transformer.transformer_blocks[0].forward = first
    for block, native in zip(transformer.transformer_blocks[1:], routed[1:]):
        block.forward = (lambda *args, _native=native, **kwargs: kwargs["hidden_states"]
                         if kwargs.get("kv_cache_mode") == "cached" and not args else _native(*args, **kwargs))


class DenoiseStepGraph:
    """A whole v1 MMDiT denoise step (mmdit.MMDiT.denoise_step, or
    denoise_step_sharded with a Ulysses/CFG plan) captured once as a CUDA
    graph and replayed for every step: the transformer's 60 blocks with their
    side-stream modulation, norm_out, and proj_out + CFG combine + Euler
    update (qia_proj_out_cfg_euler) -- the `graph` profile applied to the
    whole step rather than only to the blocks.

    The graph reads static device buffers: the latents, both prompt
    embeddings, and the (sigma, sigma_next) pair, which the step kernels read
    on the device, so one graph serves every step of a schedule. step()
    copies its inputs in (host or device tensors, stream-ordered), replays
    and returns the updated latents -- a static buffer that the next step
    overwrites. One graph per (shapes, plan); serial use only."""

    def __init__(self, model, latents: torch.Tensor, prompt_embeds: torch.Tensor, negative_embeds: torch.Tensor,
                 img_shape, cfg_scale: float = 4.0, plan=None, warmup: int = 2):
        dev = model.device
        self.lat = torch.empty(latents.shape, dtype=latents.dtype, device=dev)
        self.pe = torch.empty(prompt_embeds.shape, dtype=prompt_embeds.dtype, device=dev)
        self.ne = torch.empty(negative_embeds.shape, dtype=negative_embeds.dtype, device=dev)
        self.lat.copy_(latents)
        self.pe.copy_(prompt_embeds)
        self.ne.copy_(negative_embeds)
        self.sigmas = torch.tensor([1.0, 0.975], dtype=torch.float32, device=dev)

        def run():
            if plan is not None:
                return model.denoise_step_sharded(self.lat, self.pe, self.ne, self.sigmas, None, img_shape, plan,
                                                  cfg_scale)
            return model.denoise_step(self.lat, self.pe, self.ne, self.sigmas, None, img_shape, cfg_scale)

        for _ in range(max(1, warmup)):       # allocator pools, kernel attributes, tensor maps, NCCL set-up
            run()
        torch.cuda.synchronize(dev)
        self.graph = torch.cuda.CUDAGraph()
        with torch.cuda.graph(self.graph):
            self.out = run()
        torch.cuda.synchronize(dev)

    def step(self, latents: torch.Tensor, sigmas, prompt_embeds: torch.Tensor | None = None,
             negative_embeds: torch.Tensor | None = None) -> torch.Tensor:
        """One step: latents (host or device), sigmas = a device float32
        (sigma, sigma_next) pair such as schedule[i:i + 2] (copied on the
        stream) or a host pair; new embeddings only when they change."""
        if latents.data_ptr() != self.lat.data_ptr():
            self.lat.copy_(latents, non_blocking=True)
        if prompt_embeds is not None:
            self.pe.copy_(prompt_embeds, non_blocking=True)
        if negative_embeds is not None:
            self.ne.copy_(negative_embeds, non_blocking=True)
        if not isinstance(sigmas, torch.Tensor) or not sigmas.is_cuda:
            sigmas = torch.as_tensor(sigmas, dtype=torch.float32).to(self.sigmas.device)
        self.sigmas.copy_(sigmas[:2], non_blocking=True)
        self.graph.replay()
        return self.out

    def denoise(self, latents: torch.Tensor, schedule: torch.Tensor) -> torch.Tensor:
        """len(schedule) - 1 steps from `latents` over the device float32
        schedule (sigma_0, ..., sigma_n); returns the final latents (static)."""
        if not schedule.is_cuda or schedule.dtype != torch.float32:
            schedule = schedule.to(self.sigmas.device, torch.float32)
        x = latents
        for i in range(schedule.numel() - 1):
            x = self.step(x, schedule[i:i + 2])
        return x

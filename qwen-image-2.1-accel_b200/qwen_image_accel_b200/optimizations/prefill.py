"""Block-causal prefill attention of the Qwen-Image 2.1 prefix-KV path.

The 2.1 prefill runs the whole joint sequence (text, condition images, target
image) once, and the cached decode steps reuse its prefix K/V. Its mask
(WHL:diffusers/models/transformers/transformer_qwenimage21.py:257-306,
`mask_mod`: key kv is visible to query q when kv <= q or both belong to the
same image block, and kv is not a padded prompt token) is served in the
reference by one SDPA call per prefix segment plus one for the target image
(QwenImage21AttnProcessor, transformer_qwenimage21.py:499-543) or by a
compiled flex_attention BlockMask (:410-440).

Because every image block is one contiguous run of the sequence
(build_token_metadata, :808-844), that mask is a prefix of the keys for every
query: [0, q + 1) for a text token and [0, end of its block) for an image
token (the target image sees every key). One int32 limit per query therefore
carries the whole structure, and the tcgen05 attention kernel takes it
directly (qia_sage_attention_prefill): it masks per row and skips the key
tiles beyond a query tile's largest limit, so the causal text rows cost only
the keys they see.

Padded prompt keys (key_valid) are removed by moving every sample's valid
keys to the front, in order, and counting the limits in valid keys: the set of
keys each query sees is unchanged, so the result is the masked attention.
"""
from __future__ import annotations

import torch
import torch.nn.functional as F

from .sage_attention import sage_attention_prefill


def block_causal_kv_limits(image_ids: torch.Tensor) -> torch.Tensor:
    """int32 [S] key limits of the 2.1 prefill mask, computed on image_ids'
    device without a host sync. image_ids: int [S], -1 at text tokens and one
    id per image block, each block one contiguous run (as
    QwenImage21Transformer2DModel.build_token_metadata assigns them)."""
    if image_ids.ndim != 1:
        raise ValueError("image_ids must be 1-D [seq_len]")
    ids = image_ids.to(torch.int64)
    s = ids.shape[0]
    pos = torch.arange(s, device=ids.device)
    last = torch.ones(s, dtype=torch.bool, device=ids.device)
    last[:-1] = ids[1:] != ids[:-1]
    # the first run end at or after each token
    run_end = torch.where(last, pos + 1, torch.full_like(pos, s)).flip(0).cummin(0).values.flip(0)
    return torch.where(ids < 0, pos + 1, run_end).to(torch.int32)


def compact_valid_keys(k: torch.Tensor, v: torch.Tensor, key_valid: torch.Tensor, kv_limit: torch.Tensor):
    """Move each sample's valid keys (key_valid bool [B, Skv]) to the front in
    order and recount kv_limit ([Sq]) in valid keys. Returns (k, v, limits
    int32 [B, Sq]); the invalid keys end up past every limit."""
    b, skv = key_valid.shape
    if k.shape[0] != b or k.shape[1] != skv:
        raise ValueError("key_valid must be [batch, seq_kv]")
    valid = key_valid.to(torch.bool)
    order = torch.argsort((~valid).to(torch.int8), dim=1, stable=True)
    idx = order[:, :, None, None].expand(-1, -1, k.shape[2], k.shape[3])
    k_c = torch.gather(k, 1, idx)
    v_c = torch.gather(v, 1, idx)
    seen = torch.cumsum(valid.to(torch.int32), dim=1)                        # valid keys in [0, j]
    lim = kv_limit.to(torch.int64).clamp(0, skv)
    counted = torch.where(lim > 0, torch.gather(seen, 1, (lim - 1).clamp(min=0).expand(b, -1)),
                          torch.zeros_like(seen[:, :1]).expand(b, lim.shape[-1]))
    return k_c, v_c, counted.to(torch.int32).contiguous()


def prefix_segments(image_ids: torch.Tensor, prefix_len: int) -> list[tuple[int, int, bool]]:
    """(start, end, is_text) runs of equal image ids over the prefix, as the
    reference derives them once per forward (one host sync;
    _qwenimage21_prefix_segments, transformer_qwenimage21.py:309-323)."""
    ids = image_ids[:prefix_len].tolist()
    segs, start = [], 0
    for i in range(1, prefix_len + 1):
        if i == prefix_len or ids[i] != ids[start]:
            segs.append((start, i, ids[start] < 0))
            start = i
    return segs


def segment_prefill_sdpa(q: torch.Tensor, k: torch.Tensor, v: torch.Tensor, image_ids: torch.Tensor,
                         prefix_len: int, key_valid: torch.Tensor | None = None,
                         segments: list | None = None) -> torch.Tensor:
    """The reference's default prefill attention, restated over torch SDPA
    (QwenImage21AttnProcessor, transformer_qwenimage21.py:499-543): each
    prefix segment's queries attend to keys [0, end) (text segments with
    their causal triangle), the target's queries to every key; padded keys
    (key_valid False) are dropped. NHD bf16 in and out. This is the bf16
    library path the reference runs; prefill_attention is the tcgen05 one."""
    segs = prefix_segments(image_ids, prefix_len) if segments is None else segments
    qt, kt, vt = (t.transpose(1, 2) for t in (q, k, v))
    outs = []
    for a, b, is_text in segs:
        mask = None
        if is_text:
            n = b - a
            mask = torch.cat([torch.ones(n, a, dtype=torch.bool, device=q.device),
                              torch.tril(torch.ones(n, n, dtype=torch.bool, device=q.device))], dim=1)[None, None]
        if key_valid is not None:
            kvm = key_valid[:, None, None, :b]
            mask = kvm if mask is None else (mask & kvm)
        outs.append(F.scaled_dot_product_attention(qt[:, :, a:b], kt[:, :, :b], vt[:, :, :b], attn_mask=mask))
    mask = None if key_valid is None else key_valid[:, None, None, :]
    outs.append(F.scaled_dot_product_attention(qt[:, :, prefix_len:], kt, vt, attn_mask=mask))
    return torch.cat(outs, dim=2).transpose(1, 2)


def prefill_attention(q: torch.Tensor, k: torch.Tensor, v: torch.Tensor, image_ids: torch.Tensor,
                      key_valid: torch.Tensor | None = None, sm_scale: float | None = None,
                      workspace: torch.Tensor | None = None) -> torch.Tensor:
    """The 2.1 prefill attention: NHD bf16 q, k, v [B, S, H, 128] of the joint
    sequence, image_ids int [S], optional key_valid bool [B, S]; returns NHD
    bf16 [B, S, H, 128]. Same signature meaning as the prefill branch of
    QwenImage21AttnProcessor with `segments` / `key_valid` derived from
    image_ids."""
    if q.shape[1] != image_ids.shape[0] or k.shape[1] != image_ids.shape[0]:
        raise ValueError("prefill expects q, k, v over the whole joint sequence of image_ids")
    limits = block_causal_kv_limits(image_ids.to(q.device))
    if key_valid is not None:
        k, v, limits = compact_valid_keys(k, v, key_valid.to(q.device), limits)
    return sage_attention_prefill(q, k, v, limits, sm_scale=sm_scale, workspace=workspace)

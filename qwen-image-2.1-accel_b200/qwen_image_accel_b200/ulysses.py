"""CFG split + Ulysses sequence parallelism for the dual-stream MMDiT step.

Ranks = 2 (CFG halves: cond / uncond) x U (Ulysses degree inside a half).
Within a half the image tokens are sharded contiguously over the U ranks for
every token-local op (norms, GEMMs, RoPE, residuals); the 256 text tokens are
replicated (1.5 % of the work) so no rank is special. Joint attention needs
every token of a head, so around it Q/K/V of the image tokens go
sequence-sharded -> head-sharded (all-to-all) and O comes back head-sharded ->
sequence-sharded; the text stream's attention output is all-gathered over the
heads. Each CFG pair (u, U+u) swaps its velocity shard once per step.

The layouts follow the Ulysses template the reference's dependency ships
(WHL:diffusers/models/attention_dispatch.py:2099-2182 all-to-all helpers,
:2510-2606 Ulysses attention); the collectives are torch.distributed ones (NCCL
on GPUs; the same functions run on gloo/CPU in the tests).
"""
from __future__ import annotations

from dataclasses import dataclass

import torch
import torch.distributed as dist


@dataclass
class ShardPlan:
    """This rank's place in the (CFG half, Ulysses) grid."""
    world: int
    rank: int
    cfg_split: bool               # two CFG halves (else one half of `world` ranks)
    ulysses: int                  # U, ranks per half
    half: int                     # 0 = cond, 1 = uncond (0 when not split)
    u: int                        # rank inside the half
    group: object = None          # the half's U ranks (all-to-all / all-gather)
    pair: object = None           # (u, U + u): the CFG exchange

    def image_slice(self, img_len: int) -> tuple[int, int]:
        """[lo, hi) of the image tokens this rank owns (contiguous shards)."""
        if img_len % self.ulysses:
            raise ValueError(f"image tokens ({img_len}) must divide by the Ulysses degree {self.ulysses}")
        n = img_len // self.ulysses
        return self.u * n, (self.u + 1) * n


def make_plan(cfg_split: bool = True) -> ShardPlan:
    """Build the process groups. Every rank must call this, in the same order
    (torch.distributed.new_group is collective)."""
    world, rank = dist.get_world_size(), dist.get_rank()
    halves = 2 if (cfg_split and world >= 2) else 1
    if world % halves:
        raise ValueError(f"world size {world} does not split into {halves} CFG halves")
    U = world // halves
    plan = ShardPlan(world, rank, halves == 2, U, rank // U, rank % U)
    for h in range(halves):
        g = dist.new_group(list(range(h * U, (h + 1) * U)))
        if h == plan.half:
            plan.group = g
    if halves == 2:
        for u in range(U):
            g = dist.new_group([u, U + u])
            if u == plan.u:
                plan.pair = g
    return plan


def seq_to_head(x_local: torch.Tensor, plan: ShardPlan, out: torch.Tensor | None = None) -> torch.Tensor:
    """[S_loc, H, d] (this rank's tokens, all heads) -> [U * S_loc, H / U, d]
    (every token of the half, this rank's heads), tokens in rank order."""
    U = plan.ulysses
    S_loc, H, d = x_local.shape
    if H % U:
        raise ValueError(f"heads ({H}) must divide by the Ulysses degree {U}")
    if U == 1:
        if out is not None:
            out.copy_(x_local)
            return out
        return x_local
    send = x_local.view(S_loc, U, H // U, d).permute(1, 0, 2, 3).contiguous()   # [dest, S_loc, H/U, d]
    if out is None:
        out = torch.empty(U * S_loc, H // U, d, device=x_local.device, dtype=x_local.dtype)
    dist.all_to_all_single(out.view(U, S_loc, H // U, d), send, group=plan.group)
    return out


def projection_to_heads(qkv_local: torch.Tensor, heads: int, plan: ShardPlan) -> torch.Tensor:
    """[S_loc, 3*H*d] fused q|k|v projection rows of this rank's tokens (q at
    column 0, k at H*d, v at 2*H*d) -> [U * S_loc, 3*(H/U)*d]: every token of
    the half (rank order), the q|k|v of this rank's H/U heads laid out the same
    way with H/U heads (q at 0, k at (H/U)*d, v at 2*(H/U)*d). One all-to-all
    moves Q, K and V together, before any QK-norm/RoPE (both are per token and
    per head, so they can run after the exchange)."""
    U = plan.ulysses
    S_loc, width = qkv_local.shape
    if heads % U or width % (3 * heads):
        raise ValueError(f"a {width}-wide q|k|v projection of {heads} heads does not split over U={U}")
    if U == 1:
        return qkv_local
    Hl, d = heads // U, width // (3 * heads)
    send = qkv_local.view(S_loc, 3, U, Hl, d).permute(2, 0, 1, 3, 4).contiguous()   # [dest, S_loc, 3, H/U, d]
    out = torch.empty(U * S_loc, 3 * Hl * d, device=qkv_local.device, dtype=qkv_local.dtype)
    dist.all_to_all_single(out.view(U, S_loc, 3, Hl, d), send, group=plan.group)
    return out


def projection_heads(qkv: torch.Tensor, heads: int, plan: ShardPlan) -> torch.Tensor:
    """[S, 3*H*d] q|k|v projection rows (replicated on every rank of the half)
    -> [S, 3*(H/U)*d]: this rank's H/U heads in the projection_to_heads layout."""
    U = plan.ulysses
    S, width = qkv.shape
    if U == 1:
        return qkv
    Hl, d = heads // U, width // (3 * heads)
    h0 = plan.u * Hl
    return qkv.view(S, 3, heads, d)[:, :, h0:h0 + Hl].reshape(S, 3 * Hl * d)


def head_to_seq(o_heads: torch.Tensor, plan: ShardPlan) -> torch.Tensor:
    """[U * S_loc, H / U, d] (every token, this rank's heads) -> [S_loc, H, d]."""
    U = plan.ulysses
    if U == 1:
        return o_heads
    S, Hl, d = o_heads.shape
    S_loc = S // U
    recv = torch.empty(U, S_loc, Hl, d, device=o_heads.device, dtype=o_heads.dtype)   # [src head group, ...]
    dist.all_to_all_single(recv, o_heads.contiguous().view(U, S_loc, Hl, d), group=plan.group)
    return recv.permute(1, 0, 2, 3).reshape(S_loc, U * Hl, d)


def gather_heads(o_heads: torch.Tensor, plan: ShardPlan) -> torch.Tensor:
    """[S, H / U, d] on every rank of the half -> [S, H, d] (the replicated text stream)."""
    U = plan.ulysses
    if U == 1:
        return o_heads
    S, Hl, d = o_heads.shape
    buf = torch.empty(U * S, Hl, d, device=o_heads.device, dtype=o_heads.dtype)   # [rank-major, S, H/U, d]
    dist.all_gather_into_tensor(buf, o_heads.contiguous(), group=plan.group)
    return buf.view(U, S, Hl, d).permute(1, 0, 2, 3).reshape(S, U * Hl, d)


def exchange_cfg(v_local: torch.Tensor, plan: ShardPlan) -> tuple[torch.Tensor, torch.Tensor]:
    """(cond, uncond) velocity of this rank's token shard: the two CFG halves
    swap their shards (one all-gather inside the pair)."""
    if not plan.cfg_split:
        raise ValueError("exchange_cfg needs a CFG split plan")
    n = v_local.shape[0]
    buf = torch.empty((2 * n,) + tuple(v_local.shape[1:]), device=v_local.device, dtype=v_local.dtype)
    dist.all_gather_into_tensor(buf, v_local.contiguous(), group=plan.pair)
    return buf[:n], buf[n:]

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
:2510-2606 Ulysses attention). The functions below are torch.distributed
collectives (NCCL on GPUs; the same functions run on gloo/CPU in the tests).
PeerExchange replaces them on the GPU hot path: the ranks of a Ulysses group
map each other's exchange buffers (CUDA IPC over NVLink), a copy kernel
stores the q|k|v rows straight into the owners' buffers and the attention
kernel's epilogue stores its output straight into the ranks that own the
tokens, with in-kernel completion signals and a bounded wait.
"""
from __future__ import annotations

import ctypes
import os
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


def _head_chunk(local_heads: int, chunk: tuple[int, int]) -> tuple[int, int]:
    """(first head, heads) of chunk c of n of a rank's `local_heads` heads."""
    c, n = chunk
    if n < 1 or not 0 <= c < n or local_heads % n:
        raise ValueError(f"chunk {c} of {n} does not split {local_heads} heads")
    return c * (local_heads // n), local_heads // n


def projection_to_heads(qkv_local: torch.Tensor, heads: int, plan: ShardPlan,
                        chunk: tuple[int, int] = (0, 1)) -> torch.Tensor:
    """[S_loc, 3*H*d] fused q|k|v projection rows of this rank's tokens (q at
    column 0, k at H*d, v at 2*H*d) -> [U * S_loc, 3*Hc*d]: every token of the
    half (rank order), the q|k|v of head chunk `chunk` = (c, n) of this rank's
    H/U heads (Hc = H/U/n heads) laid out the same way with Hc heads (q at 0,
    k at Hc*d, v at 2*Hc*d). One all-to-all moves Q, K and V together, before
    any QK-norm/RoPE (both are per token and per head, so they can run after
    the exchange)."""
    U = plan.ulysses
    S_loc, width = qkv_local.shape
    if heads % U or width % (3 * heads):
        raise ValueError(f"a {width}-wide q|k|v projection of {heads} heads does not split over U={U}")
    Hl, d = heads // U, width // (3 * heads)
    c0, hc = _head_chunk(Hl, chunk)
    if U == 1 and hc == Hl:
        return qkv_local
    send = qkv_local.view(S_loc, 3, U, Hl, d)[:, :, :, c0:c0 + hc].permute(2, 0, 1, 3, 4).contiguous()
    if U == 1:
        return send.view(S_loc, 3 * hc * d)
    out = torch.empty(U * S_loc, 3 * hc * d, device=qkv_local.device, dtype=qkv_local.dtype)
    dist.all_to_all_single(out.view(U, S_loc, 3, hc, d), send, group=plan.group)   # [src, S_loc, 3, Hc, d]
    return out


def projection_heads(qkv: torch.Tensor, heads: int, plan: ShardPlan, chunk: tuple[int, int] = (0, 1)) -> torch.Tensor:
    """[S, 3*H*d] q|k|v projection rows (replicated on every rank of the half)
    -> [S, 3*Hc*d]: head chunk `chunk` of this rank's heads in the
    projection_to_heads layout."""
    U = plan.ulysses
    S, width = qkv.shape
    Hl, d = heads // U, width // (3 * heads)
    c0, hc = _head_chunk(Hl, chunk)
    if hc == heads:
        return qkv
    h0 = plan.u * Hl + c0
    return qkv.view(S, 3, heads, d)[:, :, h0:h0 + hc].reshape(S, 3 * hc * d)


def head_to_seq_into(o_heads: torch.Tensor, out: torch.Tensor, plan: ShardPlan,
                     chunk: tuple[int, int] = (0, 1)) -> torch.Tensor:
    """o_heads [U * S_loc, Hc, d] (every token, head chunk `chunk` of this
    rank's heads) -> the columns of chunk `chunk` of every rank's heads in out
    [S_loc, H, d] (this rank's tokens); returns out."""
    U = plan.ulysses
    S, hc, d = o_heads.shape
    S_loc, H = S // U, out.shape[1]
    Hl = H // U
    c0, n_hc = _head_chunk(Hl, chunk)
    if n_hc != hc or out.shape[0] != S_loc:
        raise ValueError("o_heads does not match the chunk or out")
    if U == 1:
        out[:, c0:c0 + hc].copy_(o_heads)
        return out
    recv = torch.empty(U, S_loc, hc, d, device=o_heads.device, dtype=o_heads.dtype)   # [src rank, ...]
    dist.all_to_all_single(recv, o_heads.contiguous().view(U, S_loc, hc, d), group=plan.group)
    out.view(S_loc, U, Hl, d)[:, :, c0:c0 + hc].copy_(recv.permute(1, 0, 2, 3))
    return out


def gather_heads_into(o_heads: torch.Tensor, out: torch.Tensor, plan: ShardPlan,
                      chunk: tuple[int, int] = (0, 1)) -> torch.Tensor:
    """o_heads [S, Hc, d] (head chunk `chunk` of this rank's heads, on every
    rank of the half) -> the columns of chunk `chunk` of every rank's heads in
    out [S, H, d] (the replicated text stream); returns out."""
    U = plan.ulysses
    S, hc, d = o_heads.shape
    Hl = out.shape[1] // U
    c0, _ = _head_chunk(Hl, chunk)
    if U == 1:
        out[:, c0:c0 + hc].copy_(o_heads)
        return out
    buf = torch.empty(U * S, hc, d, device=o_heads.device, dtype=o_heads.dtype)   # [rank-major, S, Hc, d]
    dist.all_gather_into_tensor(buf, o_heads.contiguous(), group=plan.group)
    out.view(S, U, Hl, d)[:, :, c0:c0 + hc].copy_(buf.view(U, S, hc, d).permute(1, 0, 2, 3))
    return out


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


class _DeviceBytes:
    """A raw device allocation exposed to torch (__cuda_array_interface__)."""

    def __init__(self, ptr: int, nbytes: int):
        self.__cuda_array_interface__ = {"shape": (nbytes,), "typestr": "|u1", "data": (ptr, False), "version": 3}


class PeerExchange:
    """The exchange buffers of one rank of a Ulysses group, mapped into every
    rank of the group with CUDA IPC (NVLink peer memory):

    * recv    [U * S_loc, 3 * Hl * 128] bf16: the q|k|v projection rows of this
      rank's Hl = H/U heads for every image token of the half (the layout the
      fused QK-norm/RoPE + Sage quantizer reads with Hl heads);
    * img_out [S_loc, H, 128] bf16: the attention output of this rank's image
      tokens, every head;
    * txt_out [L_txt, H, 128] bf16: the text tokens' attention output;
    * uint64 counters: [U] q|k|v signals, [U] output signals (one slot per
      source rank), the two wait sites' round numbers, and the scatter
      kernel's CTA count (it signals once per launch).

    Per block: scatter_qkv (qia_ulysses_scatter_qkv into every rank's recv,
    then a wait for the other ranks' rows) and attention (the attention kernel
    storing into every rank's img_out / txt_out, then a wait). A rank writes
    into another rank's buffer only after that rank has passed the previous
    wait of the other kind, which comes after its last read of the buffer, so
    one set of buffers suffices. Built by every rank of the group together,
    outside CUDA graph capture; the buffers live until close()."""

    TIMEOUT_NS = 10_000_000_000     # a wait gives up (QIA_ERR_TIMEOUT) after 10 s

    def __init__(self, plan: ShardPlan, s_loc: int, txt_len: int, heads: int, device):
        from . import _lib
        U, u = plan.ulysses, plan.u
        if heads % U:
            raise ValueError(f"heads ({heads}) must divide by the Ulysses degree {U}")
        hl = heads // U
        self.plan, self.s_loc, self.txt_len, self.heads, self.device = plan, s_loc, txt_len, heads, device
        sizes = {"recv": U * s_loc * 3 * hl * 128 * 2, "img": s_loc * heads * 128 * 2,
                 "txt": txt_len * heads * 128 * 2, "sig": (2 * U + 3) * 8}
        lib = _lib.load()
        hb = int(lib.qia_ipc_handle_bytes())
        self._own, self._mapped, handles = {}, [], {}
        for key, n in sizes.items():
            ptr, h = ctypes.c_void_p(), ctypes.create_string_buffer(hb)
            _lib.call("qia_ipc_alloc", n, ctypes.byref(ptr), h)
            self._own[key], handles[key] = ptr.value, h.raw
        every = [None] * U
        dist.all_gather_object(every, handles, group=plan.group)
        peers = {key: [] for key in sizes}
        for r in range(U):
            for key in sizes:
                if r == u:
                    peers[key].append(self._own[key])
                    continue
                ptr = ctypes.c_void_p()
                _lib.call("qia_ipc_open", ctypes.create_string_buffer(every[r][key], hb), ctypes.byref(ptr))
                peers[key].append(ptr.value)
                self._mapped.append(ptr.value)
        table = lambda ptrs: torch.tensor(ptrs, dtype=torch.int64, device=device)  # noqa: E731
        self.recv_peers, self.img_peers, self.txt_peers = table(peers["recv"]), table(peers["img"]), table(peers["txt"])
        self.sig_qkv_peers = table(peers["sig"])
        self.sig_out_peers = table([p + 8 * U for p in peers["sig"]])
        view = lambda key: torch.as_tensor(_DeviceBytes(self._own[key], sizes[key]), device=device)  # noqa: E731
        self.recv = view("recv").view(torch.bfloat16).view(U * s_loc, 3 * hl * 128)
        self.img_out = view("img").view(torch.bfloat16).view(s_loc, heads, 128)
        self.txt_out = view("txt").view(torch.bfloat16).view(txt_len, heads, 128)
        sig = self._own["sig"]
        self._sig_qkv, self._sig_out = sig, sig + 8 * U
        self._round_qkv, self._round_out = sig + 16 * U, sig + 16 * U + 8
        self._done_scatter = sig + 16 * U + 16
        self.attn_ctas = int(lib.qia_sage_attn_ctas(1, hl, txt_len + U * s_loc))

    def scatter_qkv(self, qkv_local: torch.Tensor) -> torch.Tensor:
        """This rank's [S_loc, 3*H*128] q|k|v rows into every rank's recv, then
        the other ranks' rows into this one's: returns recv."""
        from . import _lib
        U = self.plan.ulysses
        if qkv_local.shape != (self.s_loc, 3 * self.heads * 128) or qkv_local.dtype != torch.bfloat16 \
                or qkv_local.stride(1) != 1:
            raise ValueError("qkv rows must be [S_loc, 3*H*128] bf16 with contiguous rows")
        st = _lib.stream(qkv_local.device)
        _lib.call("qia_ulysses_scatter_qkv", _lib.ptr(qkv_local), qkv_local.stride(0), self.s_loc, self.heads, 128,
                  _lib.ptr(self.recv_peers), _lib.ptr(self.sig_qkv_peers), self._done_scatter, U, self.plan.u, st)
        return self.wait_qkv()

    def wait_qkv(self) -> torch.Tensor:
        """Wait until every rank's q|k|v rows of this round are in recv; returns recv."""
        from . import _lib
        _lib.call("qia_ulysses_wait", self._sig_qkv, self._round_qkv, self.plan.ulysses, 1, self.TIMEOUT_NS,
                  _lib.stream(self.device))
        return self.recv

    def attention(self, workspace: torch.Tensor, sm_scale: float | None = None):
        """The attention half on a workspace that sage_quantize_joint filled
        from (this rank's text heads, recv), its output stored into every
        rank's img_out / txt_out; returns (img_out, txt_out) once every rank's
        rows have arrived."""
        from . import _lib
        U, hl = self.plan.ulysses, self.heads // self.plan.ulysses
        st = _lib.stream(workspace.device)
        _lib.call("qia_sage_attn_quantized_peers", _lib.ptr(workspace), self.txt_len + U * self.s_loc, hl, 128,
                  self.txt_len, _lib.ptr(self.img_peers), _lib.ptr(self.txt_peers), self.s_loc, U, self.plan.u * hl,
                  self.heads, _lib.ptr(self.sig_out_peers), self.plan.u, float(sm_scale or 0.0), st)
        _lib.call("qia_ulysses_wait", self._sig_out, self._round_out, U, self.attn_ctas, self.TIMEOUT_NS, st)
        return self.img_out, self.txt_out

    def close(self):
        """Unmap the peers' buffers and free this rank's (no exchange in flight)."""
        from . import _lib
        torch.cuda.synchronize(self.device)
        for ptr in self._mapped:
            _lib.call("qia_ipc_close", ptr)
        for ptr in self._own.values():
            _lib.call("qia_ipc_free", ptr)
        self._mapped, self._own = [], {}


def peer_exchange_enabled() -> bool:
    """QIA_ULYSSES_P2P=0 selects the torch.distributed collectives instead."""
    return os.environ.get("QIA_ULYSSES_P2P", "1").strip() != "0"

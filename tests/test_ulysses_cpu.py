"""CFG split + Ulysses collectives (qwen_image_accel_b200/ulysses.py) on gloo
CPU ranks: the sequence<->head all-to-alls (of Q/K/V and of the fused q|k|v
projection rows), the head all-gather of the text stream and the CFG velocity
swap equal their single-process definitions, and a head-sharded attention
equals the unsharded one."""
import os
import socket
from datetime import timedelta

import pytest
import torch
import torch.distributed as dist
import torch.multiprocessing as mp


def _free_port() -> int:
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _attention(q, k, v):
    """Exact per-head softmax attention, [S, H, d] float64."""
    s = torch.einsum("qhd,khd->hqk", q, k) / q.shape[-1] ** 0.5
    return torch.einsum("hqk,khd->qhd", torch.softmax(s, dim=-1), v)


def _worker(rank, world, port, cfg_split, results):
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
    dist.init_process_group("gloo", rank=rank, world_size=world, timeout=timedelta(seconds=60))
    try:
        from qwen_image_accel_b200.ulysses import (exchange_cfg, gather_heads, gather_heads_into, head_to_seq,
                                                    head_to_seq_into, make_plan, projection_heads,
                                                    projection_to_heads, seq_to_head)
        plan = make_plan(cfg_split)
        U = plan.ulysses
        S, H, d = 6 * U, 3 * U, 8
        g = torch.Generator().manual_seed(100 + plan.half)       # identical inside a half
        full = torch.randn(S, H, d, generator=g, dtype=torch.float64)
        lo, hi = plan.image_slice(S)
        heads = slice(plan.u * H // U, (plan.u + 1) * H // U)
        got = seq_to_head(full[lo:hi].contiguous(), plan)
        assert torch.equal(got, full[:, heads]), "seq_to_head"
        assert torch.equal(head_to_seq(got, plan), full[lo:hi]), "head_to_seq"
        assert torch.equal(gather_heads(full[:, heads].contiguous(), plan), full), "gather_heads"
        # the fused q|k|v projection rows: this rank's heads of every token, in
        # the layout the joint quantizer reads (q, k, v sections of H/U heads)
        qkv = torch.randn(S, 3 * H * d, generator=g, dtype=torch.float64)
        want = qkv.view(S, 3, H, d)[:, :, heads].reshape(S, 3 * (H // U) * d)
        assert torch.equal(projection_to_heads(qkv[lo:hi].contiguous(), H, plan), want), "projection_to_heads"
        assert torch.equal(projection_heads(qkv, H, plan), want), "projection_heads"
        # head chunks of this rank's heads, and the outputs scattered back by chunk
        Hl = H // U
        o_img = torch.zeros(hi - lo, H, d, dtype=torch.float64)
        o_txt = torch.zeros(S, H, d, dtype=torch.float64)
        for ci in range(3):
            hs = slice(plan.u * Hl + ci * Hl // 3, plan.u * Hl + (ci + 1) * Hl // 3)
            want_c = qkv.view(S, 3, H, d)[:, :, hs].reshape(S, -1)
            assert torch.equal(projection_to_heads(qkv[lo:hi].contiguous(), H, plan, (ci, 3)), want_c), "chunk in"
            assert torch.equal(projection_heads(qkv, H, plan, (ci, 3)), want_c), "chunk text"
            head_to_seq_into(full[:, hs].contiguous(), o_img, plan, (ci, 3))
            gather_heads_into(full[:, hs].contiguous(), o_txt, plan, (ci, 3))
        assert torch.equal(o_img, full[lo:hi]), "head_to_seq_into"
        assert torch.equal(o_txt, full), "gather_heads_into"
        q, k, v = (torch.randn(S, H, d, generator=g, dtype=torch.float64) for _ in range(3))
        local = _attention(*(seq_to_head(t[lo:hi].contiguous(), plan) for t in (q, k, v)))
        assert torch.allclose(head_to_seq(local, plan), _attention(q, k, v)[lo:hi], atol=1e-12), "attention"
        if plan.cfg_split:
            mine = torch.full((3, 2), float(10 * plan.half + plan.u))
            cond, neg = exchange_cfg(mine, plan)
            assert torch.equal(cond, torch.full((3, 2), float(plan.u))), "cfg cond"
            assert torch.equal(neg, torch.full((3, 2), float(10 + plan.u))), "cfg uncond"
        results.put((rank, "ok"))
    except Exception as e:  # noqa: BLE001
        results.put((rank, repr(e)))
    finally:
        dist.destroy_process_group()


@pytest.mark.parametrize("world,cfg_split", [(2, False), (2, True), (4, True)])
def test_ulysses_collectives_gloo(world, cfg_split):
    ctx = mp.get_context("spawn")
    results = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=_worker, args=(r, world, port, cfg_split, results)) for r in range(world)]
    for p in procs:
        p.start()
    out = {}
    try:
        for _ in range(world):
            rank, msg = results.get(timeout=180)
            out[rank] = msg
    finally:
        for p in procs:
            p.join(timeout=30)
            if p.is_alive():
                p.terminate()
    assert out == {r: "ok" for r in range(world)}, out

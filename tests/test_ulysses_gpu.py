"""Sharded MMDiT step (CFG split + Ulysses) against the single-GPU step, on a
tiny model: every per-row and per-head computation is the same kernel on the
same inputs, so the results are bit-identical. With one CFG row per rank the
Ulysses exchanges go through NVLink peer memory (ulysses.PeerExchange: the
q|k|v scatter kernel and the attention's peer-store epilogue, for the MXFP8
blocks and the bf16 block 0 alike); the CFG swap of the velocities goes
through NCCL. Needs >= 2 GPUs (skipped otherwise); run as `pytest -m gpu` on a
multi-GPU box."""
import os
import socket
from datetime import timedelta

import pytest
import torch
import torch.distributed as dist
import torch.multiprocessing as mp

pytestmark = pytest.mark.gpu


def _free_port() -> int:
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _worker(rank, world, port, cfg_split, p2p, results):
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port), QIA_ULYSSES_P2P="1" if p2p else "0")
    torch.cuda.set_device(rank)
    dist.init_process_group("nccl", rank=rank, world_size=world, timeout=timedelta(seconds=120),
                            device_id=torch.device("cuda", rank))
    try:
        from qwen_image_accel_b200.mmdit import MMDiT, MMDiTConfig, random_parameters
        from qwen_image_accel_b200.ulysses import make_plan
        plan = make_plan(cfg_split)
        cfg = MMDiTConfig(num_layers=2, num_attention_heads=4, joint_attention_dim=512)
        dev = torch.device("cuda", rank)
        model = MMDiT(cfg, random_parameters(cfg, 7, "cpu"), device=dev, profile="mxfp8_sage")
        g = torch.Generator(device=dev).manual_seed(0)
        shape = (1, 16, 16)
        lat = torch.randn(1, 256, 64, device=dev, dtype=torch.bfloat16, generator=g)
        pe = torch.randn(1, 40, 512, device=dev, dtype=torch.bfloat16, generator=g)
        ne = torch.randn(1, 40, 512, device=dev, dtype=torch.bfloat16, generator=g)
        lo, hi = plan.image_slice(lat.shape[1])
        if cfg_split:
            ref = model.denoise_step(lat, pe, ne, 1.0, 0.975, shape)
            got = model.denoise_step_sharded(lat[:, lo:hi].contiguous(), pe, ne, 1.0, 0.975, shape, plan)
        else:
            t = torch.full((1,), 1.0, device=dev, dtype=torch.bfloat16)
            ref = model.forward(lat, pe, t, shape, shared_timestep=True)
            got = model.forward_sharded(lat[:, lo:hi].contiguous(), pe, t, shape, plan)
        torch.cuda.synchronize()
        same = torch.equal(got, ref[:, lo:hi])
        diff = (got.float() - ref[:, lo:hi].float()).abs().max().item()
        results.put((rank, "ok" if same else f"mismatch, max |diff| {diff}"))
    except Exception as e:  # noqa: BLE001
        results.put((rank, repr(e)))
    finally:
        dist.destroy_process_group()


# p2p=False: the torch.distributed exchanges (the path of B > 1 per rank)
@pytest.mark.parametrize("world,cfg_split,p2p", [(2, False, True), (2, False, False), (2, True, True),
                                                 (4, True, True), (8, True, True)])
def test_sharded_step_matches_single_gpu(world, cfg_split, p2p):
    if torch.cuda.device_count() < world:
        pytest.skip(f"needs {world} GPUs")
    ctx = mp.get_context("spawn")
    results = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=_worker, args=(r, world, port, cfg_split, p2p, results)) for r in range(world)]
    for p in procs:
        p.start()
    out = {}
    try:
        for _ in range(world):
            rank, msg = results.get(timeout=600)
            out[rank] = msg
    finally:
        for p in procs:
            p.join(timeout=60)
            if p.is_alive():
                p.terminate()
    assert out == {r: "ok" for r in range(world)}, out

"""Benchmark: ms per MMDiT denoise step at 2048^2 and 1024^2 on B200, with the
kernels' roofline fractions (BASELINE.json metric and configs).

Default line (`python bench.py --gpus N`): BASELINE config 5, the 60-block
dual-stream MMDiT denoise step at 2048^2 (16384 image + 256 text tokens per
CFG row) through profile `mxfp8_sage` (blocks 0 and 31 in bf16, as the
reference's default skip list), plus the CFG combine and the flow-match Euler
update. N = 1: the CFG batch of 2 on one GPU. N >= 2 (torchrun): CFG split x
Ulysses N/2 -- each CFG half a Ulysses group over NCCL (all-to-all Q/K/V and O
per block, one velocity exchange per step); strong scaling (the same step at
every N). At N = 1 the same line carries config 4 (the 1024^2 step, its
FFN-up GEMM roofline and CPU baseline) and the kernel measurements of configs
1-3 (AdaLN op vs HBM, the MXFP8 GEMM sweep beside torch._scaled_mm, the joint
attention beside the reference's SageAttention built from its sources).
Random-init weights (~N(0, 0.02)) and seeded synthetic latents / text
embeddings of the BASELINE shapes stand in for the checkpoint and prompts.

Timing: W warm-up steps, the step captured once in a CUDA graph through the
product API (optimizations/cuda_graph.DenoiseStepGraph), K replays bracketed
by barrier + synchronize and timed with CUDA events on the launching stream,
max over ranks. The step streams ~27 GB of weights (far above the 126 MB L2),
so no flush is needed between steps; the kernel-level measurements of configs
1-3 flush L2 (a 256 MiB write, then a 256 MiB read that evicts its dirty
lines) before every timed launch. `e2e`: K steps of
DenoiseStepGraph.step() with the latents and both prompt embeddings copied in
from pinned host memory and the new latents copied back, every step.

`--impl reference`: the reference's eager CPU path -- the Diffusers
QwenImageTransformer2DModel of the pinned wheel (baseline/_ref) in bf16 on
this host's cores, one whole sampled forward per step (img_in, text norm and
projection, timestep embedding, one dual-stream block, norm_out, proj_out,
then the CFG combine and the Euler update) at a bounded token count, scaled
to the configured step by its FLOP ratio.

Other configurations: `--config c4` (1024^2 only; replicas for N > 1),
`prefill` (the 2.1 block-causal prefill attention), `q21` (the Qwen-Image 2.1
cached-decode step), and `--profile-case` small fixed cases for ncu.
"""
from __future__ import annotations

import argparse
import json
import os
import statistics
import subprocess
import sys
import time
from pathlib import Path

ROOT = Path(__file__).resolve().parent
for _p in (ROOT, ROOT / "qwen-image-2.1-accel_b200"):
    if str(_p) not in sys.path:
        sys.path.insert(0, str(_p))

import torch  # noqa: E402

METRIC = "ms per MMDiT denoise step at 2048^2 (60 blocks, CFG batch 2; config 4 = 1024^2 alongside)"
METRIC_C4 = "ms per MMDiT denoise step at 1024^2 (60 blocks, CFG batch 2)"
BLOCKS, HEADS, TXT_LEN, TXT_DIM, DIM, FFN = 60, 24, 256, 3584, 3072, 12288
GRID = (1, 64, 64)                   # 1024^2 latent 16ch x 128 x 128, 2x2 patches
IMG_LEN = GRID[0] * GRID[1] * GRID[2]
GRID_C5 = (1, 128, 128)              # 2048^2 latent 16ch x 256 x 256, 2x2 patches
IMG_LEN_C5 = GRID_C5[0] * GRID_C5[1] * GRID_C5[2]
SIGMAS = (1.0, 0.975)


def step_flops(img_len: int, txt_len: int = TXT_LEN, blocks: int = BLOCKS) -> float:
    """Algorithmic FLOPs of one CFG-batch-2 step: per block and CFG row,
    2 T (4 D^2 + 2 D F) for the linears of both streams over T = image + text
    tokens, and 4 T^2 D for the joint attention."""
    t = img_len + txt_len
    return blocks * 2 * (2.0 * t * (4 * DIM * DIM + 2 * DIM * FFN) + 4.0 * t * t * DIM)


def log(*a):
    print(*a, file=sys.stderr, flush=True)


def load_peaks():
    p = ROOT / "MEASURED_PEAKS.json"
    if p.exists():
        d = json.loads(p.read_text())
        return float(d["hbm_gbs"]), float(d["bf16_tflops"]), "measured"
    return 6650.0, 1590.0, "fallback"


def max_over_ranks(vals, world, device):
    if world == 1:
        return list(vals)
    t = torch.tensor(list(vals), device=device, dtype=torch.float64)
    torch.distributed.all_reduce(t, op=torch.distributed.ReduceOp.MAX)
    return t.tolist()


# ----------------------------------------------------------------------------- clocks
class ClockSampler:
    def __init__(self, gpu_index: int):
        self.proc = None
        self.path = Path(f"/tmp/qia_clocks_{os.getpid()}_{gpu_index}.csv")
        q = ("index,clocks.sm,clocks.max.sm,power.draw,clocks_event_reasons.active,"
             "clocks_event_reasons.hw_slowdown,clocks_event_reasons.hw_thermal_slowdown,"
             "clocks_event_reasons.sw_thermal_slowdown,clocks_event_reasons.sw_power_cap")
        try:
            self.proc = subprocess.Popen(["nvidia-smi", f"--id={gpu_index}", f"--query-gpu={q}",
                                          "--format=csv,noheader,nounits", "-lms", "100"],
                                         stdout=open(self.path, "w"), stderr=subprocess.DEVNULL)
        except OSError:
            self.proc = None

    def stop(self):
        out = {"sm_mhz": None, "sm_max_mhz": None, "reasons": []}
        if self.proc is None:
            return out
        self.proc.terminate()
        try:
            self.proc.wait(timeout=5)
        except subprocess.TimeoutExpired:
            self.proc.kill()
        rows = []
        for line in self.path.read_text().splitlines():
            f = [x.strip() for x in line.split(",")]
            if len(f) >= 9:
                rows.append(f)
        if not rows:
            return out
        sm = [float(r[1]) for r in rows if r[1].replace(".", "").isdigit()]
        out["sm_mhz"] = statistics.median(sm) if sm else None
        out["sm_max_mhz"] = float(rows[0][2]) if rows[0][2].replace(".", "").isdigit() else None
        names = ["hw_slowdown", "hw_thermal_slowdown", "sw_thermal_slowdown", "sw_power_cap"]
        reasons = set()
        for r in rows:
            for i, n in enumerate(names):
                if r[5 + i].lower().startswith("active"):
                    reasons.add(n)
        out["reasons"] = sorted(reasons)
        out["samples"] = len(rows)
        return out


# ----------------------------------------------------------------------------- reference arm (CPU)
REF_SAMPLE_IMG, REF_SAMPLE_TXT = 1024, 256     # tokens of one sampled forward (B = 2, one block)
_CPU_MODEL: dict = {}


def cpu_reference_sample():
    """One bounded sample of the reference's eager CPU path: the Diffusers v1
    QwenImageTransformer2DModel (pinned wheel) with one dual-stream block at
    D 3072 / 24 heads / text 3584, bf16, the CFG batch of 2 with 1024 image +
    256 text tokens per row, then the pipeline's CFG combine and the Euler
    step. Returns (ms, threads, sample FLOPs)."""
    from oracle import diffusers_ref
    from qwen_image_accel_b200.mmdit import MMDiTConfig, init_parameter, parameter_shapes
    threads = os.cpu_count() or 1
    torch.set_num_threads(threads)
    model = _CPU_MODEL.get("m")
    if model is None:
        tq = diffusers_ref.qwen_v1()
        cfg = MMDiTConfig(num_layers=1)
        model = tq.QwenImageTransformer2DModel(patch_size=2, in_channels=64, out_channels=16, num_layers=1,
                                               attention_head_dim=128, num_attention_heads=HEADS,
                                               joint_attention_dim=TXT_DIM, axes_dims_rope=(16, 56, 56))
        model = model.to(torch.bfloat16)
        shapes = parameter_shapes(cfg)
        model.load_state_dict({n: init_parameter(n, shapes[n], 42) for n in model.state_dict()})
        model.eval()
        _CPU_MODEL["m"] = model
    g = torch.Generator().manual_seed(42)
    side = int(REF_SAMPLE_IMG ** 0.5)
    lat = torch.randn(1, REF_SAMPLE_IMG, 64, generator=g).to(torch.bfloat16)
    enc = torch.randn(2, REF_SAMPLE_TXT, TXT_DIM, generator=g).to(torch.bfloat16)
    t = torch.full((2,), SIGMAS[0], dtype=torch.bfloat16)

    def run():
        with torch.no_grad():
            v = model(hidden_states=torch.cat([lat, lat]), encoder_hidden_states=enc, timestep=t,
                      img_shapes=[(1, side, side)] * 2, return_dict=False)[0]
            cond, neg = v[:1], v[1:]
            comb = neg + 4.0 * (cond - neg)
            noise = comb * (torch.norm(cond, dim=-1, keepdim=True) / torch.norm(comb, dim=-1, keepdim=True))
            return (lat.float() + (SIGMAS[1] - SIGMAS[0]) * noise).to(lat.dtype)

    run()
    t0 = time.perf_counter()
    run()
    ms = (time.perf_counter() - t0) * 1e3
    return ms, threads, step_flops(REF_SAMPLE_IMG, REF_SAMPLE_TXT, blocks=1)


def reference_arm(args, rank, world):
    """--impl reference: rank 0 times the reference's eager CPU path (see
    cpu_reference_sample) once per step and scales each sample to the
    configured step by FLOPs; the other ranks exit without work."""
    if rank != 0:
        return
    from oracle import diffusers_ref
    img = IMG_LEN if args.config == "c4" else IMG_LEN_C5
    metric = METRIC_C4 if args.config == "c4" else METRIC
    workload = ("config4: 60-block dual-stream MMDiT, 1024^2 (4096 img + 256 txt tokens), CFG batch 2"
                if args.config == "c4" else
                "config5: 60-block dual-stream MMDiT, 2048^2 (16384 img + 256 txt tokens), CFG batch 2")
    if not diffusers_ref.available():
        print(json.dumps({"impl": "reference", "unavailable": "the pinned Diffusers wheel is not installed under "
                                                               "baseline/_ref"}), flush=True)
        return
    log("reference arm: the Diffusers v1 MMDiT of the pinned wheel, eager bf16 on the host CPU")
    target = step_flops(img)
    vals, sample_ms = [], []
    threads = 1
    for i in range(args.warmup + args.steps):
        ms, threads, flops = cpu_reference_sample()
        if i >= args.warmup:
            sample_ms.append(ms)
            vals.append(ms * target / flops)
    v = statistics.mean(vals)
    sample = (f"one eager forward of the Diffusers model with 1 of 60 blocks (B=2 CFG rows, {REF_SAMPLE_IMG} img + "
              f"{REF_SAMPLE_TXT} txt tokens) + CFG combine + Euler step per step, mean {statistics.mean(sample_ms):.0f}"
              f" ms, scaled by the FLOP ratio {target / step_flops(REF_SAMPLE_IMG, REF_SAMPLE_TXT, 1):.0f}x "
              "(extrapolated)")
    line = {"impl": "reference", "metric": metric, "value": round(v, 1), "unit": "ms/step", "n_gpus": args.gpus,
            "steps": args.steps, "warmup": args.warmup, "ms_per_step": round(v, 1), "higher_is_better": False,
            "scaling": "strong", "vs_baseline": None, "dtype": "bf16", "data": "synthetic",
            "config": {"workload": workload, "global_batch": 2, "seq_len": img + TXT_LEN},
            "cpu_baseline": {"value": round(v, 1), "unit": "ms/step", "cores": threads, "kind": "reference",
                             "sample": sample},
            "e2e": {"value": round(v, 1), "unit": "ms/step", "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0}}
    print(json.dumps(line), flush=True)


# ----------------------------------------------------------------------------- kernel timing helpers
class L2Flush:
    """Writes 256 MiB (twice the 126 MB L2), then reads another 256 MiB, so
    the next launch reads cold and starts with no dirty lines in L2: after
    the write alone, the timed kernel would pay for writing the flush's own
    dirty lines back to DRAM."""

    def __init__(self, device):
        self.buf = torch.empty(256 << 20, dtype=torch.uint8, device=device)
        self.clean = torch.ones(32 << 20, dtype=torch.int64, device=device)
        self.sink = torch.empty((), dtype=torch.int64, device=device)

    def __call__(self):
        self.buf.fill_(1)
        torch.amax(self.clean, dim=0, out=self.sink)


def time_launches(fn, flush: L2Flush, n: int = 20, warmup: int = 3) -> float:
    """Mean device time (ms) of fn() over n launches, each preceded (outside
    its event pair) by an L2 flush; CUDA events on the current stream."""
    for _ in range(warmup):
        fn()
    st = torch.cuda.current_stream()
    evs = [(torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)) for _ in range(n)]
    for e0, e1 in evs:
        flush()
        e0.record(st)
        fn()
        e1.record(st)
    torch.cuda.synchronize()
    return statistics.mean(e0.elapsed_time(e1) for e0, e1 in evs)


def roofline_entry(kernel, achieved, peak, unit, bound, peak_kind, traffic=None, **extra):
    d = {"bound": bound, "kernel": kernel, "achieved": round(achieved, 1), "peak": round(peak, 1), "unit": unit,
         "frac": round(achieved / peak, 3), "traffic": traffic, "peak_kind": peak_kind}
    d.update(extra)
    return d


def ncu_traffic(kernel: str, shape: str):
    """dram__bytes_read.sum + dram__bytes_write.sum of one launch from the
    committed ncu record (profiles/roofline_traffic.json, written from the
    capture named there), or None when no capture of this kernel and shape
    exists."""
    p = ROOT / "profiles" / "roofline_traffic.json"
    if not p.exists():
        return None, None
    recs = json.loads(p.read_text()).get(kernel) or []
    for rec in recs if isinstance(recs, list) else [recs]:
        if rec.get("shape") == shape:
            return int(rec["dram_read_bytes"]) + int(rec["dram_write_bytes"]), rec.get("source")
    return None, None


# ----------------------------------------------------------------------------- our arm: the denoise step
def build_model(device):
    from qwen_image_accel_b200.mmdit import MMDiT, MMDiTConfig, random_parameters
    cfg = MMDiTConfig(num_layers=BLOCKS)
    t0 = time.time()
    model = MMDiT(cfg, random_parameters(cfg, 42, device), device=device, profile="mxfp8_sage")
    torch.cuda.synchronize()
    log(f"model built in {time.time() - t0:.1f} s, {torch.cuda.memory_allocated() / 2**30:.1f} GiB allocated; "
        f"bf16 blocks {sorted(model.skip_blocks)}")
    return model, cfg


def time_step(model, grid, args, rank, world, device, plan=None):
    """The denoise step through DenoiseStepGraph: device-timed K replays with
    inputs resident, then K end-to-end steps from pinned host buffers."""
    from qwen_image_accel_b200 import _lib
    from qwen_image_accel_b200.optimizations.cuda_graph import DenoiseStepGraph
    img_len = grid[0] * grid[1] * grid[2]
    g = torch.Generator(device=device).manual_seed(42)
    latents = torch.randn(1, img_len, 64, device=device, dtype=torch.bfloat16, generator=g)
    pe = torch.randn(1, TXT_LEN, TXT_DIM, device=device, dtype=torch.bfloat16, generator=g)
    ne = torch.randn(1, TXT_LEN, TXT_DIM, device=device, dtype=torch.bfloat16, generator=g)
    if plan is not None:
        lo, hi = plan.image_slice(img_len)
        latents = latents[:, lo:hi].contiguous()
    _lib.launch_count = 0
    graph = DenoiseStepGraph(model, latents, pe, ne, grid, plan=plan, warmup=max(args.warmup, 3))
    launches_per_step = _lib.launch_count // (max(args.warmup, 3) + 1)
    sig = torch.tensor(SIGMAS, dtype=torch.float32, device=device)
    for _ in range(2):
        graph.step(graph.out, sig)
    torch.cuda.synchronize()
    if world > 1:
        torch.distributed.barrier()
    sampler = ClockSampler(torch.cuda.current_device()) if rank == 0 else None
    st = torch.cuda.current_stream()
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    torch.cuda.synchronize()
    if world > 1:
        torch.distributed.barrier()
    e0.record(st)
    for _ in range(args.steps):
        graph.step(graph.out, sig)
    e1.record(st)
    torch.cuda.synchronize()
    if world > 1:
        torch.distributed.barrier()
    clocks = sampler.stop() if sampler else None
    ms = e0.elapsed_time(e1) / args.steps
    # end to end through the public step(): this rank's latents and both
    # prompt embeddings from pinned host memory, the new latents back
    host_lat = latents.cpu().pin_memory()
    host_pe, host_ne = pe.cpu().pin_memory(), ne.cpu().pin_memory()
    host_sig = torch.tensor(SIGMAS, dtype=torch.float32).pin_memory()
    host_out = torch.empty(host_lat.shape, dtype=host_lat.dtype).pin_memory()
    torch.cuda.synchronize()
    if world > 1:
        torch.distributed.barrier()
    e0.record(st)
    for _ in range(args.steps):
        host_out.copy_(graph.step(host_lat, host_sig.to(device, non_blocking=True), host_pe, host_ne),
                       non_blocking=True)
    e1.record(st)
    torch.cuda.synchronize()
    e2e_ms = e0.elapsed_time(e1) / args.steps
    ms, e2e_ms = max_over_ranks([ms, e2e_ms], world, device)
    assert _lib.device_error() == 0, "a device-side wait timed out"
    h2d = host_lat.numel() * 2 + host_pe.numel() * 2 + host_ne.numel() * 2 + host_sig.numel() * 4
    d2h = host_out.numel() * 2
    del graph
    return {"ms": ms, "e2e_ms": e2e_ms, "launches_per_step": launches_per_step, "clocks": clocks, "h2d": h2d,
            "d2h": d2h}


def ffn_up_roofline(model, device, rows, peak_tflops_fp8, peak_kind, flush):
    """Live timing of the step's dominant kernel class -- the image stream's
    FFN up-projection (3072 -> 12288, bias + GELU + MXFP8 requant epilogue),
    as launched in the step, at `rows` image rows -- and cuBLASLt's MXFP8
    GEMM (torch._scaled_mm, the reference's GEMM) on the same operands."""
    from qwen_image_accel_b200.kernels.mxfp8 import quantize
    blk = model.blocks[1]
    g = torch.Generator(device=device).manual_seed(1)
    a = quantize(torch.randn(rows, DIM, device=device, dtype=torch.bfloat16, generator=g))
    ms = time_launches(lambda: blk.img_up.mx.matmul_gelu_quantize(a), flush)
    flops = 2.0 * rows * FFN * DIM
    tflops = flops / (ms * 1e-3) / 1e12
    w, ws = blk.img_up.mx.weight_fp8, blk.img_up.mx.weight_scale
    ms_lib = time_launches(lambda: torch._scaled_mm(a.values, w, scale_a=a.scales, scale_b=ws,
                                                    out_dtype=torch.bfloat16), flush)
    shape = f"M={rows} N={FFN} K={DIM}"
    traffic, source = ncu_traffic("mxfp8_gemm_kernel ffn_up gelu_quant", shape)
    algo = rows * DIM + FFN * DIM + rows * DIM // 32 + FFN * DIM // 32 + rows * FFN * (1 + 1 / 32) + FFN * 2
    return roofline_entry(f"mxfp8_gemm_kernel (FFN up, {shape}, GELU + MXFP8 requant)", tflops, peak_tflops_fp8,
                          "TFLOP/s", "tensor", peak_kind, traffic=traffic, traffic_source=source,
                          algorithmic_bytes=int(algo), ms_per_launch=round(ms, 4),
                          cublaslt_mxfp8_tflops_same_operands=round(flops / (ms_lib * 1e-3) / 1e12, 1),
                          vs_cublaslt=round(ms_lib / ms, 3))


# ----------------------------------------------------------------------------- configs 1-3 (kernel level)
def measure_c1(device, hbm, peak_kind, flush):
    """r + gate * (LN(x) * (1 + scale) + shift) over
    [1, 4096, 3072] bf16 (seed 0: x, shift, scale, r, gate) -- one launch of
    qia_adaln_residual against HBM (read x, read r, write out: 75.5 MB), and
    the eager bf16 op on this host's CPU (median of 10 after 2)."""
    from qwen_image_accel_b200.kernels.adaln import adaln_residual
    g = torch.Generator().manual_seed(0)
    x = torch.randn(1, 4096, DIM, generator=g).to(torch.bfloat16)
    shift = (0.1 * torch.randn(1, DIM, generator=g)).to(torch.bfloat16)
    scale = (0.1 * torch.randn(1, DIM, generator=g)).to(torch.bfloat16)
    r = torch.randn(1, 4096, DIM, generator=g).to(torch.bfloat16)
    gate = (0.1 * torch.randn(1, DIM, generator=g)).to(torch.bfloat16)
    xd, rd = x.to(device), r.to(device)
    one_s = (1 + scale).to(device)[:, None].contiguous()
    sh, ga = shift.to(device)[:, None].contiguous(), gate.to(device)[:, None].contiguous()
    ms = time_launches(lambda: adaln_residual(xd, rd, one_s, sh, ga), flush)
    nbytes = 3 * x.numel() * 2
    gbs = nbytes / (ms * 1e-3) / 1e9
    threads = os.cpu_count() or 1
    torch.set_num_threads(threads)
    ln = torch.nn.LayerNorm(DIM, eps=1e-6, elementwise_affine=False)

    def eager():
        with torch.no_grad():
            return r + gate * (ln(x) * (1 + scale) + shift)

    for _ in range(2):
        eager()
    cpu = []
    for _ in range(10):
        t0 = time.perf_counter()
        eager()
        cpu.append((time.perf_counter() - t0) * 1e3)
    traffic, source = ncu_traffic("adaln_residual_kernel", "[1,4096,3072]")
    return {"workload": "config1: AdaLN composite r + gate*(LN(x)*(1+scale)+shift), x/r bf16 [1,4096,3072]",
            "ms": round(ms, 4),
            "roofline": roofline_entry("adaln_residual_kernel", gbs, hbm, "GB/s", "hbm", peak_kind, traffic=traffic,
                                       traffic_source=source, algorithmic_bytes=nbytes),
            "cpu_baseline": {"value": round(statistics.median(cpu), 2), "unit": "ms", "cores": threads,
                             "kind": "reference", "sample": "the eager bf16 op at full size, median of 10 after 2"}}


C2_SHAPES = (("qkv", 3072, 9216), ("out", 3072, 3072), ("ffn_up", 3072, 12288), ("ffn_down", 12288, 3072))


def measure_c2(device, peak_fp8, hbm, peak_kind, hbm_kind, flush):
    """the MXFP8 GEMM sweep. A bf16 [M, K] ~N(0,1),
    M in {4352, 16640}; W bf16 [N, K] ~N(0,0.02), bias ~N(0,0.01), seed 1;
    both quantized to E4M3 + 1x32 E8M0. Per shape: the tcgen05 GEMM with the
    epilogue the block runs (bias; bias + GELU + MXFP8 requant on the
    up-projection; gate + residual on the output and down projections) and
    torch._scaled_mm (cuBLASLt, the reference's GEMM) on the same operands;
    plus the activation quantizer against HBM (2 B in, 1.03125 B out per
    element) and, per M, the CPU restatement (dequantize -> fp32 matmul) of
    the out-projection on a 256-row sample scaled to M."""
    from qwen_image_accel_b200.kernels.mxfp8 import quantize
    from qwen_image_accel_b200.optimizations.mxfp8 import MXFP8Linear
    import oracle
    out = {"workload": "config2: MXFP8 GEMM sweep, M in {4352, 16640}", "shapes": []}
    g = torch.Generator(device=device).manual_seed(1)
    for m in (4352, 16640):
        for name, k, n in C2_SHAPES:
            a_bf = torch.randn(m, k, device=device, dtype=torch.bfloat16, generator=g)
            lin = torch.nn.Linear(k, n, bias=True, device=device, dtype=torch.bfloat16)
            with torch.no_grad():
                lin.weight.copy_(0.02 * torch.randn(n, k, device=device, generator=g))
                lin.bias.copy_(0.01 * torch.randn(n, device=device, generator=g))
            mx = MXFP8Linear(lin)
            a = quantize(a_bf)
            if name == "ffn_up":
                fn = lambda: mx.matmul_gelu_quantize(a)  # noqa: E731
                epi = "bias+GELU+MXFP8"
            elif name == "qkv":
                fn = lambda: mx.matmul(a)  # noqa: E731
                epi = "bias"
            else:
                res = torch.randn(m, n, device=device, dtype=torch.bfloat16, generator=g)
                gate = (0.1 * torch.randn(1, n, device=device, generator=g)).to(torch.bfloat16)
                fn = lambda: mx.matmul_gate_residual(a, gate, res, out=res)  # noqa: E731
                epi = "bias+gate+residual"
            ms = time_launches(fn, flush)
            ms_lib = time_launches(lambda: torch._scaled_mm(a.values, mx.weight_fp8, scale_a=a.scales,
                                                            scale_b=mx.weight_scale, out_dtype=torch.bfloat16),
                                   flush)
            flops = 2.0 * m * n * k
            tf, tf_lib = flops / (ms * 1e-3) / 1e12, flops / (ms_lib * 1e-3) / 1e12
            out["shapes"].append({"linear": name, "M": m, "K": k, "N": n, "epilogue": epi, "ms": round(ms, 4),
                                  "tflops": round(tf, 1), "frac": round(tf / peak_fp8, 3),
                                  "scaled_mm_ms": round(ms_lib, 4), "scaled_mm_tflops": round(tf_lib, 1),
                                  "vs_scaled_mm": round(ms_lib / ms, 3)})
            del a, a_bf, mx, lin
        xq = torch.randn(m, DIM, device=device, dtype=torch.bfloat16, generator=g)
        ms_q = time_launches(lambda: quantize(xq), flush)
        nbytes = m * DIM * (2 + 1 + 1 / 32)
        traffic, source = ncu_traffic("mx_quantize_kernel", f"[{m},{DIM}]")
        out.setdefault("quantizer", []).append(
            roofline_entry(f"mx_quantize_kernel [{m},{DIM}]", nbytes / (ms_q * 1e-3) / 1e9, hbm, "GB/s", "hbm",
                           hbm_kind, traffic=traffic, traffic_source=source, algorithmic_bytes=int(nbytes),
                           ms=round(ms_q, 4)))
    fr = [s["frac"] for s in out["shapes"]]
    out["frac_min"], out["frac_mean"] = round(min(fr), 3), round(statistics.mean(fr), 3)
    out["vs_scaled_mm_min"] = round(min(s["vs_scaled_mm"] for s in out["shapes"]), 3)
    # CPU restatement sample: 256 rows of the out-projection, scaled to M rows
    threads = os.cpu_count() or 1
    torch.set_num_threads(threads)
    gc = torch.Generator().manual_seed(1)
    w = (0.02 * torch.randn(DIM, DIM, generator=gc)).to(torch.bfloat16)
    x = torch.randn(256, DIM, generator=gc).to(torch.bfloat16)
    wq = oracle.mx_quantize_numpy(w.view(torch.int16).numpy().view("uint16"))
    xq = oracle.mx_quantize_numpy(x.view(torch.int16).numpy().view("uint16"))
    t0 = time.perf_counter()
    oracle.mxfp8_gemm(xq[0], xq[1], wq[0], wq[1], 256, DIM)
    cpu_ms = (time.perf_counter() - t0) * 1e3
    out["cpu_baseline"] = {"value": {str(m): round(cpu_ms * m / 256, 1) for m in (4352, 16640)}, "unit": "ms",
                           "cores": threads, "kind": "port",
                           "sample": "out-projection (3072->3072) dequantize -> fp64 matmul on 256 rows, scaled "
                                     "to M rows"}
    return out


def measure_c3(device, peak_fp8, peak_kind, flush):
    """joint attention, B=2, H=24, d=128, 256 text + 4096
    image tokens; q, k, v ~N(0,1) bf16 (seed 2), per-head QK-RMSNorm
    (weight 1, eps 1e-6) and the v1 3D RoPE (axes 16/56/56, (1,64,64) grid,
    text positions offset) applied with qia_qknorm_rope_segment; then the
    Sage quantizers + tcgen05 attention (sage_attention) beside the
    reference's SageAttention built from its pinned sources, on the same
    inputs; plus the fused QK-norm/RoPE + quantizers of the dual-stream block
    straight from the q|k|v projections. CPU: the restated Sage attention at
    S = 544 (one head, B = 1), scaled by B H (S/544)^2."""
    import numpy as np
    from qwen_image_accel_b200.kernels.attention import joint_qk_norm_rope
    from qwen_image_accel_b200.mmdit import rope_tables
    from qwen_image_accel_b200.optimizations.sage_attention import (sage_attention, sage_quantize_joint,
                                                                    workspace_bytes)
    import oracle
    from oracle import sage_ref
    b, h, lt, li = 2, HEADS, TXT_LEN, IMG_LEN
    s = lt + li
    g = torch.Generator(device=device).manual_seed(2)
    qkv = [torch.randn(b, n, 3 * h * 128, device=device, dtype=torch.bfloat16, generator=g) for n in (lt, li)]
    ones = torch.ones(128, device=device, dtype=torch.bfloat16)
    img, txt = rope_tables(*GRID, lt)
    ft, fi = (torch.view_as_real(t).to(device).contiguous() for t in (txt, img))
    q, k, v = (torch.empty(b, s, h, 128, device=device, dtype=torch.bfloat16) for _ in range(3))
    joint_qk_norm_rope(qkv[0], ones, ones, ft, q, k, v, 0, 1e-6)
    joint_qk_norm_rope(qkv[1], ones, ones, fi, q, k, v, lt, 1e-6)
    ws = torch.empty(workspace_bytes(b, h, s, s), device=device, dtype=torch.uint8)
    o = torch.empty_like(q)
    ms = time_launches(lambda: sage_attention(q, k, v, out=o, workspace=ws), flush)
    ms_quant = time_launches(lambda: sage_quantize_joint(qkv[0], qkv[1], (ones, ones), (ones, ones), ft, fi, h),
                             flush)
    ops = 4.0 * b * h * s * s * 128
    out = {"workload": "config3: joint attention B=2 H=24 S=256+4096 d=128, QK-RMSNorm + 3D RoPE",
           "ms": round(ms, 4), "fused_norm_rope_quantizers_ms": round(ms_quant, 4),
           "roofline": roofline_entry("sage_quant_* + sage_attn_kernel", ops / (ms * 1e-3) / 1e12, peak_fp8,
                                      "TOP/s", "tensor", peak_kind, algorithmic_ops=ops)}
    traffic, source = ncu_traffic("sage_quant_* + sage_attn_kernel", f"B={b} H={h} S={s}")
    out["roofline"].update(traffic=traffic, traffic_source=source)
    if sage_ref.available():
        ref = sage_ref.attention(q, k, v)
        ms_ref = time_launches(lambda: sage_ref.attention(q, k, v), flush)
        a, r = o.double().flatten(), ref.double().flatten()
        out["reference_sageattention"] = {"ms": round(ms_ref, 4), "tops": round(ops / (ms_ref * 1e-3) / 1e12, 1),
                                          "speedup": round(ms_ref / ms, 3),
                                          "cosine": round(float(a @ r / (a.norm() * r.norm())), 6),
                                          "kernel": "SageAttention 2.2.0 sm89 qk_int8_sv_f8_accum_f32_fuse_v_scale"
                                                    "_attn_inst_buf + quantizers, built from the pinned tarball"}
    threads = os.cpu_count() or 1
    sc = 544
    qs, ks, vs = (t[:1, :sc, :1].float().cpu().numpy() for t in (q, k, v))
    t0 = time.perf_counter()
    oracle.sage_attention(np.ascontiguousarray(qs), np.ascontiguousarray(ks), np.ascontiguousarray(vs))
    cpu_ms = (time.perf_counter() - t0) * 1e3
    out["cpu_baseline"] = {"value": round(cpu_ms * b * h * (s / sc) ** 2, 1), "unit": "ms", "cores": 1,
                           "kind": "port", "sample": f"restated Sage attention (numpy) at S={sc}, one head, B=1, "
                                                     "scaled by B*H*(S/544)^2"}
    return out


# ----------------------------------------------------------------------------- the default line
def step_arm(args, rank, world, local_rank):
    """BASELINE config 5 (2048^2) as the headline at every N; at N = 1 also
    config 4 (1024^2) and the kernel measurements of configs 1-3. With
    --config c4: the 1024^2 step alone (replicas for N > 1)."""
    device = torch.device("cuda", local_rank)
    torch.cuda.set_device(device)
    hbm, bf16_tf, peak_kind = load_peaks()
    fp8_peak = 2.0 * bf16_tf     # FP8 tensor rate = 2x the bf16 rate: the denominator is 2x measured cuBLAS bf16
    fp8_kind = f"2x {peak_kind} cuBLAS bf16 burst ({bf16_tf} TFLOP/s)"
    hbm_kind = f"{peak_kind} copy bandwidth"
    model, cfg = build_model(device)
    c4_only = args.config == "c4"
    plan = None
    if world > 1 and not c4_only:
        from qwen_image_accel_b200.ulysses import make_plan
        plan = make_plan(cfg_split=True)
    grid = GRID if c4_only else GRID_C5
    img = grid[0] * grid[1] * grid[2]
    head = time_step(model, grid, args, rank, world, device, plan=plan)
    flush = L2Flush(device)
    extra = {}
    roof = None
    if rank == 0:
        rows = 2 * img if plan is None else 2 * img // plan.world
        roof = ffn_up_roofline(model, device, rows, fp8_peak, fp8_kind, flush)
        per_gpu = step_flops(img) / (head["ms"] * 1e-3) / max(1, world) / 1e12
        roof["step_tflops_per_gpu"] = round(per_gpu, 1)
        roof["step_frac"] = round(per_gpu / fp8_peak, 3)
    cpu = None
    if world == 1 and not c4_only:
        c4 = time_step(model, GRID, args, rank, world, device)
        c4_roof = ffn_up_roofline(model, device, 2 * IMG_LEN, fp8_peak, fp8_kind, flush)
        tf4 = step_flops(IMG_LEN) / (c4["ms"] * 1e-3) / 1e12
        extra["config4"] = {"workload": "config4: 60-block dual-stream MMDiT, 1024^2 (4096 img + 256 txt tokens), "
                                        "CFG batch 2, profile mxfp8_sage",
                            "ms_per_step": round(c4["ms"], 3), "e2e_ms_per_step": round(c4["e2e_ms"], 3),
                            "step_tflops": round(tf4, 1), "step_frac": round(tf4 / fp8_peak, 3),
                            "gpu_launches_per_step": c4["launches_per_step"], "roofline": c4_roof,
                            "clocks": c4["clocks"]}
        del model
        torch.cuda.empty_cache()
        extra["config1"] = measure_c1(device, hbm, hbm_kind, flush)
        extra["config2"] = measure_c2(device, fp8_peak, hbm, fp8_kind, hbm_kind, flush)
        extra["config3"] = measure_c3(device, fp8_peak, fp8_kind, flush)
    if rank == 0 and not args.no_cpu_baseline and world == 1:
        try:
            ms, threads, flops = cpu_reference_sample()
            cpu = {"value": round(ms * step_flops(img) / flops, 1), "unit": "ms/step", "cores": threads,
                   "kind": "reference",
                   "sample": f"one eager forward of the pinned Diffusers v1 model with 1 of 60 blocks (B=2, "
                             f"{REF_SAMPLE_IMG} img + {REF_SAMPLE_TXT} txt tokens) + CFG + Euler on the host CPU "
                             f"({ms:.0f} ms), scaled by FLOPs to the step (extrapolated)"}
            if "config4" in extra:
                extra["config4"]["cpu_baseline"] = dict(cpu, value=round(ms * step_flops(IMG_LEN) / flops, 1))
        except Exception as exc:  # noqa: BLE001
            log(f"CPU baseline unavailable: {exc!r}")
    if rank == 0:
        if c4_only:
            metric, workload = METRIC_C4, ("config4: 60-block dual-stream MMDiT denoise step, 1024^2 (4096 img + 256 "
                                           "txt tokens), CFG batch 2, profile mxfp8_sage")
            parallelism = f"replicas x{world}" if world > 1 else "single GPU"
            value, scaling = head["ms"] / world, "weak"
        else:
            metric, workload = METRIC, ("config5: 60-block dual-stream MMDiT denoise step, 2048^2 (16384 img + 256 "
                                        "txt tokens), CFG batch 2, profile mxfp8_sage")
            parallelism = ("single GPU (CFG batch 2)" if plan is None else
                           (f"CFG split x Ulysses {plan.ulysses} (q|k|v rows and attention output over NVLink "
                            "peer memory; NCCL for the per-step CFG exchange)" if plan.ulysses > 1
                            else "CFG split (one NCCL exchange per step)"))
            value, scaling = head["ms"], "strong"
        line = {"metric": metric, "value": round(value, 3), "unit": "ms/step", "n_gpus": world,
                "steps": args.steps, "warmup": args.warmup, "ms_per_step": round(head["ms"], 3),
                "higher_is_better": False, "scaling": scaling, "vs_baseline": None,
                "dtype": "mxfp8+int8/fp8 attn (blocks 0 and 31 bf16)",
                "data": "synthetic (random-init weights ~N(0,0.02), seeded latents/text)",
                "config": {"workload": workload, "global_batch": 2, "seq_len": img + TXT_LEN,
                           "parallelism": parallelism, "cuda_graph": "DenoiseStepGraph (whole step)",
                           "l2": "step working set (27 GB weights) >> L2, no flush; kernel lines flush L2 (256 MiB "
                                 "write, then a 256 MiB read that evicts its dirty lines) before each timed launch"},
                "e2e": {"value": round(head["e2e_ms"] / (world if c4_only else 1), 3), "unit": "ms/step",
                        "h2d_bytes_per_step": head["h2d"], "d2h_bytes_per_step": head["d2h"]},
                "gpu_launches": head["launches_per_step"] * args.steps,
                "roofline": roof, "cpu_baseline": cpu, "clocks": head["clocks"]}
        line.update(extra)
        print(json.dumps(line), flush=True)


PREFILL_RUNS = (("t", 113), ("i", 4096), ("t", 20), ("i", 4096))   # text, condition image, text, target
PREFILL_HEADS = 32                                                   # Qwen-Image 2.1: 32 x 128 heads


def _prefill_inputs(device):
    runs = PREFILL_RUNS
    ids, blk = [], 0
    for kind, n in runs:
        ids += [-1] * n if kind == "t" else [blk] * n
        blk += kind == "i"
    image_ids = torch.tensor(ids, device=device)
    g = torch.Generator(device=device).manual_seed(3)
    s = image_ids.shape[0]
    q, k, v = (torch.randn(1, s, PREFILL_HEADS, 128, device=device, dtype=torch.bfloat16, generator=g)
               for _ in range(3))
    return image_ids, q, k, v


def prefill_arm(args, rank, world, local_rank):
    """`--config prefill`: the Qwen-Image 2.1 block-causal prefill attention
    (text 113, condition image 4096, text 20, target image 4096 tokens; B=1,
    32 heads x 128) through prefill_attention (Sage quantizers + the tcgen05
    kernel with per-query key limits). Beside it, on the same inputs: the
    same kernel without limits (full attention) and the reference's per-
    segment bf16 SDPA prefill. One replica per GPU for N > 1."""
    from qwen_image_accel_b200 import _lib
    from qwen_image_accel_b200.optimizations.prefill import (block_causal_kv_limits, prefill_attention,
                                                             prefix_segments, segment_prefill_sdpa)
    from qwen_image_accel_b200.optimizations.sage_attention import (sage_attention, sage_attention_prefill,
                                                                    workspace_bytes)
    device = torch.device("cuda", local_rank)
    torch.cuda.set_device(device)
    image_ids, q, k, v = _prefill_inputs(device)
    s = q.shape[1]
    ws = torch.empty(workspace_bytes(1, PREFILL_HEADS, s, s), device=device, dtype=torch.uint8)
    out = torch.empty_like(q)
    limits = block_causal_kv_limits(image_ids)
    visible = int(limits.to(torch.int64).sum())
    tops_call = 4.0 * 128 * PREFILL_HEADS * visible / 1e12      # QK^T + PV over the visible pairs
    stream = torch.cuda.current_stream(device)

    def timed(fn):
        for _ in range(args.warmup):
            fn()
        if world > 1:
            torch.distributed.barrier()
        torch.cuda.synchronize()
        e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        e0.record(stream)
        for _ in range(args.steps):
            fn()
        e1.record(stream)
        torch.cuda.synchronize()
        ms = e0.elapsed_time(e1) / args.steps
        if world > 1:
            t = torch.tensor([ms], device=device)
            torch.distributed.all_reduce(t, op=torch.distributed.ReduceOp.MAX)
            ms = float(t.item())
        return ms

    _lib.launch_count = 0
    clk = ClockSampler(local_rank)
    # per layer: the limits are derived once per forward and shared by every block
    ms = timed(lambda: sage_attention_prefill(q, k, v, limits, out=out, workspace=ws))
    clocks = clk.stop()
    launches = _lib.launch_count // (args.warmup + args.steps)
    ms_full = timed(lambda: sage_attention(q, k, v, out=out, workspace=ws))
    prefix_len = s - PREFILL_RUNS[-1][1]
    segments = prefix_segments(image_ids, prefix_len)       # host-side, once per forward
    ms_ref = timed(lambda: segment_prefill_sdpa(q, k, v, image_ids, prefix_len, segments=segments))
    # end to end through the public prefill API (limits derived from image_ids
    # each call): q, k, v from pinned host memory, the output back to the host
    host = [t.cpu().pin_memory() for t in (q, k, v)]
    host_out = torch.empty(q.shape, dtype=q.dtype).pin_memory()
    dq, dk, dv = (torch.empty_like(q) for _ in range(3))

    def e2e():
        for h, d in zip(host, (dq, dk, dv)):
            d.copy_(h, non_blocking=True)
        host_out.copy_(prefill_attention(dq, dk, dv, image_ids, workspace=ws), non_blocking=True)

    ms_e2e = timed(e2e)
    _, bf16_tf, peak_kind = load_peaks()
    if rank == 0:
        achieved = tops_call / (ms * 1e-3)
        line = {"metric": "ms per Qwen-Image 2.1 block-causal prefill attention (1024^2 edit: 113 + 4096 + 20 + "
                          "4096 tokens, 32 heads)", "value": round(ms, 4), "unit": "ms/call", "n_gpus": world,
                "steps": args.steps, "warmup": args.warmup, "ms_per_step": round(ms, 4),
                "higher_is_better": False, "scaling": "weak", "vs_baseline": None, "dtype": "int8/fp8 attn",
                "data": "synthetic (seeded N(0,1) q, k, v)",
                "config": {"workload": "prefill: block-causal joint attention of the 2.1 prefix-KV path, "
                                       f"S={s}, B=1, H={PREFILL_HEADS}, d=128",
                           "parallelism": f"replicas x{world}" if world > 1 else "single GPU",
                           "visible_pairs_frac": round(visible / (s * s), 4),
                           "l2": "inputs (204 MB) > L2; no flush"},
                "compare": {"full_attention_same_kernel_ms": round(ms_full, 4),
                            "reference_segment_sdpa_bf16_ms": round(ms_ref, 4)},
                "e2e": {"value": round(ms_e2e, 4), "unit": "ms/call", "h2d_bytes_per_step": 3 * q.numel() * 2,
                        "d2h_bytes_per_step": q.numel() * 2},
                "gpu_launches": launches * args.steps,
                "roofline": {"bound": "tensor", "kernel": "prefill call (quantizers + attention), visible pairs "
                                                          f"{tops_call * 1e3:.1f} GOP", "achieved": round(achieved, 1),
                             "peak": round(2 * bf16_tf, 1), "unit": "TOP/s", "frac": round(achieved / (2 * bf16_tf), 3),
                             "traffic": None, "peak_kind": f"2x {peak_kind} cuBLAS bf16 burst"},
                "cpu_baseline": None, "clocks": clocks}
        print(json.dumps(line), flush=True)


Q21_LAYERS, Q21_DIM, Q21_HEADS, Q21_PREFIX, Q21_TARGET = 32, 4096, 32, 113, 4096   # Qwen-Image 2.1, 1024^2 t2i
Q21_CTX = 4096                                                                        # text embedding width


def _q21_setup(device):
    """The Qwen-Image 2.1 transformer of `--config q21` on `device`
    (qwen21_model.Qwen21Transformer, 32 Block21, mxfp8_sage, seeded random
    weights), a 1024^2 text-to-image input in the vision-language slot layout
    (113 text slots + 1024 target slots of 2x2 latent tokens), and closures:
    prefill() = the public forward with kv_cache_mode="extract"; forward(lat)
    = the public forward with kv_cache_mode="cached"; decode(lat) = the same
    cached step without its host-side glue (RoPE table, metadata, slot
    layout, and the text projection the cached step discards), so that it can
    be captured in a CUDA graph (see q21_arm)."""
    import types
    import torch.nn.functional as F
    from qwen_image_accel_b200.kernels.layernorm import layer_norm_scale
    from qwen_image_accel_b200.mmdit import init_parameter
    from qwen_image_accel_b200.qwen21 import Block21Config, KVCache, modulation_values
    from qwen_image_accel_b200.qwen21_model import Qwen21Transformer, model21_parameter_shapes, rope_table
    cfg = Block21Config(dim=Q21_DIM, heads=Q21_HEADS)
    shapes = model21_parameter_shapes(Q21_LAYERS, cfg, context_in_dim=Q21_CTX)
    model = Qwen21Transformer(lambda n: init_parameter(n, shapes[n], 42, device), num_layers=Q21_LAYERS, cfg=cfg,
                              context_in_dim=Q21_CTX, device=device, profile="mxfp8_sage")
    D, S, P = Q21_DIM, Q21_PREFIX + Q21_TARGET, Q21_PREFIX
    side = int(round(Q21_TARGET ** 0.5))
    img_shapes = [[(1, side, side)]]
    img_mask = torch.tensor([[False] * P + [True] * (Q21_TARGET // 4)], device=device)
    g = torch.Generator(device=device).manual_seed(42)
    lat = torch.randn(1, Q21_TARGET, 64, device=device, dtype=torch.bfloat16, generator=g)
    enc = torch.randn(1, P, Q21_CTX, device=device, dtype=torch.bfloat16, generator=g)
    t0, t1 = torch.tensor([0.9], device=device), torch.tensor([0.8], device=device)
    cache = KVCache(Q21_LAYERS)
    pad = torch.cat([torch.zeros(P, dtype=torch.bool), torch.ones(Q21_TARGET, dtype=torch.bool)])
    freqs_target = rope_table(img_shapes[0], pad)[P:].contiguous().to(device)

    def prefill():
        return model.forward(lat, enc, t0, img_shapes, img_mask, kv_cache=cache, kv_cache_mode="extract")

    def forward(latents):
        return model.forward(latents, enc, t1, img_shapes, img_mask, kv_cache=cache, kv_cache_mode="cached")

    t = t1.to(torch.bfloat16)
    temb_in = torch.cat([t, t.new_zeros(1)])

    def decode(latents):
        x = F.linear(latents, model.w["img_in.weight"])
        temb = model.time_embed(temb_in)
        vals = modulation_values(F.linear(F.silu(temb), model.w["modulation.1.weight"]))
        for i, blk in enumerate(model.blocks):
            x = blk.forward_cached(x, vals, freqs_target, cache.get_layer(i))
        scale = F.linear(F.silu(temb[:1]), model.w["norm_out.linear.weight"])
        return F.linear(layer_norm_scale(x, (1 + scale)[:, None].contiguous(), model.ln), model.w["proj_out.weight"])

    return types.SimpleNamespace(model=model, blocks=model.blocks, lat=lat, enc=enc, prefill=prefill, forward=forward,
                                 decode=decode, D=D, S=S, P=P, t1=t1, img_shapes=img_shapes, img_mask=img_mask,
                                 cache=cache)


def q21_arm(args, rank, world, local_rank):
    """`--config q21`: the Qwen-Image 2.1 transformer on the sm_100a kernels
    (qwen21_model.Qwen21Transformer, profile mxfp8_sage): 32 single-stream
    blocks (D 4096, 32 x 128 heads, SwiGLU 12288), 1024^2 text-to-image (4096
    target tokens, a 113-token text prefix). value = one cached-decode step,
    captured in a CUDA graph: img_in, the timestep embedder, the shared
    modulation, the 32 blocks over the target tokens against the prefix KV
    cache, norm_out and proj_out (the text projection, which the cached step
    discards, and the host-side RoPE/metadata glue are left out of the graph).
    e2e = the public forward(kv_cache_mode="cached") from pinned host buffers,
    eager, glue included. Beside it, the prefill step (the public forward with
    kv_cache_mode="extract") with the reference's per-segment SDPA and with
    the tcgen05 block-causal kernel. One replica per GPU for N > 1."""
    from qwen_image_accel_b200 import _lib
    device = torch.device("cuda", local_rank)
    torch.cuda.set_device(device)
    m = _q21_setup(device)
    blocks, lat, prefill, decode, D, S, P = m.blocks, m.lat, m.prefill, m.decode, m.D, m.S, m.P
    st = torch.cuda.current_stream()

    def time_eager(fn, n):
        for _ in range(2):
            fn()
        torch.cuda.synchronize()
        e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        e0.record(st)
        for _ in range(n):
            fn()
        e1.record(st)
        torch.cuda.synchronize()
        return e0.elapsed_time(e1) / n

    ms_prefill_sage = None
    for blk in blocks:
        blk.sage_prefill = True
    ms_prefill_sage = time_eager(prefill, 3)
    for blk in blocks:
        blk.sage_prefill = False
    ms_prefill = time_eager(prefill, 3)             # leaves the reference-path prefix K/V in the cache

    static_lat = lat.clone()
    _lib.launch_count = 0
    for _ in range(max(args.warmup, 3)):
        decode(static_lat)
    torch.cuda.synchronize()
    launches = _lib.launch_count // max(args.warmup, 3)
    graph = torch.cuda.CUDAGraph()
    with torch.cuda.graph(graph):
        static_out = decode(static_lat)
    for _ in range(2):
        graph.replay()
    torch.cuda.synchronize()
    if world > 1:
        torch.distributed.barrier()
    sampler = ClockSampler(torch.cuda.current_device()) if rank == 0 else None
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    torch.cuda.synchronize()
    e0.record(st)
    for _ in range(args.steps):
        graph.replay()
    e1.record(st)
    torch.cuda.synchronize()
    clocks = sampler.stop() if sampler else None
    ms = e0.elapsed_time(e1) / args.steps
    # end to end through the public model API (Qwen21Transformer.forward,
    # kv_cache_mode="cached", eager with its host-side glue): latents and
    # prompt embeddings from pinned host memory, the velocity back to the host
    host_lat, host_enc = lat.cpu().pin_memory(), m.enc.cpu().pin_memory()
    dev_lat, dev_enc = torch.empty_like(lat), torch.empty_like(m.enc)
    host_out = torch.empty(static_out.shape, dtype=static_out.dtype).pin_memory()

    def e2e_step():
        dev_lat.copy_(host_lat, non_blocking=True)
        dev_enc.copy_(host_enc, non_blocking=True)
        host_out.copy_(m.model.forward(dev_lat, dev_enc, m.t1, m.img_shapes, m.img_mask, kv_cache=m.cache,
                                       kv_cache_mode="cached"), non_blocking=True)

    e2e_step()
    torch.cuda.synchronize()
    e0.record(st)
    for _ in range(args.steps):
        e2e_step()
    e1.record(st)
    torch.cuda.synchronize()
    ms_e2e = e0.elapsed_time(e1) / args.steps
    if world > 1:
        t = torch.tensor([ms, ms_e2e], device=device)
        torch.distributed.all_reduce(t, op=torch.distributed.ReduceOp.MAX)
        ms, ms_e2e = t.tolist()
    assert _lib.device_error() == 0, "a device-side wait timed out"
    _, bf16_tf, peak_kind = load_peaks()
    T, F_ = Q21_TARGET, 3 * D
    tflop = Q21_LAYERS * (2.0 * T * (4 * D * D + 3 * D * F_) + 4.0 * T * S * D) / 1e12
    if rank == 0:
        achieved = tflop / (ms * 1e-3)
        line = {"metric": "ms per Qwen-Image 2.1 cached-decode denoiser step (32 blocks, 1024^2: 4096 target "
                          "tokens, 113-token prefix KV)", "value": round(ms, 3), "unit": "ms/step", "n_gpus": world,
                "steps": args.steps, "warmup": args.warmup, "ms_per_step": round(ms, 3), "higher_is_better": False,
                "scaling": "weak", "vs_baseline": None, "dtype": "mxfp8+int8/fp8 attn",
                "data": "synthetic (random-init weights ~N(0,0.02), seeded latents/embeddings, random RoPE phases)",
                "config": {"workload": "q21: Qwen-Image 2.1 transformer cached-decode step, profile mxfp8_sage "
                                       "(img_in, timestep embedder, modulation, 32 blocks, norm_out, proj_out in "
                                       "a CUDA graph; e2e = the eager public forward)", "global_batch": 1,
                           "seq_len": T,
                           "prefix_len": P, "parallelism": f"replicas x{world}" if world > 1 else "single GPU",
                           "cuda_graph": True, "l2": "weights (7 GB MXFP8) >> L2; no flush"},
                "compare": {"prefill_step_ms_segment_sdpa": round(ms_prefill, 2),
                            "prefill_step_ms_sage_block_causal": round(ms_prefill_sage, 2),
                            "reference_rtx5090_mxfp8_sage_decode_ms": 147.3,
                            "reference_rtx5090_mxfp8_sage_prefill_ms": 186.5},
                "e2e": {"value": round(ms_e2e, 3), "unit": "ms/step",
                        "h2d_bytes_per_step": host_lat.numel() * 2 + host_enc.numel() * 2,
                        "d2h_bytes_per_step": host_out.numel() * 2},
                "gpu_launches": launches * args.steps,
                "roofline": {"bound": "tensor", "kernel": f"whole decode step ({tflop:.1f} TFLOP)",
                             "achieved": round(achieved, 1), "peak": round(2 * bf16_tf, 1), "unit": "TFLOP/s",
                             "frac": round(achieved / (2 * bf16_tf), 3), "traffic": None,
                             "peak_kind": f"2x {peak_kind} cuBLAS bf16 burst"},
                "cpu_baseline": None, "clocks": clocks}
        print(json.dumps(line), flush=True)
    del graph


def profile_case(name: str):
    """Small fixed cases for ncu captures (no timing, no JSON line):
    ffn_up  - the FFN-up GEMM with the GELU+MXFP8 epilogue, M=8192 (one launch)
    attn    - Sage attention B=1, H=24, S=4352 (three calls)
    step8   - an 8-block 1024^2 step: two warm-up steps, then one inside an NVTX
              range named `step` (for `ncu --nvtx --nvtx-include step/`)
    step8_c5 - the same at 2048^2 (config 5's shapes)
    quant   - the fused QK-norm/RoPE + Sage quantization of one block (B=2, 256
              text + 4096 image tokens, 24 heads, from the two streams' q|k|v
              projections), twice (three launches each).
    prefill - the 2.1 block-causal prefill attention of `--config prefill`
              (S=8325, 32 heads), three calls (four launches each).
    q21step - the `--config q21` denoiser: prefill, two decode steps, then one
              decode step inside an NVTX range named `step`.
    ffn_up_c5 - the FFN-up GEMM (GELU+MXFP8 epilogue) at config 5's M=32768.
    exchange - the config-5 Ulysses exchange kernels at one rank's sizes of the
              4-GPU layout (U=2: 8192 image tokens per rank, 24 heads, 256 text
              tokens), two ranks emulated on one GPU as two launches into two
              buffer sets: the q|k|v scatter (twice), the wait, the fused
              quantizer and the attention with its peer-store epilogue (twice).
    kernels - one launch each of the memory-bound kernels at the step's
              shapes: LN + modulation -> MXFP8 (image + text rows, grouped),
              the AdaLN modulation GEMV (one block), the config-1 AdaLN
              composite [1,4096,3072], the MXFP8 quantizer [8192,3072],
              SwiGLU -> MXFP8 (table and direct forms, [4096,12288]), QK-norm +
              RoPE of one stream segment (B=2, 4096 tokens, 24 heads), the
              CFG/Euler update and the fused proj_out + CFG/Euler tail
              (1024^2: 4096 tokens)."""
    device = torch.device("cuda", 0)
    torch.cuda.set_device(device)
    g = torch.Generator(device=device).manual_seed(0)
    if name == "ffn_up":
        from qwen_image_accel_b200.kernels.mxfp8 import quantize
        from qwen_image_accel_b200.optimizations.mxfp8 import MXFP8Linear
        lin = torch.nn.Linear(3072, 12288, bias=True, device=device, dtype=torch.bfloat16)
        a = quantize(torch.randn(8192, 3072, device=device, dtype=torch.bfloat16, generator=g))
        MXFP8Linear(lin).matmul_gelu_quantize(a)
    elif name == "ffn_up_c5":
        from qwen_image_accel_b200.kernels.mxfp8 import quantize
        from qwen_image_accel_b200.optimizations.mxfp8 import MXFP8Linear
        lin = torch.nn.Linear(DIM, FFN, bias=True, device=device, dtype=torch.bfloat16)
        a = quantize(torch.randn(2 * IMG_LEN_C5, DIM, device=device, dtype=torch.bfloat16, generator=g))
        MXFP8Linear(lin).matmul_gelu_quantize(a)
    elif name == "kernels":
        profile_kernels(device, g)
    elif name == "exchange":
        profile_exchange(device, g)
    elif name == "attn":
        from qwen_image_accel_b200.optimizations.sage_attention import sage_attention
        q, k, v = (torch.randn(1, IMG_LEN + TXT_LEN, HEADS, 128, device=device, dtype=torch.bfloat16, generator=g)
                   for _ in range(3))
        for _ in range(3):
            sage_attention(q, k, v)
    elif name == "prefill":
        from qwen_image_accel_b200.optimizations.prefill import block_causal_kv_limits
        from qwen_image_accel_b200.optimizations.sage_attention import sage_attention_prefill
        image_ids, q, k, v = _prefill_inputs(device)
        limits = block_causal_kv_limits(image_ids)
        for _ in range(3):
            sage_attention_prefill(q, k, v, limits)
    elif name == "q21step":
        m = _q21_setup(device)
        m.prefill()
        for _ in range(2):
            m.decode(m.lat)
        torch.cuda.synchronize()
        torch.cuda.nvtx.range_push("step")
        m.decode(m.lat)
        torch.cuda.nvtx.range_pop()
    elif name == "quant":
        from qwen_image_accel_b200.mmdit import rope_tables
        from qwen_image_accel_b200.optimizations.sage_attention import sage_quantize_joint
        qkv = [torch.randn(2, n, 3 * HEADS * 128, device=device, dtype=torch.bfloat16, generator=g)
               for n in (TXT_LEN, IMG_LEN)]
        w = [tuple((1 + 0.1 * torch.randn(128, device=device, generator=g)).to(torch.bfloat16) for _ in range(2))
             for _ in range(2)]
        img, txt = rope_tables(1, GRID[1], GRID[2], TXT_LEN)
        ft, fi = (torch.view_as_real(t).to(device).contiguous() for t in (txt, img))
        for _ in range(2):
            sage_quantize_joint(qkv[0], qkv[1], w[0], w[1], ft, fi, HEADS)
    elif name in ("step8", "step8_c5"):
        from qwen_image_accel_b200.mmdit import MMDiT, MMDiTConfig, random_parameters
        grid = GRID if name == "step8" else GRID_C5
        cfg = MMDiTConfig(num_layers=8)
        # blocks 1-7 MXFP8 (block 0 bf16, as the 60-block step's blocks 0 and 31)
        model = MMDiT(cfg, random_parameters(cfg, 42, device), device=device, profile="mxfp8_sage")
        n = grid[0] * grid[1] * grid[2]
        lat = torch.randn(1, n, 64, device=device, dtype=torch.bfloat16, generator=g)
        pe = torch.randn(1, TXT_LEN, TXT_DIM, device=device, dtype=torch.bfloat16, generator=g)
        ne = torch.randn(1, TXT_LEN, TXT_DIM, device=device, dtype=torch.bfloat16, generator=g)
        for _ in range(2):
            model.denoise_step(lat, pe, ne, 1.0, 0.975, grid)
        torch.cuda.synchronize()
        torch.cuda.nvtx.range_push("step")
        model.denoise_step(lat, pe, ne, 1.0, 0.975, grid)
        torch.cuda.nvtx.range_pop()
    else:
        raise SystemExit(f"unknown profile case {name!r}")
    torch.cuda.synchronize()
    log(f"profile case {name}: done")


def profile_exchange(device, g):
    """The `exchange` profile case (see profile_case)."""
    from qwen_image_accel_b200 import _lib
    from qwen_image_accel_b200.mmdit import rope_tables
    from qwen_image_accel_b200.optimizations.sage_attention import sage_quantize_joint
    U, s_loc, H = 2, IMG_LEN_C5 // 2, HEADS
    hl, S = H // U, TXT_LEN + IMG_LEN_C5
    bf = torch.bfloat16
    qkv = torch.randn(U * s_loc, 3 * H * 128, device=device, dtype=bf, generator=g)
    qkv_t = torch.randn(TXT_LEN, 3 * H * 128, device=device, dtype=bf, generator=g)
    recv = [torch.empty(U * s_loc, 3 * hl * 128, device=device, dtype=bf) for _ in range(U)]
    img = [torch.empty(s_loc, H, 128, device=device, dtype=bf) for _ in range(U)]
    txt = [torch.empty(TXT_LEN, H, 128, device=device, dtype=bf) for _ in range(U)]
    sig = [torch.zeros(2 * U + 4, dtype=torch.int64, device=device) for _ in range(U)]
    table = lambda ts, off=0: torch.tensor([t.data_ptr() + off for t in ts], dtype=torch.int64, device=device)  # noqa: E731
    rt, it, tt, sq, so = table(recv), table(img), table(txt), table(sig), table(sig, 8 * U)
    st = _lib.stream(device)
    for u in range(U):
        rows = qkv[u * s_loc:(u + 1) * s_loc]
        _lib.call("qia_ulysses_scatter_qkv", _lib.ptr(rows), rows.stride(0), s_loc, H, 128, _lib.ptr(rt),
                  _lib.ptr(sq), _lib.ptr(sig[u][2 * U + 2:]), U, u, st)
    _lib.call("qia_ulysses_wait", _lib.ptr(sig[0]), _lib.ptr(sig[0][2 * U:]), U, 1, 10_000_000_000, st)
    w = tuple(torch.ones(128, device=device, dtype=bf) for _ in range(2))
    fi, ft = (torch.view_as_real(t).to(device).contiguous() for t in rope_tables(*GRID_C5, TXT_LEN))
    for u in range(U):
        heads_u = qkv_t.view(TXT_LEN, 3, U, hl, 128)[:, :, u].reshape(TXT_LEN, 3 * hl * 128)
        ws = sage_quantize_joint(heads_u[None], recv[u][None], w, w, ft, fi, hl)
        _lib.call("qia_sage_attn_quantized_peers", _lib.ptr(ws["_workspace"]), S, hl, 128, TXT_LEN, _lib.ptr(it),
                  _lib.ptr(tt), s_loc, U, u * hl, H, _lib.ptr(so), u, 0.0, st)
    torch.cuda.synchronize()
    if _lib.device_error():
        raise SystemExit("exchange profile case: a device-side wait timed out")


def profile_kernels(device, g):
    """The `kernels` profile case (see profile_case)."""
    from qwen_image_accel_b200.kernels.adaln import adaln_residual
    from qwen_image_accel_b200.kernels.attention import joint_qk_norm_rope
    from qwen_image_accel_b200.kernels.epilogue import layer_norm_scale_quantize_grouped, swiglu_quantize
    from qwen_image_accel_b200.kernels.modulation import adaln_modulation
    from qwen_image_accel_b200.kernels.mxfp8 import quantize
    from qwen_image_accel_b200.kernels.scheduler import cfg_euler, proj_out_cfg_euler
    from qwen_image_accel_b200.mmdit import _LNParams, rope_tables
    bf = torch.bfloat16
    rn = lambda *shape, s=1.0: (s * torch.randn(*shape, device=device, generator=g)).to(bf)  # noqa: E731
    ln = _LNParams(DIM, 1e-6)
    x, c = rn(2, IMG_LEN, DIM), rn(2, TXT_LEN, DIM)
    sc, sh = 1 + rn(2, 1, DIM, s=0.1), rn(2, 1, DIM, s=0.1)
    layer_norm_scale_quantize_grouped([(x, sc, sh), (c, sc, sh)], ln)
    adaln_modulation(rn(DIM), rn(12 * DIM, DIM, s=0.02), rn(12 * DIM, s=0.01), DIM)
    x1, r1 = rn(1, 4096, DIM), rn(1, 4096, DIM)
    adaln_residual(x1, r1, 1 + rn(1, 1, DIM, s=0.1), rn(1, 1, DIM, s=0.1), rn(1, 1, DIM, s=0.1))
    quantize(rn(8192, DIM))
    gt, vt = rn(4096, 12288), rn(4096, 12288)
    swiglu_quantize(gt, vt)
    swiglu_quantize(gt[:512].contiguous(), vt[:512].contiguous())
    img, _ = rope_tables(*GRID, TXT_LEN)
    fi = torch.view_as_real(img).to(device).contiguous()
    qkv = rn(2, IMG_LEN, 3 * DIM)
    q, k, v = (torch.empty(2, IMG_LEN, HEADS, 128, device=device, dtype=bf) for _ in range(3))
    w = 1 + rn(128, s=0.1)
    joint_qk_norm_rope(qkv, w, w, fi, q, k, v, 0, 1e-6)
    lat = rn(1, IMG_LEN, 64)
    sig = torch.tensor(SIGMAS, device=device, dtype=torch.float32)
    cfg_euler(rn(1, IMG_LEN, 64), rn(1, IMG_LEN, 64), lat, 4.0, sigmas=sig)
    proj_out_cfg_euler(rn(2, IMG_LEN, DIM), rn(64, DIM, s=0.02), rn(64, s=0.01), lat, 4.0, sig)
    from qwen_image_accel_b200.qwen21_model import rope_table_device
    mask = torch.cat([torch.zeros(113, dtype=torch.bool), torch.ones(4096, dtype=torch.bool),
                      torch.zeros(20, dtype=torch.bool), torch.ones(4096, dtype=torch.bool)]).to(device)
    rope_table_device([(1, 64, 64), (1, 64, 64)], mask)


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=10)
    ap.add_argument("--warmup", type=int, default=3)
    ap.add_argument("--impl", default="ours", choices=["ours", "reference"])
    ap.add_argument("--no-cpu-baseline", action="store_true")
    ap.add_argument("--config", default="c5", choices=["c5", "c4", "prefill", "q21"],
                    help="c5 (default): the 2048^2 step (CFG split x Ulysses for N>1), with config 4 and the "
                         "configs 1-3 kernel lines at N=1; c4: the 1024^2 step (replicas for N>1); prefill: the "
                         "2.1 block-causal prefill attention; q21: the 2.1 cached-decode step")
    ap.add_argument("--profile-case", choices=["ffn_up", "ffn_up_c5", "kernels", "exchange", "attn", "step8", "step8_c5",
                                               "quant", "prefill", "q21step"],
                    help="run one small fixed case for an ncu capture and exit")
    args = ap.parse_args()
    if args.profile_case:
        profile_case(args.profile_case)
        return
    world = int(os.environ.get("WORLD_SIZE", "1"))
    rank = int(os.environ.get("RANK", "0"))
    local_rank = int(os.environ.get("LOCAL_RANK", "0"))
    if args.impl == "reference":
        reference_arm(args, rank, world)
        return
    if world > 1:
        from datetime import timedelta
        torch.cuda.set_device(local_rank)
        torch.distributed.init_process_group("nccl", timeout=timedelta(seconds=300))
    try:
        if args.config == "prefill":
            prefill_arm(args, rank, world, local_rank)
        elif args.config == "q21":
            q21_arm(args, rank, world, local_rank)
        else:
            step_arm(args, rank, world, local_rank)
    finally:
        if world > 1:
            torch.distributed.destroy_process_group()


if __name__ == "__main__":
    main()

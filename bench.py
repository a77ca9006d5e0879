"""Benchmark: VisionHOPE-T forward images/s at 224x224 (bf16 autocast, channels-last, CUDA graph).

    python bench.py [--gpus N] [--steps K] [--warmup W] [--impl ours|reference] [--batch B]

One step = one forward of B synthetic images per GPU (N(0,1), seed 3 + rank) through the
prepared model, plus the NCCL all-gather of the logits when N > 1 (batch sharding: weak
scaling).  Inputs and the model's activation footprint are far larger than L2, and a
256 MiB buffer is additionally rewritten between timed steps (outside the timed events).
Rank 0 prints one JSON line; the time is the max over ranks of the summed per-step CUDA
event times.  Extra keys:
  e2e          -- the same metric through the public model call, timed over the whole run:
                  every step's batch is copied from pinned host memory (on a copy stream,
                  overlapping the previous step's forward, then device to device into the
                  graph's input) and its logits are copied back to pinned host memory;
  roofline     -- the dominant kernel (the fused SRNL operator at the stage-1 shape of this
                  batch) timed alone with CUDA events, against the measured bf16 tensor peak
                  (MEASURED_PEAKS.json); roofline.kernels lists every hot-path kernel (the scan
                  at each stage, qnorm, direction fusion, GRN, LayerNorm) against its peak;
  ref_kernel   -- the reference's own fused operator kernel timed beside ours per stage;
  cpu_baseline -- the reference's own modules on the host CPU (SRNL recurrence on the oracle's
                  float port: the reference has none) on a small sample, rank 0 at N = 1 only;
  clocks       -- nvidia-smi samples taken during the timed region.
--impl reference runs only that CPU workload (rank 0), timed per step, and prints its line.
"""
from __future__ import annotations

import argparse
import contextlib
import json
import os
import statistics
import subprocess
import sys
import tempfile
import time
import types
from pathlib import Path

import torch
import torch.distributed as dist

ROOT = Path(__file__).resolve().parent
sys.path.insert(0, str(ROOT))

METRIC = "VisionHOPE-T fwd images/sec @224"
UNIT = "images/s"
IMG = 224          # classification input side
IMG_HW = (224, 224)  # this run's input (H, W): --image
# Per-stage (mixer heads) of the model configurations (models/factory.py:9-16, head_dim 16).
STAGE_HEADS = {"visionhope_tiny": (2, 4, 8, 16), "visionhope_small": (2, 5, 10, 16),
               "visionhope_base": (3, 6, 14, 20)}


def parse():
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=10)
    ap.add_argument("--warmup", type=int, default=3)
    ap.add_argument("--impl", choices=("ours", "reference"), default="ours")
    ap.add_argument("--batch", type=int, default=256)
    ap.add_argument("--model", default="visionhope_tiny")
    ap.add_argument("--task", choices=("classify", "dense"), default="classify",
                    help="classify: logits (config 4); dense: forward_intermediates, the four stage "
                         "feature maps of the dense-prediction backbone (config 5)")
    ap.add_argument("--image", default="224", help="input size: S or HxW (config 5: 512x2048)")
    ap.add_argument("--cpu-sample", type=int, default=8, help="images per CPU baseline step")
    ap.add_argument("--no-cpu-baseline", action="store_true")
    ap.add_argument("--only-scan", action="store_true",
                    help="time only the fused SRNL operator at the stage-1 shape (profiling aid)")
    ap.add_argument("--only-depthwise", action="store_true",
                    help="time the block's depthwise kernels and GRN apply at the model's shapes and exit")
    ap.add_argument("--only-backward", action="store_true",
                    help="time the backward (training) kernels at the operator and GRN/LN configurations' "
                         "shapes, and the reference's own backward kernels beside them, and exit")
    ap.add_argument("--only-norms", action="store_true",
                    help="time only GRN and LayerNorm at the GRN/LN configuration's shapes")
    args = ap.parse_args()
    global IMG_HW
    hw = [int(v) for v in args.image.lower().split("x")]
    IMG_HW = (hw[0], hw[-1])
    return args


def metric_name(args):
    if args.task == "dense":
        return f"{args.model} backbone (forward_intermediates) images/sec @{IMG_HW[0]}x{IMG_HW[1]}"
    if args.model == "visionhope_tiny" and IMG_HW == (224, 224):
        return METRIC
    return f"{args.model} fwd images/sec @{IMG_HW[0]}x{IMG_HW[1]}"


def dist_env():
    world = int(os.environ.get("WORLD_SIZE", "1"))
    rank = int(os.environ.get("RANK", "0"))
    local = int(os.environ.get("LOCAL_RANK", "0"))
    return world, rank, local


def config(args, world):
    H, W = IMG_HW
    kind = "classification forward" if args.task == "classify" else "backbone forward_intermediates"
    gathered = "logits" if args.task == "classify" else "the four stage feature maps"
    return {"workload": f"{args.model} {kind}, {H}x{W}, batch {args.batch}/GPU",
            "model": args.model, "global_batch": args.batch * world, "batch_per_gpu": args.batch,
            "image_size": [H, W], "precision": "bf16 autocast, fp32 params", "channels_last": True,
            "execution": "cuda_graph", "parallelism": f"dp{world} (batch-sharded, all_gather {gathered})",
            "l2": "L2 evicted between timed steps (a 256 MiB buffer written, then another 256 MiB read, "
                  "outside the timed events); activations >> L2",
            "seed": 3}


# ----------------------------------------------------------------------------------------
# The reference on the host CPU: the reference's own modules (staged unmodified by
# oracle/build_ref.py, imported by oracle/refmodel.py), prepared for inference exactly as on a
# GPU.  They have no CPU SRNL recurrence (SRNL._run rejects CPU tensors, models/srnl.py:113-114),
# so that one method is routed to the oracle's float port of the reference kernels
# (oracle/vhope_oracle.c, OpenMP over chains); everything else -- the four serialized scans,
# W_q, the PyTorch direction fusion of the ordinary path (operator.py:121-139), LayerNorm's
# F.layer_norm, grn_reference, the convolutions -- is the reference's own CPU code.
def reference_cpu_model(name, **kwargs):
    """(reference namespace, prepared reference model on CPU), weights from seed 3."""
    from oracle import refmodel

    ref = refmodel.load("native")  # on CPU none of the reference's kernels is ever reached
    torch.manual_seed(3)
    model = ref.create_model(name, **kwargs).to(memory_format=torch.channels_last)
    ref.prepare_for_inference(model)
    return ref, model


@contextlib.contextmanager
def oracle_srnl(ref):
    """Run the reference SRNL module's recurrence (SRNL._run) on the oracle's float port."""
    import numpy as np

    from oracle import oracle as orc

    saved = ref.SRNL._run

    def run(self, x, queries, spatial_shape):
        height, width = spatial_shape if spatial_shape is not None else (None, None)
        chunk = self.chunk_size if self.chunk_size is not None else (width or 64)
        chunks = [chunk] * x.shape[1]
        if self.chunk_size is None and spatial_shape is not None:
            chunks = [width, width, height, height]
        y = orc.srnl_sequence([m.detach() for m in self.initial_memories], x, queries, chunks, use_f32=True)
        return torch.from_numpy(y.astype(np.float32))

    ref.SRNL._run = run
    try:
        yield
    finally:
        ref.SRNL._run = saved


def build_model(name, device):
    from visionhope_b200.backbone import create_model, prepare_for_inference

    torch.manual_seed(3)
    model = create_model(name).to(device)
    model = model.to(memory_format=torch.channels_last)
    prepare_for_inference(model)
    return model


def sync_model(model, world):
    """Make every rank's weights identical to rank 0's (one broadcast per tensor at init)."""
    if world > 1:
        for p in model.parameters():
            dist.broadcast(p.data, 0)
        for buf in model.buffers():
            dist.broadcast(buf, 0)


def rank_inputs(batch, rank, device, generator_device=None):
    """This rank's shard of the synthetic batch: N(0,1) images from seed 3 + rank."""
    gen = torch.Generator(device=generator_device or device).manual_seed(3 + rank)
    x = torch.randn(batch, 3, *IMG_HW, device=generator_device or device, generator=gen)
    return x.to(device).contiguous(memory_format=torch.channels_last)


def max_over_ranks(value, device, world):
    t = torch.tensor([float(value)], device=device)
    if world > 1:
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
    return float(t.item())


def cpu_threads():
    return len(os.sched_getaffinity(0)) if hasattr(os, "sched_getaffinity") else os.cpu_count()


def cpu_plan(args, steps, warmup):
    """(steps, warm-up) of the CPU reference sample, bounded to tens of seconds: a dense
    512 x 2048 image takes tens of seconds on the host, so that task times one image per step,
    at most two steps, without warm-up."""
    if args.task == "dense":
        args.cpu_sample = 1
        return max(1, min(steps, 2)), 0
    return steps, warmup


def run_cpu(args, steps, warmup):
    """Time the reference on the host CPU: returns (images/s, per-step seconds, cores, sample)."""
    steps, warmup = cpu_plan(args, steps, warmup)
    cores = cpu_threads()
    torch.set_num_threads(cores)
    os.environ.setdefault("OMP_NUM_THREADS", str(cores))
    ref, model = reference_cpu_model(args.model)
    gen = torch.Generator().manual_seed(3)
    x = torch.randn(args.cpu_sample, 3, *IMG_HW, generator=gen).contiguous(memory_format=torch.channels_last)
    times = []
    with oracle_srnl(ref), torch.inference_mode():
        for i in range(warmup + steps):
            t0 = time.perf_counter()
            model(x) if args.task == "classify" else model.forward_intermediates(x)
            dt = time.perf_counter() - t0
            if i >= warmup:
                times.append(dt)
    ips = args.cpu_sample * len(times) / sum(times)
    sample = (f"{args.cpu_sample} image(s)/step of the same {args.model} {args.task} forward at "
              f"{IMG_HW[0]}x{IMG_HW[1]}, fp32 on "
              f"{cores} host threads: the reference's own modules (prepared), SRNL recurrence on the oracle's "
              f"float port (the reference has no CPU SRNL), {steps} timed steps after {warmup} warm-up")
    return ips, times, cores, sample


# ----------------------------------------------------------------------------------------
class ClockSampler:
    """nvidia-smi clock/throttle samples of every visible GPU during the timed region (every
    ``interval_ms``; entering waits, up to 5 s, for the first sample, so that the sampler runs
    before the timed region starts).  Under torchrun only rank 0 samples (``enabled``), at a
    longer interval: one nvidia-smi per rank, each polling all eight GPUs, took driver time
    from the ranks' own launches."""

    FIELDS = ("index,clocks.sm,clocks.max.sm,power.draw,clocks_event_reasons.active,"
              "clocks_event_reasons.hw_slowdown,clocks_event_reasons.hw_thermal_slowdown,"
              "clocks_event_reasons.sw_thermal_slowdown,clocks_event_reasons.sw_power_cap,pci.bus_id")

    def __init__(self, enabled=True, interval_ms=50):
        self.enabled = enabled
        self.interval_ms = interval_ms
        self.proc = None
        self.path = None
        self.skip = 0

    def __enter__(self):
        if not self.enabled:
            return self
        fd, self.path = tempfile.mkstemp(suffix=".csv")
        os.close(fd)
        try:
            self.proc = subprocess.Popen(
                ["nvidia-smi", f"--query-gpu={self.FIELDS}", "--format=csv,noheader,nounits",
                 "-lms", str(self.interval_ms)], stdout=open(self.path, "w"), stderr=subprocess.DEVNULL)
        except (FileNotFoundError, OSError):
            self.proc = None
        t0 = time.time()
        while self.proc is not None and time.time() - t0 < 5.0 and self.proc.poll() is None:
            if Path(self.path).stat().st_size > 0:
                break
            time.sleep(0.02)
        self.skip = len(Path(self.path).read_text().splitlines()) if self.path else 0
        return self

    def __exit__(self, *exc):
        if self.proc is not None:
            self.proc.terminate()
            try:
                self.proc.wait(timeout=5)
            except subprocess.TimeoutExpired:
                self.proc.kill()

    def summary(self, bus_ids):
        """Clock record of the GPUs the job ran on, named by PCI bus id ("domain:bus:device",
        from every rank's own device), so GPUs of the node that the job does not use never
        enter the figures; per-GPU medians are listed so an idle GPU would show."""
        if self.proc is None or not self.path:
            return {"sm_mhz": None, "sm_max_mhz": None, "reasons": ["nvidia-smi unavailable"]}
        mhz, mx, reasons, power, per_gpu = [], [], set(), [], {}
        names = ("hw_slowdown", "hw_thermal_slowdown", "sw_thermal_slowdown", "sw_power_cap")
        for line in Path(self.path).read_text().splitlines()[self.skip:]:
            parts = [p.strip() for p in line.split(",")]
            if len(parts) < 10:
                continue
            bus = normalize_bus_id(parts[9])
            if bus not in bus_ids:
                continue
            try:
                mhz.append(float(parts[1]))
                mx.append(float(parts[2]))
                power.append(float(parts[3]))
            except ValueError:
                continue
            per_gpu.setdefault(bus, []).append(float(parts[1]))
            for n, v in zip(names, parts[5:9]):
                if v.lower() == "active":
                    reasons.add(n)
        os.unlink(self.path)
        return {"sm_mhz": statistics.median(mhz) if mhz else None, "sm_max_mhz": max(mx) if mx else None,
                "power_w_max": max(power) if power else None, "samples": len(mhz),
                "per_gpu_sm_mhz": {b: statistics.median(v) for b, v in sorted(per_gpu.items())},
                "gpus": sorted(bus_ids), "reasons": sorted(reasons)}


def normalize_bus_id(text):
    """nvidia-smi's "00000000:1B:00.0" -> "0:1b:0" (domain, bus and device as hex numbers)."""
    try:
        dom, bus, rest = text.strip().split(":")
        return f"{int(dom, 16):x}:{int(bus, 16):x}:{int(rest.split('.')[0], 16):x}"
    except ValueError:
        return text.strip().lower()


def job_bus_ids(device, world):
    """PCI bus ids of the GPUs of every rank of the job (one all_gather at set-up)."""
    p = torch.cuda.get_device_properties(device)
    mine = f"{p.pci_domain_id:x}:{p.pci_bus_id:x}:{p.pci_device_id:x}"
    if world == 1:
        return {mine}
    ids = [None] * world
    dist.all_gather_object(ids, mine)
    return set(ids)


def measure_ffma_peak(device):
    """Measured FP32 (non-tensor) FMA throughput of this GPU, TFLOP/s (own probe kernel)."""
    from visionhope_b200 import _lib

    lib = _lib.load()
    sms = torch.cuda.get_device_properties(device).multi_processor_count
    blocks, iters = sms * 16, 4096
    out = torch.empty(blocks * 256, device=device)
    st = _lib.stream_handle(device)
    for _ in range(2):
        _lib.check(lib.vh_probe_ffma(out.data_ptr(), blocks, iters, st), "vh_probe_ffma")
    best = 0.0
    for _ in range(5):
        a, b = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        a.record()
        _lib.check(lib.vh_probe_ffma(out.data_ptr(), blocks, iters, st), "vh_probe_ffma")
        b.record()
        b.synchronize()
        flops = 2.0 * 32 * iters * blocks * 256
        best = max(best, flops / (a.elapsed_time(b) * 1e-3) / 1e12)
    return best


def srnl_flops(B, H, W, heads, D=16):
    """2 x the reference's analytic recurrence MACs (analysis/operation_count.py:226-258)."""
    token = 6 * D * D + 20 * D
    boundary = 3 * D ** 3 + 2 * D ** 2
    macs = 0
    for chunk, nchunks in ((W, H), (W, H), (H, W), (H, W)):
        macs += B * heads * (nchunks * chunk * token + nchunks * boundary)
    return 2.0 * macs


def measured_peaks():
    path = ROOT / "MEASURED_PEAKS.json"
    return json.loads(path.read_text()) if path.exists() else {}


class L2Flush:
    """Evicts the L2 cache (126 MB on B200) between timed kernel launches, outside the timed
    events: a 256 MiB buffer is written, then a second 256 MiB buffer is read.  The read pass
    writes the first buffer's dirty lines back before the timed launch, so the timed kernel
    starts from a cache that holds none of its data and no dirty lines to write back (after a
    write-only flush, a short kernel pays ~126 MB of someone else's write-backs, ~19 us)."""

    def __init__(self, device):
        self.a = torch.empty(64 * 1024 * 1024, device=device)
        self.b = torch.ones(64 * 1024 * 1024, device=device)
        self.sink = torch.empty((), device=device)

    def __call__(self):
        self.a.fill_(1.0)
        torch.amax(self.b, dim=0, out=self.sink)


_flush = {}


def l2_flush(device):
    """The L2Flush of `device` (one pair of buffers per GPU, however the device is named)."""
    key = torch.device("cuda", device) if isinstance(device, int) else torch.device(device)
    if key.index is None:
        key = torch.device("cuda", torch.cuda.current_device())
    if key not in _flush:
        _flush[key] = L2Flush(key)
    return _flush[key]


def _event_ms(fn, iters, flush=None):
    """Mean CUDA-event time (ms) of one call of fn over `iters` calls after 3 warm-up calls,
    with the L2 cache evicted before each call (outside the events)."""
    for _ in range(3):
        fn()
    torch.cuda.synchronize()
    flush = flush or l2_flush(torch.cuda.current_device())
    times = []
    for _ in range(iters):
        flush()
        a, b = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        a.record()
        fn()
        b.record()
        b.synchronize()
        times.append(a.elapsed_time(b))
    return statistics.mean(times)


def _scan_inputs(device, B, H, W, heads, D=16, seed=1):
    g = torch.Generator(device=device).manual_seed(seed)
    C = heads * D
    x = torch.randn(B, H, W, C, device=device, generator=g).to(torch.bfloat16)
    q = torch.randn(B, H, W, C, device=device, generator=g).to(torch.bfloat16)
    mems = [torch.randn(4, heads, D, D, device=device, generator=g) * 0.01 for _ in range(3)]
    mems += [torch.zeros(4, heads, D, device=device) for _ in range(2)]
    return x, q, mems, torch.zeros(C, device=device), torch.ones(4, C, device=device)


def scan_roofline(device, B, H, W, heads, iters, label):
    """The fused four-direction operator (one vh_srnl_spatial_fwd call, bf16 in, fp32 out) at
    one shape: algorithmic FLOPs (2 x the reference's analytic MACs) and bytes (read x and q
    once, write the fp32 result once) per call over its CUDA-event time, against the measured
    bf16 tensor and HBM peaks."""
    from visionhope_b200 import _lib
    from visionhope_b200.srnl_core.fused import spatial_forward

    D = 16
    x, q, mems, skip, wts = _scan_inputs(device, B, H, W, heads, D)
    out = torch.empty(B, H, W, heads * D, device=device)
    fn = lambda: spatial_forward(mems, x, q, skip, wts, H, W, D, layout="image", out=out)
    n0 = _lib.launch_count
    fn()
    launches = _lib.launch_count - n0
    ms = _event_ms(fn, max(iters, 5))
    pk = measured_peaks()
    flops = srnl_flops(B, H, W, heads, D)
    nbytes = B * H * W * heads * D * (2 + 2 + 4)
    tfs, gbs = flops / (ms * 1e-3) / 1e12, nbytes / (ms * 1e-3) / 1e9
    return {"kernel": "srnl scan (fused 4-direction operator)", "shape": label, "B": B, "H": H, "W": W,
            "heads": heads, "ms": ms, "launches": launches, "flops": flops, "alg_bytes": nbytes,
            "tflops": tfs, "gbs": gbs,
            "tensor_frac": tfs / pk["bf16_tflops"] if "bf16_tflops" in pk else None,
            "hbm_frac": gbs / pk["hbm_gbs"] if "hbm_gbs" in pk else None}


def roofline_scan(args, device, steps):
    """The dominant kernel of the forward (the SRNL operator at the stage-1 shape of this batch),
    timed alone with CUDA events, against the measured bf16 tensor peak (its contractions run
    on the tensor cores); the HBM fraction and the FP32-FMA fraction (own probe, not in
    MEASURED_PEAKS.json) are listed beside it."""
    H, W = IMG_HW[0] // 4, IMG_HW[1] // 4
    heads = STAGE_HEADS[args.model][0]
    r = scan_roofline(device, args.batch, H, W, heads, steps, f"{args.model} stage 1")
    pk = measured_peaks()
    ffma = measure_ffma_peak(device)
    peak = pk.get("bf16_tflops")
    return {
        "kernel": "SRNL operator, one vh_srnl_spatial_fwd call (warp-per-chain scan, or the tensor-core "
                  "scan plus its fold where a launch has few chains)",
        "shape": f"B={args.batch} H={H} W={W} C={16 * heads} heads={heads} D=16 bf16 in, fp32 out",
        "launches_per_call": r["launches"],
        "bound": "tensor", "unit": "TFLOP/s", "achieved": r["tflops"], "peak": peak,
        "frac": r["tflops"] / peak if peak else None,
        "peak_source": "MEASURED_PEAKS.json bf16_tflops (cuBLAS bf16 GEMM burst) -- of measured",
        "traffic": None,
        "traffic_note": "not measured in this run (ncu is not run inside the bench); one launch's DRAM "
                        "bytes from an ncu capture are in profiles/srnl_warp_kernel_stage1_b256.md",
        "launch_ms": r["ms"], "flops_per_launch": r["flops"], "alg_bytes_per_launch": r["alg_bytes"],
        "hbm_frac_of_measured": r["hbm_frac"], "tensor_frac_of_measured": r["tensor_frac"],
        "fp32_ffma_peak_tflops": ffma, "fp32_ffma_frac": r["tflops"] / ffma if ffma else None,
    }


def roofline_fusion(device, iters=5):
    """Query normalization and direction fusion (the ordinary path's bandwidth kernels) at the
    operator configuration's shape, B = 64, 56 x 56, C = 96: qnorm reads bf16 q [B, 4, L, C] and
    writes fp32 [B, 4, heads, L, D] (6 B per element); dirfuse reads fp32 y and x
    [B, 4, heads, L, D] and writes the fp32 NCHW output (36 B per output element)."""
    from visionhope_b200.utils.direction_fusion import visionhope_postprocess_scale
    from visionhope_b200.utils.query_normalization import visionhope_qnorm

    B, H, W, heads, D = 64, 56, 56, 6, 16
    L, C = H * W, heads * D
    g = torch.Generator(device=device).manual_seed(2)
    hbm = measured_peaks().get("hbm_gbs")
    qr = torch.randn(B, 4, L, C, device=device, generator=g).to(torch.bfloat16)
    y = torch.randn(B, 4, heads, L, D, device=device, generator=g)
    xx = torch.randn(B, 4, heads, L, D, device=device, generator=g)
    skip = torch.randn(heads, D, device=device, generator=g)
    scale = torch.randn(4, C, device=device, generator=g)
    rows = []
    for name, fn, nbytes in (
            ("qnorm", lambda: visionhope_qnorm(qr, heads, D), qr.numel() * 6),
            ("dirfuse (NCHW out)", lambda: visionhope_postprocess_scale(y, xx, skip, scale, H, W, False),
             B * L * C * 36),
            ("dirfuse (channels-last out)", lambda: visionhope_postprocess_scale(y, xx, skip, scale, H, W, True),
             B * L * C * 36)):
        ms = _event_ms(fn, iters)
        gbs = nbytes / (ms * 1e-3) / 1e9
        rows.append({"kernel": name, "shape": [B, 4, heads, L, D], "ms": ms, "alg_bytes": nbytes,
                     "achieved_gbs": gbs, "hbm_frac": gbs / hbm if hbm else None})
    return rows


def ref_kernel_compare(device, B, iters=3):
    """The reference's own fused operator kernel (srnl_line_forward_seq_noatomic, built from its
    sources into oracle/_ref) beside ours at VisionHOPE-T's four stage shapes and this batch:
    the reference gets its four serialized scans (materialised outside the timed call), ours
    the channels-last image; both bf16 in, fp32 out."""
    from oracle.build_ref import load_built
    from visionhope_b200.srnl_core.fused import spatial_forward

    try:
        ext = load_built("vhref_fused_bf16")
    except (FileNotFoundError, ImportError, OSError) as exc:
        return {"unavailable": str(exc)}
    rows = []
    for stage, (H, heads) in enumerate(((56, 2), (28, 4), (14, 8), (7, 16)), 1):
        x, q, mems, skip, wts = _scan_inputs(device, B, H, H, heads)
        C = heads * 16

        def serialize(t):
            hw = t.reshape(B, H * H, C)
            wh = t.transpose(1, 2).reshape(B, H * H, C)
            return torch.stack([hw, hw.flip(1), wh, wh.flip(1)], dim=1).contiguous()

        xs, qs = serialize(x), serialize(q)
        t_ref = _event_ms(lambda: ext.srnl_line_forward_seq_noatomic(*mems, xs, qs, skip, wts, H, H, 16), iters)
        t_ours = _event_ms(lambda: spatial_forward(mems, x, q, skip, wts, H, H, 16, layout="image"), iters)
        del xs, qs
        rows.append({"stage": stage, "shape": [B, H, H, C], "reference_ms": t_ref, "ours_ms": t_ours,
                     "speedup": t_ref / t_ours})
    return {"kernel": "reference srnl_line_token_parallel + merge (fused.cu:307-351) vs vh_srnl_spatial_fwd",
            "stages": rows}


def per_kernel_rooflines(args, device):
    """roofline.kernels: every hot-path kernel against MEASURED_PEAKS.json (the scan at each of
    this model's stage shapes, then the operator configuration's shape, qnorm, direction fusion,
    GRN and LayerNorm)."""
    B = args.batch
    rows = [scan_roofline(device, B, IMG_HW[0] >> (i + 1), IMG_HW[1] >> (i + 1), heads, 5,
                          f"{args.model} stage {i}")
            for i, heads in enumerate(STAGE_HEADS[args.model], 1)]
    rows.append(scan_roofline(device, 64, 56, 56, 6, 5, "operator configuration (B=64, C=96)"))
    rows += roofline_fusion(device)
    rows += roofline_norms(device, 5)["norms_roofline"]
    return rows


def roofline_norms(device, iters=10):
    """GRN and LayerNorm alone at the GRN/LN configuration's shapes (channels-last
    [128, 56, 56, 96] and [128, 7, 7, 768], fp32 and bf16 in, fp32 out): achieved HBM GB/s of
    the algorithmic bytes (one read of x, one write of y) against the measured copy bandwidth.
    "grn" is the standalone op (statistics and apply from x); "grn_apply" is the apply pass
    fed with per-slice sums of x^2, as the model runs it after the FFN depthwise kernel (the
    sums come from an untimed pre-pass here).  The L2 cache is evicted before every timed
    launch (outside the events, L2Flush)."""
    from visionhope_b200 import _lib
    from visionhope_b200.utils.grn_cuda import grn_apply, grn_forward
    from visionhope_b200.utils.layer_norm_cuda import layernorm_rows

    peaks = json.loads((ROOT / "MEASURED_PEAKS.json").read_text()) if (ROOT / "MEASURED_PEAKS.json").exists() else {}
    hbm = peaks.get("hbm_gbs")
    flush = l2_flush(device)
    g = torch.Generator(device=device).manual_seed(2)
    rows = []
    for (B, H, W, C) in ((128, 56, 56, 96), (128, 7, 7, 768)):
        for dt in (torch.float32, torch.bfloat16):
            x = torch.randn(B, H, W, C, device=device, generator=g).to(dt).permute(0, 3, 1, 2)
            gam = torch.randn(C, device=device, generator=g) * 0.02
            bet = torch.randn(C, device=device, generator=g) * 0.02
            w = 1 + torch.randn(C, device=device, generator=g) * 0.02
            xr = x.permute(0, 2, 3, 1).reshape(-1, C)
            sums = x.float().pow(2).sum(dim=(2, 3)).reshape(B, 1, C)
            for name, fn in (("grn", lambda: grn_forward(x, gam, bet, 1e-6)),
                             ("grn_apply", lambda: grn_apply(x, sums, gam, bet, 1e-6)),
                             ("layernorm", lambda: layernorm_rows(xr, w, bet, 1e-6))):
                ms, launches = _time_calls(fn, iters, flush)
                nbytes = x.numel() * (x.element_size() + 4)
                gbs = nbytes / (ms * 1e-3) / 1e9
                rows.append({"kernel": name, "shape": [B, H, W, C], "dtype_in": str(dt).split(".")[-1],
                             "dtype_out": "float32", "ms": ms, "alg_bytes": nbytes, "achieved_gbs": gbs,
                             "launches": launches, "frac_of_measured_hbm": gbs / hbm if hbm else None})
    return {"norms_roofline": rows, "peak_hbm_gbs": hbm, "peak_source": "MEASURED_PEAKS.json hbm_gbs"}


def _time_calls(fn, iters, flush):
    """Median CUDA-event time (ms) of fn over `iters` calls after 3 warm-up calls, with the L2
    cache evicted before each (outside the events, L2Flush), and libvhope launches per call."""
    from visionhope_b200 import _lib

    for _ in range(3):
        fn()
    times = []
    n0 = _lib.launch_count
    for _ in range(iters):
        flush()
        a, b = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        a.record()
        fn()
        b.record()
        b.synchronize()
        times.append(a.elapsed_time(b))
    return statistics.median(times), (_lib.launch_count - n0) // iters


def roofline_backward(device, iters=5):
    """The backward kernels at the configurations' shapes, each timed alone (L2 evicted before
    every call, outside the events): query normalization and direction fusion at the operator
    configuration (B = 64, 56 x 56, C = 96, bf16 activations as under autocast), LayerNorm and GRN
    at the GRN/LN configuration's large shape (128 x 56 x 56 x 96, fp32), the LayerScale residual
    add (forward and backward; fp32 residual, bf16 branch) at that shape, and the SRNL recurrence
    backward at the operator configuration (1536 chains of 3136 tokens in chunks of 56, raw bf16
    queries).  HBM-bound kernels report achieved GB/s of their algorithmic bytes (every input read
    once, every output written once) against MEASURED_PEAKS.json; the recurrence reports
    chain-tokens per second.  `reference` times the reference's own backward kernels (built from
    its sources into oracle/_ref) on the same tensors where it has them."""
    from visionhope_b200.srnl_core.chunk import recurrence_constants_tuple, sequence_backward
    from visionhope_b200.utils.direction_fusion import postprocess_backward
    from visionhope_b200.utils.grn_cuda import grn_backward, grn_forward
    from visionhope_b200.utils.layer_norm_cuda import layernorm_rows, layernorm_rows_backward
    from visionhope_b200.utils.query_normalization import _qnorm_forward, qnorm_backward

    hbm = measured_peaks().get("hbm_gbs")
    flush = l2_flush(device)
    g = torch.Generator(device=device).manual_seed(9)
    rows = []

    def add(name, shape, fn, nbytes=None, units=None, unit_name=None, ref_fn=None):
        ms, launches = _time_calls(fn, iters, flush)
        row = {"kernel": name, "shape": shape, "ms": ms, "launches": launches}
        if nbytes:
            gbs = nbytes / (ms * 1e-3) / 1e9
            row.update(alg_bytes=nbytes, achieved_gbs=gbs, frac_of_measured_hbm=gbs / hbm if hbm else None)
        if units:
            row[unit_name] = units / (ms * 1e-3)
        if ref_fn is not None:
            try:
                rms, _ = _time_calls(ref_fn, iters, flush)
                row.update(reference_ms=rms, speedup_vs_reference=rms / ms)
            except Exception as exc:  # the reference's kernels are optional here
                row["reference"] = f"unavailable: {exc}"
        rows.append(row)

    def ref_mod(name):
        try:
            from oracle.build_ref import load_built
            return load_built(name)
        except Exception:
            return None

    # query normalization and direction fusion, operator configuration
    B, H, W, heads, D = 64, 56, 56, 6, 16
    L, C = H * W, heads * D
    qr = torch.randn(B, 4, L, C, device=device, generator=g).to(torch.bfloat16)
    qo, inv = _qnorm_forward(qr, heads, D, want_inv=True)
    gq = torch.randn_like(qo)
    rq = ref_mod("vhref_qnorm_bf16")
    add("qnorm backward", [B, 4, L, C], lambda: qnorm_backward(gq, qo, inv, heads, D, torch.bfloat16),
        nbytes=qo.numel() * (4 + 4 + 2) + inv.numel() * 4,
        ref_fn=(lambda: rq.visionhope_qnorm_backward(gq, qo, inv, heads, D, True)) if rq else None)
    del qo, gq
    y = torch.randn(B, 4, heads, L, D, device=device, generator=g).to(torch.bfloat16)
    xx = torch.randn(B, 4, heads, L, D, device=device, generator=g).to(torch.bfloat16)
    skip = torch.randn(C, device=device, generator=g)
    scale = torch.randn(4, C, device=device, generator=g)
    gout = torch.randn(B, C, H, W, device=device, generator=g)
    rd = ref_mod("vhref_dirfuse_bf16")
    add("dirfuse backward (NCHW grad)", [B, 4, heads, L, D],
        lambda: postprocess_backward(gout, y, xx, skip, scale, H, W),
        nbytes=gout.numel() * 4 + y.numel() * 2 * 4,
        ref_fn=(lambda: rd.visionhope_postprocess_scale_backward(gout, y, xx, skip, scale, H, W, False, False, 128))
        if rd else None)
    del y, xx, gout
    try:
        from oracle import refmodel
        refmodel.load("native")
        import visionhope.models.srnl_core.chunk as ref_chunk
        import visionhope.utils.layer_norm_cuda as ref_ln
        import visionhope.utils.residual as ref_res
    except Exception:
        ref_chunk = ref_ln = ref_res = None
    # LayerNorm and GRN, GRN/LN configuration (large shape)
    Bn, Hn, Wn, Cn = 128, 56, 56, 96
    x = torch.randn(Bn, Cn, Hn, Wn, device=device, generator=g).contiguous(memory_format=torch.channels_last)
    xr = x.permute(0, 2, 3, 1).reshape(-1, Cn)
    w = torch.randn(Cn, device=device, generator=g)
    bb = torch.randn(Cn, device=device, generator=g)
    _, mean, rstd = layernorm_rows(xr, w, bb, 1e-6, want_stats=True)
    gy = torch.randn_like(xr)
    # The reference's Triton backward (utils/layer_norm_cuda.py:150-185) called on the same
    # saved tensors through its autograd Function's backward.
    ln_ctx = types.SimpleNamespace(saved_tensors=(x, w, mean, rstd), shape=(Bn, Cn, Hn, Wn))
    gy4 = gy.view(Bn, Hn, Wn, Cn).permute(0, 3, 1, 2)
    add("layernorm backward", [Bn, Hn, Wn, Cn], lambda: layernorm_rows_backward(gy, xr, w, mean, rstd),
        nbytes=xr.numel() * 4 * 3,
        ref_fn=(lambda: ref_ln._VisionHOPELayerNorm2dFunction.backward(ln_ctx, gy4)) if ref_ln else None)
    # LayerScale residual add (fp32 residual, bf16 branch as under autocast) and its backward
    from visionhope_b200.utils.residual import residual_add_backward, residual_add_forward
    br = torch.randn(Bn, Cn, Hn, Wn, device=device, generator=g).to(torch.bfloat16).contiguous(
        memory_format=torch.channels_last)
    lsg = torch.randn(Cn, 1, 1, device=device, generator=g)
    keep = torch.ones(Bn, device=device)
    rs_ctx = types.SimpleNamespace(save_for_backward=lambda *t: None, saved_tensors=(br, lsg, keep),
                                   shape=(Bn, Cn, Hn, Wn))
    add("residual add forward", [Bn, Hn, Wn, Cn], lambda: residual_add_forward(x, br, lsg, keep),
        nbytes=x.numel() * (4 + 2 + 4),
        ref_fn=(lambda: ref_res._VisionHOPEResidualFunction.forward(rs_ctx, x, br, lsg, keep)) if ref_res else None)
    gres = torch.randn_like(x)
    add("residual add backward", [Bn, Hn, Wn, Cn], lambda: residual_add_backward(gres, br, lsg, keep),
        nbytes=x.numel() * (4 + 2 + 2),
        ref_fn=(lambda: ref_res._VisionHOPEResidualFunction.backward(rs_ctx, gres)) if ref_res else None)
    del br, gres
    gamma = torch.randn(Cn, device=device, generator=g) * 0.5
    _, gx, invd = grn_forward(x, gamma, bb, 1e-6, want_stats=True)
    gyn = torch.randn_like(x)
    rg = ref_mod("vhref_grn")

    def ref_grn():
        s = torch.empty((Bn, Cn), device=device)
        dg, db = torch.empty((Bn, Cn), device=device), torch.empty((Bn, Cn), device=device)
        ssg = torch.empty((Bn,), device=device)
        dx = torch.empty_like(x)
        dgam, dbet = torch.empty(Cn, device=device), torch.empty(Cn, device=device)
        rg.grn_backward_cuda(gyn, x, gamma, gx, invd, s, dg, db, ssg, dx, dgam, dbet)

    add("grn backward", [Bn, Hn, Wn, Cn], lambda: grn_backward(gyn, x, gamma, gx, invd),
        nbytes=x.numel() * 4 * 3, ref_fn=ref_grn if rg else None)
    del x, xr, gy, gyn
    # SRNL recurrence backward, operator configuration
    mems = [torch.randn(4, heads, D, D, device=device, generator=g) * 0.3 for _ in range(3)]
    mems += [torch.randn(4, heads, D, device=device, generator=g) * 0.6 for _ in range(2)]
    xs = torch.randn(B, 4, heads, L, D, device=device, generator=g).to(torch.bfloat16)
    qs = torch.randn(B, 4, L, C, device=device, generator=g).to(torch.bfloat16)
    gys = torch.randn(B, 4, heads, L, D, device=device, generator=g)
    chains = B * 4 * heads

    def ref_train():
        # The reference's own training step of the recurrence (chunk.py SRNLRawQueryFunction on its
        # kernels: srnl_forward_qraw saving its buffers, then srnl_backward_qraw), against which
        # ours is timed as forward + backward too.
        leaves = [t.detach().requires_grad_(True) for t in (*mems, xs, qs)]
        ref_chunk.srnl_raw_query(*leaves, W, heads, D).backward(gys.to(torch.bfloat16))

    def ours_train():
        from visionhope_b200.srnl_core.chunk import srnl_raw_query
        leaves = [t.detach().requires_grad_(True) for t in (*mems, xs, qs)]
        srnl_raw_query(*leaves, W, heads, D).backward(gys.to(torch.bfloat16))

    add("srnl recurrence backward (raw queries, chunk 56)", [B, 4, heads, L, D],
        lambda: sequence_backward(mems, xs, qs, [W] * 4, gys, q_normalized=False),
        units=chains * L, unit_name="chain_tokens_per_s")
    add("srnl recurrence forward + backward (autograd, raw queries, chunk 56)", [B, 4, heads, L, D], ours_train,
        units=chains * L, unit_name="chain_tokens_per_s", ref_fn=ref_train if ref_chunk is not None else None)
    del xs, qs, gys
    out = {"backward": rows, "peak_hbm_gbs": hbm, "peak_source": "MEASURED_PEAKS.json hbm_gbs",
           "consts": list(recurrence_constants_tuple())}
    try:
        out["training_step"] = training_step_compare(device, iters)
    except Exception as exc:  # the reference's modules are optional here
        out["training_step"] = {"unavailable": f"{type(exc).__name__}: {exc}"}
    return out


def training_step_compare(device, iters, batch=64):
    """One training step (forward and backward, no optimizer) of the reference's own
    VisionHOPE-T (models/factory.py, unchanged) at 224 x 224 under bf16 autocast, channels-last,
    in training mode: once on the reference's kernels ("native") and once with its kernel-owning
    modules bound to this package ("dropin").  The same seeded weights and input; the loss is
    the sum of the logits.  Every operator takes the ordinary path (training mode), so the step
    runs query normalization, the SRNL recurrence, direction fusion, LayerNorm, GRN and the
    residual adds forward and backward on the library under test."""
    from oracle import refmodel

    res = {"model": "visionhope_tiny", "batch": batch, "image": [224, 224],
           "precision": "bf16 autocast, fp32 params", "mode": "train (drop path on), forward + backward"}
    for mode in ("native", "dropin"):
        ref = refmodel.load(mode)
        torch.manual_seed(0)
        model = ref.create_model("visionhope_tiny").to(device).train().to(memory_format=torch.channels_last)
        x = torch.randn(batch, 3, 224, 224, device=device).contiguous(memory_format=torch.channels_last)

        def step():
            model.zero_grad(set_to_none=True)
            with torch.autocast("cuda", dtype=torch.bfloat16):
                logits = model(x)
            logits.float().sum().backward()

        ms, _ = _time_calls(step, iters, lambda: None)
        res[f"{mode}_ms"] = ms
        res[f"{mode}_images_per_s"] = batch / (ms * 1e-3)
        del model, x
        torch.cuda.empty_cache()
    res["speedup_vs_reference"] = res["native_ms"] / res["dropin_ms"]
    return res


def roofline_depthwise(device, iters=10):
    """The block's depthwise kernels and the statistics-fed GRN at VisionHOPE-T's shapes, batch
    256 (the bench workload), each timed alone: achieved HBM GB/s of the algorithmic bytes
    against the measured copy bandwidth.  Per element: gelu (FFN, 3x3, with the GRN sums)
    reads bf16 x and writes bf16 y (4 B); gate (7x7) also reads the bf16 gate (6 B); bias (5x5)
    4 B; resid_add (cpe, 3x3) reads fp32 x and the bf16 pending branch and writes fp32 (10 B);
    grn_apply (bf16 in and out, sums from the gelu call) 4 B; grn is the standalone cluster
    kernel on the same tensor (4 B); gate + position (the gated 7x7 and the 5x5 position term
    in one call, 14x14 and 7x7 images) reads x and the gate and writes both outputs (8 B)."""
    from visionhope_b200.utils.dwconv import depthwise_fused
    from visionhope_b200.utils.grn_cuda import grn_apply, grn_forward

    peaks = json.loads((ROOT / "MEASURED_PEAKS.json").read_text()) if (ROOT / "MEASURED_PEAKS.json").exists() else {}
    hbm = peaks.get("hbm_gbs")
    flush = l2_flush(device)
    g = torch.Generator(device=device).manual_seed(5)
    B, bf = 256, torch.bfloat16
    rows = []
    with torch.inference_mode():
        for H, emb, mix in ((56, 64, 32), (28, 128, 64), (14, 256, 128), (7, 512, 256)):
            def img(C, dt):
                return torch.randn(B, C, H, H, device=device, generator=g).to(dt).contiguous(
                    memory_format=torch.channels_last)

            def conv(C, k):
                return torch.nn.Conv2d(C, C, k, padding=k // 2, groups=C).to(device)

            h, cg = img(4 * emb, bf), conv(4 * emb, 3)
            y, sums = depthwise_fused(h, cg, "gelu", with_sumsq=True)
            gam = torch.randn(4 * emb, device=device, generator=g) * 0.02
            bet = torch.randn(4 * emb, device=device, generator=g) * 0.02
            xl, gate, cl, cp = img(mix, bf), img(mix, bf), conv(mix, 7), conv(mix, 5)
            xr, pend, cc = img(emb, torch.float32), img(emb, bf), conv(emb, 3)
            cases = (("dwconv gelu + GRN sums (3x3)", h, 4, lambda: depthwise_fused(h, cg, "gelu", with_sumsq=True)),
                     ("grn_apply", y, 4, lambda: grn_apply(y, sums, gam, bet, 1e-6, out_dtype=bf)),
                     ("grn (cluster)", y, 4, lambda: grn_forward(y, gam, bet, 1e-6, out_dtype=bf)),
                     ("dwconv gate (7x7)", xl, 6, lambda: depthwise_fused(xl, cl, "gate", gate=gate)),
                     ("dwconv bias (5x5)", xl, 4, lambda: depthwise_fused(xl, cp, "bias")),
                     ("dwconv resid_add (3x3, fp32)", xr, 10, lambda: depthwise_fused(xr, cc, "resid", addend=pend)))
            if H in (14, 7):  # whole images per CTA: the gated 7x7 and the position 5x5 in one call
                def gate_pos():
                    with torch.autocast("cuda", dtype=bf):  # the mode's eligibility rule asks for it
                        return depthwise_fused(xl, cl, "gate_pos", gate=gate, pos_conv=cp)
                cases += (("dwconv gate + position (7x7, 5x5)", xl, 8, gate_pos),)
            for name, t, bpe, fn in cases:
                ms, launches = _time_calls(fn, iters, flush)
                nbytes = t.numel() * bpe
                gbs = nbytes / (ms * 1e-3) / 1e9
                rows.append({"kernel": name, "shape": [B, H, H, t.shape[1]], "ms": ms, "alg_bytes": nbytes,
                             "achieved_gbs": gbs, "launches": launches,
                             "frac_of_measured_hbm": gbs / hbm if hbm else None})
    return {"depthwise_roofline": rows, "peak_hbm_gbs": hbm, "peak_source": "MEASURED_PEAKS.json hbm_gbs"}


def run_ours(args, world, rank, local):
    device = torch.device("cuda", local)
    torch.cuda.set_device(device)
    from visionhope_b200 import _lib

    model = build_model(args.model, device)
    sync_model(model, world)
    bus_ids = job_bus_ids(device, world)
    static_in = rank_inputs(args.batch, rank, device)

    def fwd():
        with torch.autocast("cuda", dtype=torch.bfloat16):
            if args.task == "dense":
                return list(model.forward_intermediates(static_in))
            return [model(static_in)]

    with torch.inference_mode():
        for _ in range(2):
            out = fwd()
        torch.cuda.synchronize()
        c0 = _lib.launch_count
        graph = torch.cuda.CUDAGraph()
        with torch.cuda.graph(graph):
            static_outs = fwd()
        launches_per_step = _lib.launch_count - c0
        gathered = [[torch.empty_like(o) for _ in range(world)] for o in static_outs] if world > 1 else None
        flush = l2_flush(device)  # evicts L2 between steps, outside the timed events

        def gather():
            for g_list, o in zip(gathered, static_outs):
                dist.all_gather(g_list, o)

        def step():
            graph.replay()
            if world > 1:
                gather()

        for _ in range(args.warmup):
            step()
        evs = [(torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True))
               for _ in range(args.steps)]
        with ClockSampler(enabled=rank == 0, interval_ms=50 if world == 1 else 100) as clk:
            # The barrier comes after the sampler has started (rank 0 waits for its first
            # sample): ranks that entered the timed loop earlier would otherwise time their
            # all-gather waiting for rank 0.
            torch.cuda.synchronize()
            if world > 1:
                dist.barrier()
            torch.cuda.synchronize()
            for a, b in evs:
                flush()
                a.record()
                step()
                b.record()
            torch.cuda.synchronize()
        if world > 1:
            dist.barrier()
        torch.cuda.synchronize()
        ms = sum(a.elapsed_time(b) for a, b in evs) / args.steps
        ms_max = max_over_ranks(ms, device, world)
        clocks = clk.summary(bus_ids)

        # ---- end to end: pinned host batch in, logits out, every step inside the timed run ----
        # A serving pipeline: batch i+1 crosses PCIe on a copy stream into a staging buffer
        # while batch i runs; each step then moves its batch from staging into the graph's
        # input (device to device) and copies its logits back to pinned host memory.  The
        # timed region spans the whole run, from the first host-to-device copy to the last
        # logits copy, so all K copies in and out are inside it.
        host_in = torch.randn(args.batch, 3, *IMG_HW, generator=torch.Generator().manual_seed(3 + rank)
                              ).contiguous(memory_format=torch.channels_last).pin_memory()
        host_outs = [torch.empty(o.shape, dtype=o.dtype).pin_memory() for o in static_outs]
        staging = torch.empty_like(static_in)
        copy_stream = torch.cuda.Stream(device)
        main = torch.cuda.current_stream(device)

        def e2e_run(k):
            copied, freed = torch.cuda.Event(), torch.cuda.Event()
            copy_stream.wait_stream(main)
            with torch.cuda.stream(copy_stream):
                staging.copy_(host_in, non_blocking=True)
                copied.record()
            # No L2 eviction inside this timed run: every step's batch is a fresh copy from the host
            # and every forward moves far more than L2 through the cache.
            for i in range(k):
                main.wait_event(copied)
                static_in.copy_(staging, non_blocking=True)
                freed.record()
                if i + 1 < k:
                    copy_stream.wait_event(freed)
                    with torch.cuda.stream(copy_stream):
                        staging.copy_(host_in, non_blocking=True)
                        copied.record()
                graph.replay()
                if world > 1:
                    gather()
                for h, o in zip(host_outs, static_outs):
                    h.copy_(o, non_blocking=True)

        e2e_run(2)
        torch.cuda.synchronize()
        if world > 1:
            dist.barrier()
        a, b = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        a.record()
        e2e_run(args.steps)
        b.record()
        torch.cuda.synchronize()
        e2e_ms = max_over_ranks(a.elapsed_time(b) / args.steps, device, world)
        if not all(torch.isfinite(h).all() for h in host_outs):
            raise RuntimeError("non-finite outputs")

        roof = ref_cmp = None
        if rank == 0:
            roof = roofline_scan(args, device, args.steps)
            if world == 1:
                roof["kernels"] = per_kernel_rooflines(args, device)
                ref_cmp = ref_kernel_compare(device, args.batch) if args.model == "visionhope_tiny" else None
        del graph
    result = None
    if rank == 0:
        result = {
            "metric": metric_name(args), "value": world * args.batch * 1000.0 / ms_max, "unit": UNIT,
            "n_gpus": world, "steps": args.steps, "warmup": args.warmup, "ms_per_step": ms_max,
            "higher_is_better": True, "scaling": "weak", "vs_baseline": None, "dtype": "bf16",
            "data": "synthetic N(0,1) images, random-init weights (seed 3)",
            "config": config(args, world),
            "e2e": {"value": world * args.batch * 1000.0 / e2e_ms, "unit": UNIT,
                    "h2d_bytes_per_step": host_in.numel() * host_in.element_size(),
                    "d2h_bytes_per_step": sum(h.numel() * h.element_size() for h in host_outs),
                    "ms_per_step": e2e_ms,
                    "pipeline": "host-to-device copy of batch i+1 on a copy stream overlaps the forward of "
                                "batch i; timed from the first copy in to the last output copy out"},
            "ref_kernel": ref_cmp,
            "gpu_launches": launches_per_step * args.steps,
            "gpu_launches_per_step": launches_per_step,
            "roofline": roof, "clocks": clocks,
        }
    return result


def main():
    args = parse()
    world, rank, local = dist_env()
    if world > 1:
        from datetime import timedelta

        backend = "nccl" if args.impl == "ours" else "gloo"
        if args.impl == "ours":
            torch.cuda.set_device(local)
        dist.init_process_group(backend, timeout=timedelta(seconds=300))
    try:
        if args.impl == "reference":
            if rank != 0:
                return
            try:
                ips, times, cores, sample = run_cpu(args, args.steps, args.warmup)
            except FileNotFoundError as exc:  # the reference package was not staged with the repo
                print(json.dumps({"impl": "reference", "unavailable": str(exc)}), flush=True)
                return
            line = {"metric": metric_name(args), "value": ips, "unit": UNIT, "n_gpus": world, "steps": args.steps,
                    "warmup": args.warmup, "ms_per_step": 1000.0 * statistics.mean(times),
                    "higher_is_better": True, "scaling": "weak", "vs_baseline": None, "dtype": "f32",
                    "data": "synthetic N(0,1) images, random-init weights (seed 3)", "impl": "reference",
                    "config": dict(config(args, world), workload=f"{args.model} forward on host CPU "
                                   f"(reference stand-in), {args.cpu_sample} images/step"),
                    "cpu_baseline": {"value": ips, "unit": UNIT, "cores": cores, "kind": "port",
                                     "sample": sample},
                    "e2e": {"value": ips, "unit": UNIT, "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0}}
            print(json.dumps(line), flush=True)
            return
        if args.only_scan or args.only_norms or args.only_depthwise or args.only_backward:
            if rank == 0:
                torch.cuda.set_device(local)
                dev = torch.device("cuda", local)
                if args.only_scan:
                    res = {"roofline": roofline_scan(args, dev, args.steps),
                           "kernels": per_kernel_rooflines(args, dev),
                           "ref_kernel": ref_kernel_compare(dev, args.batch)}
                elif args.only_norms:
                    res = roofline_norms(dev, args.steps)
                elif args.only_backward:
                    res = roofline_backward(dev, max(args.steps, 3))
                else:
                    res = roofline_depthwise(dev, args.steps)
                print(json.dumps(res), flush=True)
            return
        result = run_ours(args, world, rank, local)
        if rank == 0:
            if world == 1 and not args.no_cpu_baseline:
                try:
                    ips, times, cores, sample = run_cpu(args, steps=5, warmup=1)
                    result["cpu_baseline"] = {"value": ips, "unit": UNIT, "cores": cores, "kind": "port",
                                              "sample": sample}
                except FileNotFoundError as exc:
                    result["cpu_baseline"] = {"value": None, "unavailable": str(exc)}
            print(json.dumps(result), flush=True)
    finally:
        if world > 1 and dist.is_initialized():
            dist.destroy_process_group()


if __name__ == "__main__":
    main()

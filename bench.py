"""Benchmark: FPN-neck images/s on B200 (R50 800x1216, bf16, batch 2 per GPU).

  python bench.py [--gpus N] [--steps K] [--warmup W] [--impl ours|reference]
  python bench.py --train [--dtype bf16|fp16] ...   (training step: forward + backward)

One step = one forward of the whole neck (4 fused laterals + 4 implicit-GEMM 3x3
convs + P6) over one batch.  Multi-GPU (torchrun, one process per GPU): every
rank runs its own batch slice with no collective on the data path (weak
scaling); timing is a barrier-bracketed CUDA-event window, max over ranks.

Prints ONE JSON line (rank 0).  Keys beyond the base contract:
  e2e         same metric through the public API (UnifiedFPN.forward) with the
              inputs copied from pinned host memory and P2..P6 copied back each step
  roofline    the dominant kernel (P2 3x3 implicit GEMM) timed live with CUDA events
  cpu_baseline  the CPU oracle neck (fp32 torch CPU, all host threads) on a bounded sample
  clocks      nvidia-smi samples taken during the timed window
  extra       (N = 1) the other configurations' per-GPU shards timed after the headline:
              e4m3 R50 640x640 16 images, bf16 R50 1024x1024 8 images, bf16 Swin 1333x800
              8 images, and the fp32 single-level lateral + top-down op
  per_rank_ms_per_step  (N > 1) every rank's step time

--train times the neck's training step instead (its own JSON line, metric METRIC_TRAIN): the
forward of unified_fpn.FPNNeck (fp32 master weights, 16-bit kernels) and the backward to every
input, weight and bias gradient, for seeded gradients of P2..P6; gradients are reset to None
between steps (no accumulation adds).  Not the headline metric.
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
sys.path.insert(0, str(ROOT))
sys.path.insert(0, str(ROOT / "-unifiedfpn_b200"))

import torch  # noqa: E402

METRIC = "FPN-neck images/sec, R50 800×1216 bf16 @1/2/4/8 B200; % of roofline"
METRIC_FP8 = "FPN-neck images/sec, FP8 (e4m3) R50 640×640, 16 images/GPU @1/2/4/8 B200; % of roofline"
METRIC_TRAIN = "FPN-neck training steps (forward + backward, all gradients) images/sec, R50 800×1216"
R50_CHANNELS = (256, 512, 1024, 2048)
# Library kernels per training step (FPNNeck forward + backward with gradients for P2..P6):
# one launch preparing every weight layout of the step; forward per level: lateral (with the
# fused top-down add), 3x3 (+P6); backward per level: 3x3 input gradient, weight-gradient GEMM
# (bias gradient included) + its reduction; lateral input gradient (one launch for all channel
# slices), weight-gradient GEMM + reduction; the P6 adjoint once and the top-down adjoint for
# P3, P4, P5.
TRAIN_LAUNCHES = 1 + 4 * 2 + 4 * 3 + 4 * 3 + 1 + 3


def level_sizes(h, w):
    return [(-(-h // s), -(-w // s)) for s in (4, 8, 16, 32)]


def neck_flops(batch, chans, sizes):
    f = 0.0
    for c, (h, w) in zip(chans, sizes):
        px = batch * h * w
        f += 2.0 * px * 256 * c + 2.0 * px * 256 * 256 * 9
    return f


def neck_bytes(batch, chans, sizes, esz, out_esz=None):
    """Compulsory HBM bytes: read C2..C5 and weights (esz), write P2..P6 (out_esz)."""
    out_esz = esz if out_esz is None else out_esz
    b = 0.0
    for c, (h, w) in zip(chans, sizes):
        px = batch * h * w
        b += px * c * esz + px * 256 * out_esz + (256 * c + 9 * 256 * 256) * esz
    h5, w5 = sizes[3]
    b += batch * ((h5 + 1) // 2) * ((w5 + 1) // 2) * 256 * out_esz
    return b


def rank_images(rank, per_rank):
    """Global image indices of a rank's batch slice (contiguous, per_rank images each)."""
    return list(range(rank * per_rank, (rank + 1) * per_rank))


def job_throughput(ms_local, images_local, world, device=None):
    """Whole-job timing across ranks: (slowest rank's ms, images processed by all ranks).
    The only collectives of a run; they sit outside the timed window."""
    if world <= 1:
        return float(ms_local), int(images_local)
    import torch.distributed as dist
    t = torch.tensor([float(ms_local)], dtype=torch.float64, device=device)
    n = torch.tensor([float(images_local)], dtype=torch.float64, device=device)
    dist.all_reduce(t, op=dist.ReduceOp.MAX)
    dist.all_reduce(n, op=dist.ReduceOp.SUM)
    return float(t.item()), int(round(n.item()))


def per_rank_ms(ms_local, world, device=None):
    """Every rank's step time (ms), gathered outside the timed window (N > 1: names the
    straggler behind the max-over-ranks figure)."""
    if world <= 1:
        return None
    import torch.distributed as dist
    t = torch.tensor([float(ms_local)], dtype=torch.float64, device=device)
    out = [torch.zeros_like(t) for _ in range(world)]
    dist.all_gather(out, t)
    return [round(float(x.item()), 5) for x in out]


def time_steps(fn, steps, warmup=3, stream=None):
    """ms per call of fn() (CUDA events on the current stream, after warm-up)."""
    for _ in range(warmup):
        fn()
    torch.cuda.synchronize()
    e0 = torch.cuda.Event(enable_timing=True)
    e1 = torch.cuda.Event(enable_timing=True)
    e0.record(stream)
    for _ in range(steps):
        fn()
    e1.record(stream)
    torch.cuda.synchronize()
    return e0.elapsed_time(e1) / steps


def cupti_timeline(fwd, n=14, skip=3, gap_us=15.0):
    """Per-kernel device timeline of the concurrent schedule: torch.profiler (CUPTI) over n
    forwards, each followed by a synchronize so that forwards separate by an idle gap (one of
    more than gap_us starts a new forward); the first `skip` are dropped.  Per kernel (in start order within a forward): median start,
    end and duration in us from the forward's first kernel start, and the median forward
    span.  None if the profiler is unavailable (for instance CUPTI held by another tool)."""
    import statistics
    import tempfile
    try:
        from torch.profiler import ProfilerActivity, profile
        with profile(activities=[ProfilerActivity.CUDA]) as prof:
            for i in range(n):
                fwd(i)
                torch.cuda.synchronize()
        with tempfile.TemporaryDirectory() as td:
            path = os.path.join(td, "trace.json")
            prof.export_chrome_trace(path)
            with open(path) as f:
                ev = [e for e in json.load(f)["traceEvents"] if e.get("cat") == "kernel"]
    except Exception:
        return None
    ev.sort(key=lambda e: e["ts"])
    fwds, end = [], None
    for e in ev:  # a gap of > gap_us with no kernel running separates forwards
        if end is None or e["ts"] > end + gap_us:
            fwds.append([])
        fwds[-1].append(e)
        end = max(end or 0.0, e["ts"] + e["dur"])
    fwds = fwds[skip:]
    if not fwds:
        return None
    k = statistics.mode(len(f) for f in fwds)
    fwds = [f for f in fwds if len(f) == k]
    rows = []
    for j in range(k):
        name = fwds[0][j]["name"]
        short = name.replace("(anonymous namespace)::", "").split("(")[0].replace(
            "void ", "").replace("ufpn::", "")
        st = [f[j]["ts"] - f[0]["ts"] for f in fwds]
        du = [f[j]["dur"] for f in fwds]
        rows.append({"kernel": short[:80], "start_us": round(statistics.median(st), 1),
                     "end_us": round(statistics.median(s + d for s, d in zip(st, du)), 1),
                     "us": round(statistics.median(du), 1)})
    span = statistics.median(max(e["ts"] + e["dur"] for e in f) - f[0]["ts"] for f in fwds)
    return {"forward_us": round(span, 1), "forwards": len(fwds), "kernels": rows,
            "what": "CUPTI kernel records (torch.profiler) of the concurrent schedule, each forward "
                    "followed by a synchronize; median over forwards; a kernel's duration includes "
                    "the time it waits for SMs held by kernels of other streams and, under a "
                    "programmatic launch, for the kernel before it"}


def extra_workloads(dev, peaks):
    """The other configurations' per-GPU shards, timed in the same run (not the headline):
    each the whole neck through UnifiedFPN on device-resident inputs rotating over 2 sets,
    with its own neck roofline (slower of FLOPs at the sustained tensor peak and compulsory
    bytes at HBM peak); the fp32 single-level op with its GB/s and FFMA fraction."""
    import unified_fpn as U
    res = {}
    gen = torch.Generator(device=dev)
    gen.manual_seed(7)

    def neck(name, chans, sizes, batch, dtype, steps):
        fp8 = dtype == torch.float8_e4m3fn
        sets, scs = [], []
        for _ in range(2):
            if fp8:
                qs = [U.quantize_fp8(torch.randn(batch, c, h, w, device=dev, generator=gen).contiguous(
                    memory_format=torch.channels_last)) for c, (h, w) in zip(chans, sizes)]
                sets.append([q for q, _ in qs])
                scs.append(torch.cat([sc for _, sc in qs]))
            else:
                sets.append([torch.randn(batch, c, h, w, device=dev, generator=gen).to(dtype)
                             .contiguous(memory_format=torch.channels_last) for c, (h, w) in zip(chans, sizes)])
                scs.append(None)
        fpn = U.UnifiedFPN(device=dev)
        outs = [fpn(sets[i], return_p6=True, input_scales=scs[i]) for i in range(2)]
        it = [0]

        def step():
            i = it[0] % 2
            it[0] += 1
            fpn(sets[i], return_p6=True, out=outs[i], input_scales=scs[i])
        ms = time_steps(step, steps, warmup=4)
        if fpn.device_status() != 0:
            raise RuntimeError(f"{name}: device pipeline timeout")
        mult = 2.0 if fp8 else 1.0
        esz = 1 if fp8 else 2
        f_all = neck_flops(batch, chans, sizes)
        b_all = neck_bytes(batch, chans, sizes, esz, 2)
        t_roof = max(f_all / (peaks["bf16_tflops_sustained"] * mult * 1e12), b_all / (peaks["hbm_gbs"] * 1e9))
        res[name] = {"images_per_s": round(batch * 1e3 / ms, 1), "ms_per_step": round(ms, 4),
                     "batch": batch, "levels": [[batch, c, h, w] for c, (h, w) in zip(chans, sizes)],
                     "dtype": "e4m3" if fp8 else str(dtype).replace("torch.", ""),
                     "tflops": round(f_all / (ms * 1e-3) / 1e12, 1),
                     "neck_frac_of_roofline": round(t_roof * 1e3 / ms, 4)}
        del fpn, sets, outs
        torch.cuda.empty_cache()

    swin = (128, 256, 512, 1024)
    neck("fp8_r50_640x640_16img", R50_CHANNELS, level_sizes(640, 640), 16, torch.float8_e4m3fn, 20)
    neck("bf16_r50_1024x1024_8img", R50_CHANNELS, level_sizes(1024, 1024), 8, torch.bfloat16, 10)
    neck("bf16_swin_1333x800_8img", swin, [(200, 334), (100, 167), (50, 84), (25, 42)], 8, torch.bfloat16, 20)
    # single-level fused lateral + top-down add, fp32 NCHW (CUDA cores: TF32 would not meet 1e-4)
    x = torch.randn(1, 512, 64, 64, device=dev, generator=gen)
    c = torch.randn(1, 256, 32, 32, device=dev, generator=gen)
    w = torch.randn(256, 512, device=dev, generator=gen) * (2.0 / 512) ** 0.5
    b = torch.zeros(256, device=dev)
    ms = time_steps(lambda: U.fpn_lateral_conv(x, w, b, c), 50, warmup=5)
    flops = 2.0 * 64 * 64 * 256 * 512 + 9.0 * 64 * 64 * 256
    nbytes = (x.numel() + c.numel() + w.numel() + b.numel() + 256 * 64 * 64) * 4
    fp32_peak = U.get_peaks()["fp32_tflops"]
    res["fp32_lateral_topdown_512x64x64"] = {
        "us_per_call": round(ms * 1e3, 2), "gb_s": round(nbytes / (ms * 1e-3) / 1e9, 1),
        "hbm_frac": round(nbytes / (ms * 1e-3) / 1e9 / peaks["hbm_gbs"], 4),
        "ffma_tflops": round(flops / (ms * 1e-3) / 1e12, 2),
        "ffma_frac": round(flops / (ms * 1e-3) / 1e12 / fp32_peak, 4),
        "ffma_peak_src": "nominal 80 TFLOP/s fp32 (no measured fp32 peak on this pool)",
        "note": "includes one launch latency per call (a 14 MB op)"}
    return res


def e2e_ceiling(dev, h2d_bytes, d2h_bytes, steps, images_per_step):
    """Plain pinned copies of the e2e line's bytes per step (host -> device and device -> host
    on two streams, overlapped as HostPipeline overlaps them), no compute: the images/s that
    host memory and PCIe allow this process."""
    hin = torch.empty(h2d_bytes, dtype=torch.uint8, pin_memory=True)
    hout = torch.empty(d2h_bytes, dtype=torch.uint8, pin_memory=True)
    din = torch.empty(h2d_bytes, dtype=torch.uint8, device=dev)
    dout = torch.empty(d2h_bytes, dtype=torch.uint8, device=dev)
    s_in, s_out = torch.cuda.Stream(dev), torch.cuda.Stream(dev)
    cur = torch.cuda.current_stream(dev)

    def run(k):
        ev = torch.cuda.Event()
        ev.record(cur)
        s_in.wait_event(ev)
        s_out.wait_event(ev)
        for _ in range(k):
            with torch.cuda.stream(s_in):
                din.copy_(hin, non_blocking=True)
            with torch.cuda.stream(s_out):
                hout.copy_(dout, non_blocking=True)
        for s in (s_in, s_out):
            e = torch.cuda.Event()
            e.record(s)
            cur.wait_event(e)
    run(2)
    torch.cuda.synchronize(dev)
    e0 = torch.cuda.Event(enable_timing=True)
    e1 = torch.cuda.Event(enable_timing=True)
    e0.record(cur)
    run(steps)
    e1.record(cur)
    torch.cuda.synchronize(dev)
    ms = e0.elapsed_time(e1)
    return ms, images_per_step * steps


def run_bandwidth_kernels(args, dev):
    """--kernels bandwidth: the standalone HBM-bound ops on maps larger than the 126 MB L2
    (bf16): the top-down upsample-add (NHWC: the merge kernel of the neck; NCHW) and P6 (NHWC,
    NCHW); per op the CUDA-event time of one call (after warm-up), algorithmic bytes (compulsory
    reads + writes) and GB/s against the measured HBM copy bandwidth.  One JSON line."""
    import unified_fpn as U
    peaks = measured_peaks()
    gen = torch.Generator(device=dev)
    gen.manual_seed(11)
    cl = torch.channels_last
    res = {}

    def run(name, fn, nbytes):
        ms = time_steps(fn, max(1, args.steps), warmup=max(3, args.warmup))
        res[name] = {"us": round(ms * 1e3, 1), "mb": round(nbytes / 1e6, 1),
                     "gb_s": round(nbytes / (ms * 1e-3) / 1e9, 0),
                     "frac_of_hbm": round(nbytes / (ms * 1e-3) / 1e9 / peaks["hbm_gbs"], 4)}

    c = torch.randn(4, 256, 200, 304, device=dev, generator=gen).to(torch.bfloat16)
    l = torch.randn(4, 256, 400, 608, device=dev, generator=gen).to(torch.bfloat16)
    nb = 2 * l.numel() * 2 + c.numel() * 2  # read lateral + coarse, write the sum
    cn, ln = c.contiguous(memory_format=cl), l.contiguous(memory_format=cl)
    run("upsample_add_nhwc_4x256x400x608", lambda: U.fpn_upsample_add(cn, ln), nb)
    run("upsample_add_nchw_4x256x400x608", lambda: U.fpn_upsample_add(c, l), nb)
    del c, l, cn, ln
    p5 = torch.randn(16, 256, 200, 304, device=dev, generator=gen).to(torch.bfloat16)
    p5c = p5.contiguous(memory_format=cl)
    nb6 = p5.numel() * 2 // 2  # read the even pixels of the even rows (1/4), write them (1/4)
    run("p6_nhwc_16x256x200x304", lambda: U.fpn_p6(p5c), nb6)
    run("p6_nchw_16x256x200x304", lambda: U.fpn_p6(p5), nb6)
    line = {"metric": "HBM-bound neck ops, GB/s on maps larger than L2 (bf16)", "value": None,
            "unit": "GB/s", "n_gpus": 1, "higher_is_better": True, "dtype": "bf16",
            "data": "synthetic (seeded N(0,1))", "peak_hbm_gbs": peaks["hbm_gbs"],
            "peak_src": peaks["src"], "kernels": res}
    line["value"] = min(v["gb_s"] for v in res.values())
    print(json.dumps(line), flush=True)
    return 0


def measured_peaks():
    p = ROOT / "MEASURED_PEAKS.json"
    if p.exists():
        d = json.loads(p.read_text())
        return {"hbm_gbs": d["hbm_gbs"], "bf16_tflops": d["bf16_tflops"],
                "bf16_tflops_sustained": d.get("bf16_tflops_sustained", d["bf16_tflops"]), "src": "measured"}
    return {"hbm_gbs": 6650.0, "bf16_tflops": 1590.0, "bf16_tflops_sustained": 1400.0, "src": "fallback"}


def profile_traffic(name):
    """dram bytes per launch from a committed ncu summary (profiles/<name>.txt), else None."""
    p = ROOT / "profiles" / f"{name}.txt"
    if not p.exists():
        return None
    for line in p.read_text().splitlines():
        if line.startswith("dram_bytes_per_launch:"):
            try:
                return float(line.split(":", 1)[1].split()[0])
            except ValueError:
                return None
    return None


class ClockSampler:
    """nvidia-smi clocks / throttle reasons sampled every 200 ms during the timed window."""

    FIELDS = ("index,clocks.sm,clocks.max.sm,power.draw,clocks_event_reasons.active,"
              "clocks_event_reasons.hw_slowdown,clocks_event_reasons.hw_thermal_slowdown,"
              "clocks_event_reasons.sw_thermal_slowdown,clocks_event_reasons.sw_power_cap")

    def __init__(self, gpu_index):
        self.gpu = gpu_index
        self.proc = None
        self.out = None

    def start(self):
        try:
            self.out = open(os.devnull, "w")
            self.proc = subprocess.Popen(
                ["nvidia-smi", "-i", str(self.gpu), f"--query-gpu={self.FIELDS}", "--format=csv,noheader,nounits",
                 "-lms", "200"], stdout=subprocess.PIPE, stderr=self.out, text=True)
        except OSError:
            self.proc = None

    def stop(self):
        if self.proc is None:
            return {"sm_mhz": None, "sm_max_mhz": None, "reasons": ["nvidia-smi unavailable"]}
        self.proc.terminate()
        try:
            text, _ = self.proc.communicate(timeout=5)
        except subprocess.TimeoutExpired:
            self.proc.kill()
            text, _ = self.proc.communicate()
        sm, mx, reasons = [], None, set()
        names = ["hw_slowdown", "hw_thermal_slowdown", "sw_thermal_slowdown", "sw_power_cap"]
        for line in text.strip().splitlines():
            parts = [p.strip() for p in line.split(",")]
            if len(parts) < 9:
                continue
            try:
                sm.append(float(parts[1]))
                mx = float(parts[2])
            except ValueError:
                continue
            for n, v in zip(names, parts[5:9]):
                if v.lower() == "active":
                    reasons.add(n)
        return {"sm_mhz": statistics.median(sm) if sm else None, "sm_max_mhz": mx,
                "reasons": sorted(reasons), "samples": len(sm)}


def cpu_baseline(seconds=12.0, image=(800, 1216)):
    """The CPU oracle neck (fp32, torch CPU, all host threads) on one image per iteration
    of the workload's image size."""
    from oracle import fpn_oracle as O
    torch.set_num_threads(os.cpu_count() or 1)
    sizes = level_sizes(*image)
    feats = O.make_features(1, R50_CHANNELS, sizes, seed=0)
    wts = O.make_weights(R50_CHANNELS, seed=1)
    with torch.no_grad():
        O.fpn_neck(feats, wts)  # warm-up
        n, t0 = 0, time.perf_counter()
        while True:
            O.fpn_neck(feats, wts)
            n += 1
            el = time.perf_counter() - t0
            if el >= seconds or n >= 50:
                break
    return {"value": n / el, "unit": "images/s", "cores": torch.get_num_threads(), "kind": "port",
            "sample": f"{n} x 1 image R50 {image[0]}x{image[1]} fp32 (torch CPU oracle neck, {el:.1f} s)"}


def run_reference(args, rank, world):
    """Reference arm: the reference's CPU path for this neck, i.e. the oracle port
    (the reference's own host code covers only the bilinear upsample; its neck
    does not build), on rank 0 with all host threads."""
    if rank != 0:
        return 0
    from oracle import fpn_oracle as O
    torch.set_num_threads(os.cpu_count() or 1)
    sizes = level_sizes(args.height, args.width)
    feats = O.make_features(1, R50_CHANNELS, sizes, seed=0)
    wts = O.make_weights(R50_CHANNELS, seed=1)
    with torch.no_grad():
        for _ in range(max(1, min(args.warmup, 1))):
            O.fpn_neck(feats, wts)
        steps = max(1, min(args.steps, 5))
        t0 = time.perf_counter()
        for _ in range(steps):
            O.fpn_neck(feats, wts)
        el = time.perf_counter() - t0
    v = steps / el
    line = {
        "impl": "reference", "metric": METRIC, "value": v, "unit": "images/s", "n_gpus": world,
        "steps": steps, "warmup": 1, "ms_per_step": el * 1e3 / steps, "higher_is_better": True,
        "scaling": "weak", "vs_baseline": None, "dtype": "f32", "data": "synthetic (seeded N(0,1) after ReLU clamp)",
        "config": {"workload": f"R50 FPN neck {args.height}x{args.width}, 1 image per step (bounded CPU sample)",
                   "global_batch": 1, "parallelism": "host threads"},
        "cpu_baseline": {"value": v, "unit": "images/s", "cores": torch.get_num_threads(), "kind": "port",
                         "sample": f"{steps} x 1 image R50 {args.height}x{args.width} fp32 torch CPU oracle neck"},
        "e2e": {"value": v, "unit": "images/s", "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0},
    }
    print(json.dumps(line), flush=True)
    return 0


def run_train(args, rank, world, local, dev):
    """Training-step throughput: FPNNeck forward + backward over 3 rotating input sets."""
    import torch.distributed as dist
    import unified_fpn as U

    dtype = {"bf16": torch.bfloat16, "fp16": torch.float16}[args.dtype]
    sizes = level_sizes(args.height, args.width)
    B = args.batch
    n_sets = 3
    gen = torch.Generator(device=dev)
    feats, grads = [], []
    for s in range(n_sets):
        gen.manual_seed(1000 * rank + s)
        feats.append([torch.randn(B, c, h, w, device=dev, generator=gen).clamp_min_(0).to(dtype)
                      .contiguous(memory_format=torch.channels_last).requires_grad_()
                      for c, (h, w) in zip(R50_CHANNELS, sizes)])
        out_sizes = list(sizes) + [((sizes[3][0] - 1) // 2 + 1, (sizes[3][1] - 1) // 2 + 1)]
        grads.append([torch.randn(B, 256, h, w, device=dev, generator=gen).to(dtype)
                      .contiguous(memory_format=torch.channels_last) for h, w in out_sizes])
    in_mb = sum(B * c * h * w * 2 for c, (h, w) in zip(R50_CHANNELS, sizes)) / 1e6
    neck = U.FPNNeck(R50_CHANNELS).to(dev)
    # graphs read their captured input buffers: each step copies its set into them (on the
    # device, inside the timed region, 117 MB per step)
    run = neck
    static = None
    if args.graph:
        static = [f.detach().clone().requires_grad_() for f in feats[0]]
        run = neck.make_graphed(static)

    def step(i):
        k = i % n_sets
        for p in neck.parameters():
            p.grad = None
        for f in feats[k] + (static or []):
            f.grad = None
        if static is not None:
            with torch.no_grad():
                for dst, src in zip(static, feats[k]):
                    dst.copy_(src)
            outs = run(static)
        else:
            outs = run(feats[k])
        torch.autograd.backward(outs, grads[k])

    for i in range(args.warmup):
        step(i)
    torch.cuda.synchronize(dev)
    if U.device_status() != 0:
        raise RuntimeError("device pipeline timeout during warm-up")
    stream = torch.cuda.current_stream(dev)
    e0 = torch.cuda.Event(enable_timing=True)
    e1 = torch.cuda.Event(enable_timing=True)
    clocks = ClockSampler(local)
    if world > 1:
        dist.barrier()
    torch.cuda.synchronize(dev)
    clocks.start()
    time.sleep(0.3)
    e0.record(stream)
    for i in range(args.steps):
        step(i)
    e1.record(stream)
    torch.cuda.synchronize(dev)
    if world > 1:
        dist.barrier()
    clk = clocks.stop()
    ms, images = job_throughput(e0.elapsed_time(e1), B * args.steps, world, dev)
    ms_per_step = ms / args.steps
    kernel_timeline = None
    if rank == 0 and world == 1 and not args.no_roofline:
        def spaced(i):  # (steps apart by > 1 ms of idle GPU; the forward-backward gap is less)
            step(i)
            time.sleep(0.003)
        kernel_timeline = cupti_timeline(spaced, gap_us=1000.0)
        if kernel_timeline is not None:
            kernel_timeline["step_us"] = kernel_timeline.pop("forward_us")
            kernel_timeline["steps"] = kernel_timeline.pop("forwards")
    peaks = measured_peaks()
    flops = 3.0 * neck_flops(B, R50_CHANNELS, sizes)  # forward + input and weight gradients
    achieved = flops / (ms_per_step * 1e-3) / 1e12
    if rank == 0:
        line = {
            "metric": METRIC_TRAIN, "value": round(images / (ms / 1e3), 2), "unit": "images/s",
            "n_gpus": world, "steps": args.steps, "warmup": args.warmup,
            "ms_per_step": round(ms_per_step, 5), "higher_is_better": True, "scaling": "weak",
            "vs_baseline": None, "dtype": args.dtype,
            "data": "synthetic (seeded N(0,1) after ReLU clamp; seeded N(0,1) output gradients; "
                    "random Kaiming-normal fp32 master weights)",
            "config": {"workload": f"R50 FPN neck training step {args.height}x{args.width}, {B} images/GPU, "
                                   f"{args.dtype} NHWC, gradients of every input, weight and bias"
                                   + (", replayed as CUDA graphs (inputs copied into the captured "
                                      "buffers each step)" if args.graph else ""),
                       "global_batch": B * world, "per_gpu_batch": B,
                       "l2": f"inputs rotate over {n_sets} sets ({n_sets} x {in_mb:.0f} MB) > 126 MB L2",
                       "parallelism": f"dp{world} batch shards (gradients not reduced)"},
            "clocks": clk, "gpu_launches": TRAIN_LAUNCHES * args.steps,
            "roofline": {"bound": "tensor", "achieved": round(achieved, 1),
                         "peak": peaks["bf16_tflops_sustained"], "unit": "TFLOP/s",
                         "frac": round(achieved / peaks["bf16_tflops_sustained"], 4),
                         "flops_per_step": flops, "peak_source": peaks["src"] + " (sustained)",
                         "traffic": None},
            "device_status": U.device_status(),
        }
        if kernel_timeline is not None:
            line["kernel_timeline"] = kernel_timeline
        print(json.dumps(line), flush=True)
    if world > 1:
        dist.barrier()
        dist.destroy_process_group()
    return 0


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=50)
    ap.add_argument("--warmup", type=int, default=5)
    ap.add_argument("--impl", choices=["ours", "reference"], default="ours")
    ap.add_argument("--batch", type=int, default=None,
                    help="images per GPU (default 2; 16 for e4m3)")
    ap.add_argument("--height", type=int, default=None, help="default 800 (640 for e4m3)")
    ap.add_argument("--width", type=int, default=None, help="default 1216 (640 for e4m3)")
    ap.add_argument("--dtype", choices=["bf16", "fp16", "e4m3"], default="bf16",
                    help="e4m3: the FP8 neck on e4m3 inputs (bf16 outputs), R50 640x640, "
                         "16 images/GPU by default")
    ap.add_argument("--no-cpu-baseline", action="store_true")
    ap.add_argument("--no-e2e", action="store_true")
    ap.add_argument("--no-roofline", action="store_true")
    ap.add_argument("--no-extra", action="store_true",
                    help="skip the other configurations' shards timed after the headline")
    ap.add_argument("--schedule", choices=["fused", "split", "serial"], default="split",
                    help="one persistent neck kernel, per-level kernels on two streams, or the "
                         "per-level kernels one after the other on one stream")
    ap.add_argument("--train", action="store_true",
                    help="time the training step (FPNNeck forward + backward) instead")
    ap.add_argument("--kernels", choices=["bandwidth"], default=None,
                    help="bandwidth: time the standalone HBM-bound ops (upsample-add, P6) on "
                         "maps larger than L2 instead (one JSON line, GB/s per op)")
    ap.add_argument("--graph", action="store_true",
                    help="with --train: replay the step as CUDA graphs (FPNNeck.make_graphed)")
    args = ap.parse_args()
    if args.train and args.dtype == "e4m3":
        ap.error("--train runs on bf16 or fp16")
    fp8 = args.dtype == "e4m3"
    if args.batch is None:
        args.batch = 16 if fp8 else 2
    if args.height is None:
        args.height = 640 if fp8 else 800
    if args.width is None:
        args.width = 640 if fp8 else 1216
    if args.warmup < 3 and args.impl == "ours":
        args.warmup = 3

    world = int(os.environ.get("WORLD_SIZE", "1"))
    rank = int(os.environ.get("RANK", "0"))
    local = int(os.environ.get("LOCAL_RANK", "0"))
    if args.impl == "reference":
        return run_reference(args, rank, world)

    import torch.distributed as dist
    from datetime import timedelta
    torch.cuda.set_device(local)
    dev = torch.device("cuda", local)
    if world > 1:
        dist.init_process_group("nccl", device_id=dev, timeout=timedelta(seconds=120))

    import unified_fpn as U

    if args.train:
        return run_train(args, rank, world, local, dev)
    if args.kernels == "bandwidth":
        return run_bandwidth_kernels(args, dev)
    fp8 = args.dtype == "e4m3"
    dtype = {"bf16": torch.bfloat16, "fp16": torch.float16, "e4m3": torch.float8_e4m3fn}[args.dtype]
    esz = 1 if fp8 else 2
    out_esz = 2
    sizes = level_sizes(args.height, args.width)
    B = args.batch
    n_sets = 3  # rotating input sets, together larger than the 126 MB L2
    gen = torch.Generator(device=dev)
    feats, scales = [], []
    for s in range(n_sets):
        gen.manual_seed(1000 * rank + s)
        if fp8:
            # seeded N(0,1) features, quantised per tensor (scale = absmax / 448) on the device
            qs = [U.quantize_fp8(torch.randn(B, c, h, w, device=dev, generator=gen).contiguous(
                memory_format=torch.channels_last)) for c, (h, w) in zip(R50_CHANNELS, sizes)]
            feats.append([q for q, _ in qs])
            scales.append(torch.cat([sc for _, sc in qs]))
        else:
            feats.append([torch.randn(B, c, h, w, device=dev, generator=gen, dtype=torch.float32)
                          .clamp_min_(0).to(dtype).contiguous(memory_format=torch.channels_last)
                          for c, (h, w) in zip(R50_CHANNELS, sizes)])
            scales.append(None)
    in_mb = sum(B * c * h * w * esz for c, (h, w) in zip(R50_CHANNELS, sizes)) / 1e6
    fpn = U.UnifiedFPN(device=dev)
    fpn.set_schedule(fused_neck_kernel=args.schedule == "fused", single_stream=args.schedule == "serial")
    outs = []
    for s in range(n_sets):
        o = fpn(feats[s], return_p6=True, input_scales=scales[s])
        outs.append(o)
    torch.cuda.synchronize(dev)

    def step(i):
        fpn(feats[i % n_sets], return_p6=True, out=outs[i % n_sets], input_scales=scales[i % n_sets])

    for i in range(args.warmup):
        step(i)
    torch.cuda.synchronize(dev)
    if fpn.device_status() != 0:
        raise RuntimeError("device pipeline timeout during warm-up")
    launches_per_step = int(fpn.get_performance_breakdown()[1][4].item())

    stream = torch.cuda.current_stream(dev)
    e0 = torch.cuda.Event(enable_timing=True)
    e1 = torch.cuda.Event(enable_timing=True)
    clocks = ClockSampler(local)
    if world > 1:
        dist.barrier()
    torch.cuda.synchronize(dev)
    clocks.start()
    time.sleep(0.3)  # let the sampler take its first reading
    e0.record(stream)
    for i in range(args.steps):
        step(i)
    e1.record(stream)
    torch.cuda.synchronize(dev)
    if world > 1:
        dist.barrier()
    clk = clocks.stop()
    ms_local = e0.elapsed_time(e1)
    ms, images = job_throughput(ms_local, B * args.steps, world, dev)
    ranks_ms = per_rank_ms(ms_local / args.steps, world, dev)
    status = fpn.device_status()
    value = images / (ms / 1e3)
    ms_per_step = ms / args.steps

    # ---------------------------------------------------------------- e2e through the public API
    # Host-resident batches streamed through unified_fpn.HostPipeline: every step copies its
    # C2..C5 (and e4m3 scales) from pinned host memory and P2..P6 back to pinned host memory;
    # step i's neck overlaps step i+1's copy-in and step i-1's copy-out.
    e2e = None
    if not args.no_e2e:
        pipe = U.HostPipeline(fpn, feats[0], return_p6=True, depth=2)
        host_in = [f.cpu().pin_memory() for f in feats[0]]
        host_sc = scales[0].cpu().pin_memory() if fp8 else None
        host_out = [pipe.host_buffers() for _ in range(2)]
        h2d = sum(t.numel() * t.element_size() for t in host_in) + (16 if fp8 else 0)
        d2h = sum(t.numel() * t.element_size() for t in host_out[0])
        for k in range(4):
            pipe.submit(host_in, host_out[k % 2], host_sc)
        pipe.synchronize()
        n_e2e = max(6, min(args.steps, 20))
        if world > 1:
            dist.barrier()
        torch.cuda.synchronize(dev)
        a0 = torch.cuda.Event(enable_timing=True)
        a1 = torch.cuda.Event(enable_timing=True)
        a0.record(stream)
        pipe.fork(stream)
        for k in range(n_e2e):
            pipe.submit(host_in, host_out[k % 2], host_sc)
        pipe.join(stream)
        a1.record(stream)
        torch.cuda.synchronize(dev)
        ems, e_images = job_throughput(a0.elapsed_time(a1), B * n_e2e, world, dev)
        e2e = {"value": e_images / (ems / 1e3), "unit": "images/s", "h2d_bytes_per_step": h2d,
               "d2h_bytes_per_step": d2h, "steps": n_e2e,
               "api": "unified_fpn.HostPipeline (copy-in / neck / copy-out overlapped across steps)"}
        if world > 1:
            dist.barrier()
        cms, c_images = e2e_ceiling(dev, h2d, d2h, n_e2e, B)
        cms, c_images = job_throughput(cms, c_images, world, dev)
        e2e["ceiling"] = {"value": c_images / (cms / 1e3), "unit": "images/s",
                          "what": "the same bytes as plain pinned cudaMemcpyAsync H2D + D2H on two "
                                  "overlapped streams, no compute (host memory / PCIe bound)"}

    # ---------------------------------------------------------------- roofline of the dominant kernel
    roofline = None
    peaks = measured_peaks()
    kernel_share = None
    if not args.no_roofline:
        kt, mt = fpn.get_performance_breakdown(feats[0], input_scales=scales[0])  # serialised, event-timed
        total = float(kt.sum().item())
        from unified_fpn.helpers import STAGES_TC
        kernel_share = {n: {"ms": round(float(v), 4), "share": round(float(v) / total, 4)}
                        for n, v in zip(STAGES_TC, kt.tolist())} if total > 0 else None
        h2, w2 = sizes[0]
        xr = torch.randn(B, 256, h2, w2, device=dev, generator=gen).contiguous(
            memory_format=torch.channels_last)
        w3 = torch.randn(256, 256, 3, 3, device=dev, generator=gen) * 0.03
        bias = torch.zeros(256, device=dev)
        # the engine's form: single-CTA halo tiles, with the mixed tiling (tile_w -4: the own
        # view for whole 16-row tile rows, the transposed view for the last 1..8 rows) or the
        # transposed view (-2) when that needs fewer 8 x 16 tiles (200 x 304: 475 instead of 494
        # per image)
        plain_tiles = -(-w2 // 8) * -(-h2 // 16)
        trans_tiles = -(-h2 // 8) * -(-w2 // 16)
        mixed_tiles = -(-w2 // 8) * (h2 // 16) + -(-w2 // 16)
        mixed_ok = (h2 >= 16 and 0 < h2 % 16 <= 8
                    and mixed_tiles < plain_tiles and mixed_tiles <= trans_tiles)
        tw = -4 if mixed_ok else (-2 if trans_tiles < plain_tiles else 0)
        if fp8:
            xq, xs = U.quantize_fp8(xr, per_image=True)
            wq, wsc = U.quantize_fp8_rows(w3, pack3x3=True)
            conv = lambda: U.fpn_conv3x3_fp8(xq, xs, wq, wsc, bias, tile_w=tw)  # noqa: E731
        else:
            x = xr.to(dtype)
            wt = U.pack_conv3x3_weight(w3, dtype)
            conv = lambda: U.fpn_conv3x3(x, wt, bias, tile_w=tw)  # noqa: E731
        reps = 20
        for _ in range(3):
            conv()
        r0 = torch.cuda.Event(enable_timing=True)
        r1 = torch.cuda.Event(enable_timing=True)
        r0.record(stream)
        for _ in range(reps):
            conv()
        r1.record(stream)
        torch.cuda.synchronize(dev)
        kms = r0.elapsed_time(r1) / reps
        flops = 2.0 * B * h2 * w2 * 256 * 256 * 9
        achieved = flops / (kms * 1e-3) / 1e12
        # e4m3 runs at twice the bf16 dense rate; no e4m3 GEMM peak is measured on this
        # pool, so its peak is derived as 2 x the measured bf16 figures.
        mult = 2.0 if fp8 else 1.0
        peak = peaks["bf16_tflops"] * mult
        traffic = profile_traffic("conv3x3_fp8_p2_r50_640x640_b16" if fp8
                                  else "conv3x3_p2_r50_800x1216_b2")
        # the engine's P2 3x3: single-CTA halo tiles (tcgen05, TMEM accumulators)
        form = {-4: "mixed tiling", -2: "transposed view", 0: "own view"}[tw]
        roofline = {"kernel": f"conv3x3 P2 implicit GEMM (tcgen05 "
                              f"{'kind::f8f6f4' if fp8 else 'kind::f16'}, halo tiles, {form}), "
                              f"{B}x{h2}x{w2}x256 -> 256",
                    "bound": "tensor", "achieved": round(achieved, 1), "peak": peak,
                    "unit": "TFLOP/s", "frac": round(achieved / peak, 4),
                    "peak_src": (f"derived: 2 x {peaks['src']} bf16 burst" if fp8
                                 else f"{peaks['src']} bf16 burst (kernel timed alone)"),
                    "launch_ms": round(kms, 4), "flops_per_launch": flops, "traffic": traffic,
                    "neck_frac_of_roofline": None}
        # whole-neck roofline: slower of FLOPs at the sustained tensor peak and bytes at HBM peak
        f_all = neck_flops(B, R50_CHANNELS, sizes)
        b_all = neck_bytes(B, R50_CHANNELS, sizes, esz, out_esz)
        t_roof = max(f_all / (peaks["bf16_tflops_sustained"] * mult * 1e12),
                     b_all / (peaks["hbm_gbs"] * 1e9))
        roofline["neck_frac_of_roofline"] = round(t_roof * 1e3 / ms_per_step, 4)
        roofline["neck_roofline_ms"] = round(t_roof * 1e3, 4)

    kernel_timeline = None
    if rank == 0 and world == 1 and not args.no_roofline:
        kernel_timeline = cupti_timeline(step)
    timeline = None
    if args.schedule == "fused" and not args.no_roofline:
        timeline = {k: (round(v, 1) if v is not None else None)
                    for k, v in fpn.neck_timeline(feats[0]).items()}

    extra = None
    if not args.no_extra and world == 1 and not fp8 and not args.no_roofline:
        extra = extra_workloads(dev, peaks)

    cpu = None
    if rank == 0 and not args.no_cpu_baseline and world == 1:
        cpu = cpu_baseline(image=(args.height, args.width))

    if rank == 0:
        data = ("synthetic (seeded N(0,1) features quantised per tensor to e4m3 on the device; "
                "random Kaiming-normal weights quantised per output channel)" if fp8 else
                "synthetic (seeded N(0,1) after ReLU clamp; random Kaiming-normal weights)")
        line = {
            "metric": METRIC_FP8 if fp8 else METRIC, "value": round(value, 2), "unit": "images/s",
            "n_gpus": world, "steps": args.steps,
            "warmup": args.warmup, "ms_per_step": round(ms_per_step, 5), "higher_is_better": True,
            "scaling": "weak", "vs_baseline": None, "dtype": args.dtype, "data": data,
            "config": {"workload": f"R50 FPN neck {args.height}x{args.width}, {B} images/GPU, {args.dtype} NHWC"
                                   + (" (bf16 outputs)" if fp8 else ""),
                       "global_batch": B * world, "per_gpu_batch": B,
                       "levels": [[B, c, h, w] for c, (h, w) in zip(R50_CHANNELS, sizes)],
                       "l2": f"inputs rotate over {n_sets} sets ({n_sets} x {in_mb:.0f} MB) > 126 MB L2",
                       "parallelism": f"dp{world} batch shards, no collective on the data path"},
            "clocks": clk, "e2e": e2e, "gpu_launches": launches_per_step * args.steps,
            "schedule": args.schedule, "neck_timeline_us": timeline,
            "roofline": roofline, "kernel_time_share": kernel_share,
            "kernel_time_share_what": "device time per stage of one forward with the stages serialised "
                                      "on one stream (replayed as a CUDA graph, events between stages; "
                                      "the concurrent schedule overlaps them)",
            "kernel_timeline_us": kernel_timeline,
            "cpu_baseline": cpu,
            "device_status": status, "per_rank_ms_per_step": ranks_ms, "extra": extra,
        }
        print(json.dumps(line), flush=True)
    if world > 1:
        dist.barrier()
        dist.destroy_process_group()
    return 0


if __name__ == "__main__":
    sys.exit(main())

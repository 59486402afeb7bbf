"""DCNv2 forward benchmark (one JSON line on rank 0).

  python bench.py [--gpus N] [--steps K] [--warmup W] [--impl ours|reference] [--workload NAME]
                  [--global-batch G]

A step is one forward of the DCNv2 layer over one batch of seeded synthetic input (the
dcnv2_b200.workloads table; default fp16_n64_256c_64: N=64, C=O=256, 64x64, 3x3, fp16). With
N GPUs (torchrun, one process per GPU) every rank runs its own batch of the same size: the
batch-sharded layer has no exchange step, so there is no collective on the data path and the
scaling is weak. --global-batch G instead splits one batch of G images over the ranks (rank r
takes the contiguous slice dcnv2_b200.shard.shard_range(G, N, r)): strong scaling. The default
line carries that split of the headline workload (G = 64) under "split".

Timing: W untimed steps; K steps between barriers and device synchronisation, CUDA events on the
launching stream, max over ranks. Where a step's inputs and outputs exceed twice the 126 MB L2
nothing is flushed; smaller working sets get a 252 MB write before every timed step, outside the
timed events ("l2" in config says which).

Keys beyond the base contract: roofline (dominant kernel, timed live by CUDA events recorded
between the launches of each forward), cpu_baseline (the oracle's CPU restatement of the
reference on a bounded sample, rank 0 at N=1), e2e (host buffers through the C ABI's
host-buffer forward dcnv2_forward_host: inputs uploaded and y downloaded inside the timed region),
clocks (nvidia-smi sampled during the timed region), gpu_launches, secondary (every other
workload of the table measured the same way, with fewer steps, plus the headline in the fp32
sampler mode), split (the batch split described above).

--impl reference times the reference's own CPU implementation of the path (the oracle port of
src/dcn_kernel.cu + the reference GEMM, all host threads) on the same workload and config, each
step a bounded band of output pixels; it also reports the reference's GPU path (its im2col +
cuBLAS kernels built for sm_100a, oracle/_ref) under "reference_gpu" when that build is present.
That arm maps no library of this repository's product.
"""
import argparse
import json
import os
import statistics
import subprocess
import sys
import threading
import time

ROOT = os.path.dirname(os.path.abspath(__file__))
sys.path.insert(0, os.path.join(ROOT, "tensorrt-dcnv2-plugin_b200"))

import numpy as np  # noqa: E402
import torch  # noqa: E402

# Pure Python: importing it maps no library (capi loads libdcnv2.so on first use).
from dcnv2_b200 import workloads as wl  # noqa: E402
from dcnv2_b200.shard import shard_range  # noqa: E402

PROFILE_TRAFFIC = os.path.join(ROOT, "profiles", "traffic.txt")
HEADLINE = "fp16_n64_256c_64"
SPLIT_GLOBAL_BATCH = 64            # the headline batch, split evenly over the GPUs
L2_BYTES = 126 * 1024 * 1024
SPEC_PEAK = {"fp16": 2250.0, "int8": 4500.0}      # B200 dense tensor peaks (no 2:4 sparsity)
# fp32 runs on CUDA cores: 148 SMs x 128 FMA/clk x 2 FLOP x 1.965 GHz (nominal, not measured)
FP32_SIMT_PEAK = 148 * 128 * 2 * 1.965e9 / 1e12


def parse_args():
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=3000)
    ap.add_argument("--warmup", type=int, default=20)
    ap.add_argument("--impl", default="ours", choices=["ours", "reference"])
    ap.add_argument("--workload", default=HEADLINE, choices=list(wl.WORKLOADS))
    ap.add_argument("--global-batch", type=int, default=0,
                    help="split one batch of this many images over the ranks (strong scaling)")
    ap.add_argument("--math", type=int, default=0,
                    help="dcnv2_desc.math of the main workload (1 = DCNV2_MATH_PRECISE)")
    ap.add_argument("--batch", type=int, default=0,
                    help="images per rank instead of the workload's batch (small profiling cases)")
    ap.add_argument("--head", action="store_true",
                    help="time only the headline layer with its offset / mask head "
                         "(dcnv2_forward_with_head) and print that entry")
    ap.add_argument("--e2e-steps", type=int, default=20)
    ap.add_argument("--cpu-seconds", type=float, default=12.0)
    ap.add_argument("--no-cpu-baseline", action="store_true")
    ap.add_argument("--no-secondary", action="store_true")
    return ap.parse_args()


# ---------------------------------------------------------------- what both arms print
def unit_of(precision: str) -> str:
    return "TOP/s" if precision == "int8" else "TFLOP/s"


def metric_of(workload: str) -> str:
    if workload == HEADLINE:
        return "DCNv2 fwd TFLOP/s (256ch 64x64 3x3) fp16, 1-8 B200"
    return f"DCNv2 fwd {unit_of(parts_meta(workload)[1])} ({workload}), 1-8 B200"


def parts_meta(workload: str, n=None):
    """Layers of one step of `workload` without drawing its tensors (shapes only)."""
    if workload == "fpn_fp16_b32":
        return [wl.Layer(n or 32, 256, s, s, 256) for s in wl.FPN_LEVELS], "fp16"
    if workload == "fp32_n1_256c_64":
        return [wl.Layer(n or 1, 256, 64, 64, 256)], "fp32"
    if workload in ("fp16_n64_256c_64", "int8_n64_256c_64"):
        return [wl.Layer(n or 64, 256, 64, 64, 256)], workload[:4]
    prec = "int8" if workload.endswith("int8") else "fp16"
    return [wl.Layer(n or 16, 512, 128, 128, 512, 3, 1, 2, 2, 8)], prec


def step_bytes(layers, precision: str) -> int:
    xb = {"fp32": 4, "fp16": 2, "int8": 1}[precision]
    gb = 2 if precision == "fp16" else 4  # offset / mask / bias / y
    tot = 0
    for L in layers:
        T = L.kernel ** 2
        P = L.ho * L.wo
        tot += L.n * L.c * L.h * L.w * xb + L.out_c * L.c * T * xb + L.out_c * gb
        tot += L.n * 3 * L.groups * T * P * gb + L.n * L.out_c * P * gb
    return tot


def flushes_l2(workload: str, n=None) -> bool:
    layers, prec = parts_meta(workload, n)
    return step_bytes(layers, prec) < 2 * L2_BYTES


def config_of(workload: str, world: int, batch_per_rank: int, global_batch: int,
              scaling: str) -> dict:
    layers, prec = parts_meta(workload, batch_per_rank)
    L = layers[0]
    l2 = ("L2 flushed before every timed step (a 252 MB write outside the timed events)"
          if flushes_l2(workload, batch_per_rank) else "step working set exceeds L2 (no flush)")
    cfg = {"workload": workload, "batch_per_gpu": batch_per_rank, "global_batch": global_batch,
           "c": L.c, "out_c": L.out_c, "hw": [L.h, L.w], "kernel": L.kernel, "stride": L.stride,
           "padding": L.padding, "dilation": L.dilation, "deformable_groups": L.groups,
           "precision": prec,
           "parallelism": (f"batch-shard x{world}, {scaling} scaling (one process per GPU, "
                           "no collective on the data path)"),
           "l2": l2}
    if len(layers) > 1:
        cfg["levels_hw"] = [x.h for x in layers]
        cfg["step"] = ("the five levels as one CUDA graph, one stream per level "
                       "(dcnv2_b200.levels.LevelsRunner)")
    return cfg


# ---------------------------------------------------------------- distributed plumbing
class Dist:
    def __init__(self):
        self.world = int(os.environ.get("WORLD_SIZE", "1"))
        self.rank = int(os.environ.get("RANK", "0"))
        self.local = int(os.environ.get("LOCAL_RANK", "0"))
        self.pg = False

    def init(self, backend="nccl"):
        if self.world > 1:
            import datetime
            os.environ.setdefault("MASTER_ADDR", "127.0.0.1")
            torch.distributed.init_process_group(
                backend, timeout=datetime.timedelta(seconds=120),
                device_id=torch.device(f"cuda:{self.local}"))
            self.pg = True

    def barrier(self):
        if self.pg:
            torch.distributed.barrier()

    def max(self, v: float) -> float:
        if not self.pg:
            return v
        t = torch.tensor([v], dtype=torch.float64, device=f"cuda:{self.local}")
        torch.distributed.all_reduce(t, op=torch.distributed.ReduceOp.MAX)
        return float(t.item())

    def close(self):
        if self.pg:
            torch.distributed.destroy_process_group()


# ---------------------------------------------------------------- clock sampling
class ClockSampler:
    """nvidia-smi --query-gpu ... -lms 200 while the timed region runs."""
    FIELDS = ("index,clocks.sm,clocks.max.sm,power.draw,clocks_event_reasons.active,"
              "clocks_event_reasons.hw_slowdown,clocks_event_reasons.hw_thermal_slowdown,"
              "clocks_event_reasons.sw_thermal_slowdown,clocks_event_reasons.sw_power_cap")

    def __init__(self, gpu_index):
        self.gpu = gpu_index
        self.proc = None
        self.lines = []

    def start(self):
        try:
            self.proc = subprocess.Popen(
                ["nvidia-smi", f"--id={self.gpu}", f"--query-gpu={self.FIELDS}",
                 "--format=csv,noheader,nounits", "-lms", "200"],
                stdout=subprocess.PIPE, stderr=subprocess.DEVNULL, text=True)
            self.t = threading.Thread(target=self._read, daemon=True)
            self.t.start()
        except OSError:
            self.proc = None

    def _read(self):
        for line in self.proc.stdout:
            self.lines.append(line.strip())

    def stop(self):
        if not self.proc:
            return None
        self.proc.terminate()
        try:
            self.proc.wait(timeout=5)
        except subprocess.TimeoutExpired:
            self.proc.kill()
        self.t.join(timeout=2)
        mhz, maxmhz, reasons = [], None, set()
        names = ["hw_slowdown", "hw_thermal_slowdown", "sw_thermal_slowdown", "sw_power_cap"]
        for ln in self.lines:
            f = [x.strip() for x in ln.split(",")]
            if len(f) < 9:
                continue
            try:
                mhz.append(float(f[1]))
                maxmhz = float(f[2])
            except ValueError:
                continue
            for nm, v in zip(names, f[5:9]):
                if v.lower() == "active":
                    reasons.add(nm)
        if not mhz:
            return None
        return {"sm_mhz": statistics.median(mhz), "sm_max_mhz": maxmhz,
                "reasons": sorted(reasons), "samples": len(mhz)}


# ---------------------------------------------------------------- helpers
def peaks():
    """(burst bf16 dense TFLOP/s, sustained bf16 dense TFLOP/s, HBM GB/s, source)."""
    try:
        with open(os.path.join(ROOT, "MEASURED_PEAKS.json")) as f:
            d = json.load(f)
        return (d.get("bf16_tflops", 1590.0), d.get("bf16_tflops_sustained", 1400.0),
                d.get("hbm_gbs", 6650.0), "measured")
    except OSError:
        return 1590.0, 1400.0, 6650.0, "fallback"


def traffic_for(workload: str, kernel: str):
    """Per-launch DRAM bytes of `kernel` on `workload` from the committed ncu summary."""
    try:
        with open(PROFILE_TRAFFIC) as f:
            for line in f:
                p = line.split()
                if len(p) >= 3 and p[0] == workload and p[1] == kernel:
                    return int(p[2])
    except OSError:
        pass
    return None


def dtype_of(capi, precision):
    return {"fp32": capi.DType.FLOAT, "fp16": capi.DType.HALF, "int8": capi.DType.INT8}[precision]


def desc_of(inp, math=0):
    from dcnv2_b200 import capi
    L = inp.layer
    return capi.make_desc(L.n, L.c, L.h, L.w, L.out_c, L.kernel, L.stride, L.padding, L.dilation,
                          L.groups, dtype_of(capi, inp.precision), math)


def alloc_for(inp, device, math=0):
    from dcnv2_b200 import capi
    L = inp.layer
    ws = torch.empty(capi.workspace_size(desc_of(inp, math)), dtype=torch.uint8, device=device)
    ydt = torch.float16 if inp.precision == "fp16" else torch.float32
    out = torch.empty((L.n, L.out_c, L.ho, L.wo), dtype=ydt, device=device)
    return ws, out


def step_fn(inp, ws, out, math=0):
    """One forward through the public C ABI on the given stream."""
    from dcnv2_b200 import capi
    desc = desc_of(inp, math)
    ptrs = [t.data_ptr() for t in inp.tensors()]

    def run(stream):
        st = capi.forward_raw(desc, *ptrs, out.data_ptr(), ws.data_ptr(), ws.numel(),
                              inp.x_scale, inp.w_scale, stream)
        if st != 0:
            raise RuntimeError(f"dcnv2_forward failed: {capi.status_string(st)}")
    return desc, ptrs, run


def time_steps(run, stream, steps, warmup, dist):
    for _ in range(warmup):
        run(stream.cuda_stream)
    torch.cuda.synchronize()
    dist.barrier()
    torch.cuda.synchronize()
    e0 = torch.cuda.Event(enable_timing=True)
    e1 = torch.cuda.Event(enable_timing=True)
    e0.record(stream)
    for _ in range(steps):
        run(stream.cuda_stream)
    e1.record(stream)
    torch.cuda.synchronize()
    dist.barrier()
    torch.cuda.synchronize()
    return e0.elapsed_time(e1) / steps


def time_steps_flushed(runs, stream, steps, dist, flush):
    """Per-step CUDA-event timing with the L2 flushed (a write larger than L2) before each step;
    the flush is outside the events. Returns ms per step and ms per part of a step."""
    torch.cuda.synchronize()
    dist.barrier()
    torch.cuda.synchronize()
    per_part = np.zeros(len(runs))
    evs = [[torch.cuda.Event(enable_timing=True) for _ in range(len(runs) + 1)]
           for _ in range(steps)]
    for i in range(steps):
        with torch.cuda.stream(stream):
            flush.add_(1)
        for k, run in enumerate(runs):
            evs[i][k].record(stream)
            run(stream.cuda_stream)
        evs[i][len(runs)].record(stream)
    torch.cuda.synchronize()
    dist.barrier()
    torch.cuda.synchronize()
    for i in range(steps):
        per_part += [evs[i][k].elapsed_time(evs[i][k + 1]) for k in range(len(runs))]
    per_part /= steps
    return float(per_part.sum()), per_part


def kernel_breakdown(inp, ws, out, stream, steps, math=0, flush=None):
    """Per-launch CUDA-event timing of one forward (events recorded between the launches, on the
    launching stream); with `flush`, the L2 is flushed before each forward."""
    from dcnv2_b200 import capi
    desc, ptrs, _ = step_fn(inp, ws, out, math)
    n = capi.launch_count(desc)
    evs = [[torch.cuda.Event(enable_timing=True) for _ in range(n + 1)] for _ in range(steps)]
    for row in evs:  # torch creates the cudaEvent_t on first record
        for e in row:
            e.record(stream)
    torch.cuda.synchronize()
    for i in range(steps):
        if flush is not None:
            with torch.cuda.stream(stream):
                flush.add_(1)
        st = capi.forward_events_raw(desc, *ptrs, out.data_ptr(), ws.data_ptr(), ws.numel(),
                                     inp.x_scale, inp.w_scale, stream.cuda_stream,
                                     [e.cuda_event for e in evs[i]])
        if st != 0:
            raise RuntimeError(capi.status_string(st))
    torch.cuda.synchronize()
    per = np.array([[evs[i][k].elapsed_time(evs[i][k + 1]) for k in range(n)]
                    for i in range(steps)])
    return per.mean(axis=0)  # ms per launch slot


def e2e_measure(inp_host, device, stream, steps, dist, math=0):
    """Host buffers in, host buffer out, through the C ABI's host-buffer forward
    (dcnv2_forward_host): per step the weight and bias are copied to the device and x, offset and
    mask are uploaded, computed and y downloaded in chunks of images with the copies overlapped.
    Every byte of every input crosses to the device and y comes back inside the timed region."""
    from dcnv2_b200 import capi
    L = inp_host.layer
    host = [t.contiguous().pin_memory() for t in inp_host.tensors()]  # x, offset, mask, w, b
    desc = desc_of(inp_host, math)
    oshape = capi.output_shape(desc)
    ydt = torch.float16 if inp_host.precision == "fp16" else torch.float32
    y_host = torch.empty(oshape, dtype=ydt).pin_memory()
    w_dev = torch.empty_like(host[3], device=device)
    b_dev = torch.empty_like(host[4], device=device)
    wsz = capi.forward_host_workspace_size(desc, 0)
    ws = torch.empty(wsz, dtype=torch.uint8, device=device)
    xs, wscale = inp_host.x_scale, inp_host.w_scale
    h2d = sum(t.numel() * t.element_size() for t in host)
    d2h = y_host.numel() * y_host.element_size()

    def step():
        with torch.cuda.stream(stream):
            w_dev.copy_(host[3], non_blocking=True)
            b_dev.copy_(host[4], non_blocking=True)
            rc = capi.forward_host_raw(desc, host[0].data_ptr(), host[1].data_ptr(),
                                       host[2].data_ptr(), w_dev.data_ptr(), b_dev.data_ptr(),
                                       y_host.data_ptr(), ws.data_ptr(), wsz, xs, wscale, 0,
                                       stream.cuda_stream)
            if rc != 0:
                raise RuntimeError(f"dcnv2_forward_host failed {rc}")

    for _ in range(2):
        step()
    torch.cuda.synchronize()
    dist.barrier()
    torch.cuda.synchronize()
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    e0.record(stream)
    for _ in range(steps):
        step()
    e1.record(stream)
    torch.cuda.synchronize()
    dist.barrier()
    ms = dist.max(e0.elapsed_time(e1) / steps)
    del ws, w_dev, b_dev
    return ms, h2d, d2h


def host_copy_bound(inp_host, device, stream, steps, dist):
    """The host<->device copy rate the ranks get together: per step each rank uploads its
    inputs (pinned, one cudaMemcpyAsync per tensor) on one stream while it downloads a buffer of
    its output's size on another; all ranks at once. Returns ms per step (max over ranks)."""
    host_in = [t.contiguous().pin_memory() for t in inp_host.tensors()[:3]]
    L = inp_host.layer
    ydt = torch.float16 if inp_host.precision == "fp16" else torch.float32
    y_host = torch.empty((L.n, L.out_c, L.ho, L.wo), dtype=ydt).pin_memory()
    dev_in = [torch.empty_like(t, device=device) for t in host_in]
    y_dev = torch.empty_like(y_host, device=device)
    down = torch.cuda.Stream(device)

    def step():
        down.wait_stream(stream)
        with torch.cuda.stream(stream):
            for d, h in zip(dev_in, host_in):
                d.copy_(h, non_blocking=True)
        with torch.cuda.stream(down):
            y_host.copy_(y_dev, non_blocking=True)
        stream.wait_stream(down)

    step()
    torch.cuda.synchronize()
    dist.barrier()
    torch.cuda.synchronize()
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    e0.record(stream)
    for _ in range(steps):
        step()
    e1.record(stream)
    torch.cuda.synchronize()
    dist.barrier()
    ms = dist.max(e0.elapsed_time(e1) / steps)
    up = sum(t.numel() * t.element_size() for t in host_in)
    dn = y_host.numel() * y_host.element_size()
    return {"ms_per_step": round(ms, 3), "h2d_bytes_per_rank": up, "d2h_bytes_per_rank": dn,
            "aggregate_gbs": round((up + dn) * dist.world / (ms * 1e-3) / 1e9, 1),
            "what": "concurrent pinned uploads and downloads of one step's bytes on every rank "
                    "(cudaMemcpyAsync), the bound of e2e"}


def cpu_baseline(inp_cpu, seconds: float):
    """The oracle's CPU restatement (reference fast-path semantics), all host threads, on a
    bounded band of output pixels of image 0; returns (rate, description, threads)."""
    sys.path.insert(0, os.path.join(ROOT, "oracle"))
    import oracle
    L = inp_cpu.layer
    threads = os.cpu_count() or 1
    x, off, msk, w, b = [t[:1].float().numpy() if i < 3 else t.float().numpy()
                         for i, t in enumerate(inp_cpu.tensors())]
    prec = "fp16" if inp_cpu.precision == "fp16" else "fp32"
    P = L.ho * L.wo
    per_px = 2 * L.out_c * L.c * L.kernel ** 2
    # calibrate on a small band, then size the timed band for about `seconds`
    band = min(P, 64)
    t0 = time.perf_counter()
    oracle.forward_ref_band(x, off, msk, w, b, 0, band, L.stride, L.padding, L.dilation,
                            L.groups, precision=prec, threads=threads)
    dt = time.perf_counter() - t0
    px = int(min(P, max(band, band * seconds / max(dt, 1e-6))))
    t0 = time.perf_counter()
    done, p0 = 0, 0
    while time.perf_counter() - t0 < seconds and done < 64 * P:
        p1 = min(P, p0 + px)
        oracle.forward_ref_band(x, off, msk, w, b, p0, p1, L.stride, L.padding, L.dilation,
                                L.groups, precision=prec, threads=threads)
        done += p1 - p0
        p0 = 0 if p1 >= P else p1
    el = time.perf_counter() - t0
    rate = per_px * done / el / 1e12
    what = {"fp16": "fp16", "fp32": "fp32", "int8": "int8 (fp32 columns on the integer "
                                                    "amplitudes)"}[inp_cpu.precision]
    return rate, (f"{done} output pixels of the {wl_name(inp_cpu)} layer (image 0), {what} "
                  f"reference semantics, {el:.1f} s"), threads


def wl_name(inp):
    L = inp.layer
    return f"{L.c}->{L.out_c} {L.h}x{L.w} k{L.kernel} d{L.dilation} dg{L.groups} {inp.precision}"


def torchvision_cpu(inp_cpu, seconds: float):
    """torchvision.ops.deform_conv2d fp32 on the host cores for one image (the reference's
    oracle path), in the line's unit."""
    try:
        from torchvision.ops import deform_conv2d
    except Exception:
        return None
    L = inp_cpu.layer
    torch.set_num_threads(os.cpu_count() or 1)
    x, off, msk, w, b = [t[:1].float() if i < 3 else t.float()
                         for i, t in enumerate(inp_cpu.tensors())]
    if inp_cpu.precision == "int8":
        x = x * inp_cpu.x_scale
        w = w * inp_cpu.w_scale
    t0, n = time.perf_counter(), 0
    while True:
        deform_conv2d(x, off, w, b, stride=L.stride, padding=L.padding, dilation=L.dilation,
                      mask=msk)
        n += 1
        if time.perf_counter() - t0 > seconds or n >= 20:
            break
    el = time.perf_counter() - t0
    per_img = 2 * L.out_c * L.c * L.kernel ** 2 * L.ho * L.wo
    return {"value": per_img * n / el / 1e12, "unit": unit_of(inp_cpu.precision),
            "cores": os.cpu_count(), "sample": f"{n} x 1 image fp32, {el:.1f} s"}


def roofline_of(workload, inp, kname, per):
    """Dominant-kernel roofline from the live per-launch timing `per` (ms per launch slot)."""
    peak_tf, peak_sus, _, peak_kind = peaks()
    main_ms = float(per[-1])
    achieved = inp.layer.flops / (main_ms * 1e-3) / 1e12
    unit = unit_of(inp.precision)
    if inp.precision == "fp32":
        roof = {"bound": "fp32 CUDA cores", "achieved": round(achieved, 1),
                "peak": round(FP32_SIMT_PEAK, 1), "unit": unit,
                "frac": round(achieved / FP32_SIMT_PEAK, 4),
                "peak_source": "nominal fp32 FMA rate (148 SMs x 128 FMA/clk x 1.965 GHz)"}
    else:
        int8 = inp.precision == "int8"
        tensor_peak = peak_tf * (2.0 if int8 else 1.0)
        sus_peak = peak_sus * (2.0 if int8 else 1.0)
        roof = {"bound": "tensor", "achieved": round(achieved, 1), "peak": round(tensor_peak, 1),
                "unit": unit, "frac": round(achieved / tensor_peak, 4),
                "frac_sustained": round(achieved / sus_peak, 4),
                "frac_spec": round(achieved / SPEC_PEAK[inp.precision], 4),
                "peak_source": f"{peak_kind} bf16 dense, burst (frac) and sustained under the "
                               f"power cap (frac_sustained)"
                               + (" x2 (int8 dense rate)" if int8 else "")}
    roof.update({"traffic": traffic_for(workload, kname), "kernel": kname,
                 "kernel_ms": round(main_ms, 4),
                 "launch_ms": [round(float(v), 4) for v in per]})
    alg_bytes = inp.input_bytes + inp.output_bytes
    roof["hbm_alg_gbs"] = round(alg_bytes / (float(per.sum()) * 1e-3) / 1e9, 1)
    return roof


# ---------------------------------------------------------------- one workload, measured
def measure(workload, dist, device, stream, steps, warmup, e2e_steps, cpu_seconds, tv_seconds,
            math=0, parts_cpu=None, with_clocks=False, n=None):
    """Times one workload on this rank's batch (all ranks take the same collective steps) and
    returns its measurement dict; `parts_cpu` overrides the drawn inputs (the batch split), `n`
    the workload's batch."""
    from dcnv2_b200 import capi
    if parts_cpu is None:
        parts_cpu = wl.workload_parts(workload, n=n, seed=1000 * dist.rank)
    parts = [p.to(device) for p in parts_cpu]
    bufs = [alloc_for(p, device, math) for p in parts]
    fns = [step_fn(p, ws, out, math) for p, (ws, out) in zip(parts, bufs)]
    runs = [f[2] for f in fns]
    launches = sum(capi.launch_count(f[0]) for f in fns)
    dom = max(range(len(parts)), key=lambda i: parts[i].layer.flops)
    inp, inp_cpu = parts[dom], parts_cpu[dom]
    (ws, out), (desc, _, _) = bufs[dom], fns[dom]
    n_img = parts[0].layer.n
    flush = None
    if flushes_l2(workload, n_img):
        flush = torch.empty(2 * L2_BYTES // 4, dtype=torch.float32, device=device)

    def run_all(st):
        for r in runs:
            r(st)

    for _ in range(warmup):
        run_all(stream.cuda_stream)
    torch.cuda.synchronize()
    clocks = None
    if with_clocks:
        try:  # nvidia-smi addresses the physical GPU; torch's index may be remapped
            gpu_id = "GPU-" + str(torch.cuda.get_device_properties(device).uuid)
        except Exception:
            gpu_id = str(dist.local)
        clocks = ClockSampler(gpu_id)
        clocks.start()
        time.sleep(0.3)
    part_ms = None
    if len(parts) > 1:
        # several layers per step (the FPN levels): one CUDA graph of all of them, each on its
        # own stream so the small levels run beside each other (dcnv2_b200.levels)
        from dcnv2_b200.levels import LevelsRunner
        runner = LevelsRunner([dict(x=p.x, offset=p.offset, mask=p.mask, weight=p.weight,
                                    bias=p.bias, stride=p.layer.stride, padding=p.layer.padding,
                                    dilation=p.layer.dilation, deformable_groups=p.layer.groups,
                                    math=math) for p in parts])
        grouped = [lambda _h: runner.run(stream)]
        for _ in range(3):  # replays before timing (the first uploads the graph)
            runner.run(stream)
        torch.cuda.synchronize()
        if flush is None:
            ms = time_steps(grouped[0], stream, steps, 0, dist)
        else:
            ms, _ = time_steps_flushed(grouped, stream, steps, dist, flush)
    elif flush is None:
        ms = time_steps(run_all, stream, steps, 0, dist)
    else:
        ms, _ = time_steps_flushed(runs, stream, steps, dist, flush)
    clk = clocks.stop() if clocks else None
    ms = dist.max(ms)
    if len(parts) > 1:  # each level alone, one after another (breakdown only)
        if flush is None:
            flush = torch.empty(2 * L2_BYTES // 4, dtype=torch.float32, device=device)
        _, part_ms = time_steps_flushed(runs, stream, min(steps, 200), dist, flush)

    flops = sum(p.layer.flops for p in parts)
    unit = unit_of(inp.precision)
    per = kernel_breakdown(inp, ws, out, stream, min(steps, 200), math,
                           flush if len(parts) == 1 else None)
    kname = capi.main_kernel(desc)
    res = {"value": round(flops * dist.world / (ms * 1e-3) / 1e12, 2), "unit": unit,
           "ms_per_step": round(ms, 4), "images_per_s": round(n_img * dist.world / (ms * 1e-3), 1),
           "roofline": roofline_of(workload, inp, kname, per),
           "gpu_launches_per_step": launches}
    if part_ms is not None:
        res["levels"] = [{"hw": p.layer.h, "ms_alone": round(float(m), 4),
                          "tflops_alone": round(p.layer.flops / (m * 1e-3) / 1e12, 1)}
                         for p, m in zip(parts, part_ms)]
        res["levels_sequential_ms"] = round(float(sum(part_ms)), 4)
    del runs, fns, bufs, parts, ws, out, inp
    flush = None
    torch.cuda.empty_cache()
    if e2e_steps > 0:
        e2e_ms, h2d, d2h = 0.0, 0, 0
        for p in parts_cpu:
            m, i_b, o_b = e2e_measure(p, device, stream, e2e_steps, dist, math)
            e2e_ms, h2d, d2h = e2e_ms + m, h2d + i_b, d2h + o_b
        res["e2e"] = {"value": round(flops * dist.world / (e2e_ms * 1e-3) / 1e12, 3),
                      "unit": unit, "ms_per_step": round(e2e_ms, 3), "h2d_bytes_per_step": h2d,
                      "d2h_bytes_per_step": d2h}
        torch.cuda.empty_cache()
    if dist.rank == 0 and dist.world == 1 and cpu_seconds > 0:
        v, sample, thr = cpu_baseline(inp_cpu, cpu_seconds)
        cpu = {"value": round(v, 5), "unit": unit, "cores": thr, "kind": "port", "sample": sample}
        tv = torchvision_cpu(inp_cpu, tv_seconds) if tv_seconds > 0 else None
        if tv:
            cpu["torchvision"] = tv
        res["cpu_baseline"] = cpu
    res["_clocks"] = clk
    return res


def measure_head(dist, device, stream, steps, cpu_seconds, n=None):
    """The headline layer with its offset / mask head (dcnv2_forward_with_head): one call per
    step computes om = conv2d(x, Wh, bh) on tensor cores from the layer's channels-last x, splits
    offset / sigmoid(mask) and runs the layer. Beside it: the layer alone on precomputed offsets
    (dcnv2_forward) and the unfused head as a detector runs it without this fusion (torch
    conv2d through cuDNN + slice + sigmoid, fp16), a library baseline."""
    from dcnv2_b200 import capi
    inp_cpu = wl.workload(HEADLINE, n=n, seed=1000 * dist.rank)
    L = inp_cpu.layer
    hw32, hb32 = wl.head_inputs(L, seed=1000 * dist.rank)
    inp = inp_cpu.to(device)
    hw, hb = hw32.half().to(device), hb32.half().to(device)
    desc = desc_of(inp)
    wsz = capi.forward_with_head_workspace_size(desc)
    ws = torch.empty(wsz, dtype=torch.uint8, device=device)
    y = torch.empty((L.n, L.out_c, L.ho, L.wo), dtype=torch.float16, device=device)
    ptrs = [t.data_ptr() for t in (inp.x, hw, hb, inp.weight, inp.bias)]

    def run(st):
        rc = capi.forward_with_head_raw(desc, *ptrs, y.data_ptr(), None, None, ws.data_ptr(), wsz,
                                        st)
        if rc != 0:
            raise RuntimeError(f"dcnv2_forward_with_head failed: {capi.status_string(rc)}")

    ms = dist.max(time_steps(run, stream, steps, 5, dist))
    ws2, out2 = alloc_for(inp, device)
    _, _, run_plain = step_fn(inp, ws2, out2)
    ms_plain = dist.max(time_steps(run_plain, stream, steps, 5, dist))
    n_off = 2 * L.groups * L.kernel ** 2

    def torch_head(_st):
        with torch.cuda.stream(stream):
            om = torch.nn.functional.conv2d(inp.x, hw, hb, padding=(L.kernel - 1) // 2)
            om[:, :n_off].contiguous()
            torch.sigmoid(om[:, n_off:])

    ms_torch = dist.max(time_steps(torch_head, stream, steps, 5, dist))
    head_flops = 2 * L.n * L.ho * L.wo * (3 * L.groups * L.kernel ** 2) * L.c * L.kernel ** 2
    del ws, ws2, out2, y, inp
    torch.cuda.empty_cache()
    return {"value": round((L.flops + head_flops) * dist.world / (ms * 1e-3) / 1e12, 2),
            "unit": "TFLOP/s", "ms_per_step": round(ms, 4),
            "layer_alone_ms": round(ms_plain, 4), "head_ms": round(ms - ms_plain, 4),
            "unfused_head_torch_cudnn_ms": round(ms_torch, 4),
            "what": f"om = conv2d(x, Wh[27,256,3,3], bh) + split + sigmoid fused in front of "
                    f"the 256->256 64x64 N={L.n} fp16 layer (dcnv2_forward_with_head); head_ms = "
                    f"the call minus the layer alone; the unfused head through torch/cuDNN for "
                    f"comparison"}


def split_inputs(workload, global_batch, dist):
    """This rank's slice of one seeded batch of `global_batch` images."""
    if global_batch < dist.world:
        raise SystemExit(f"--global-batch {global_batch} is smaller than the {dist.world} ranks")
    a, b = shard_range(global_batch, dist.world, dist.rank)
    return [p.images(a, b) for p in wl.workload_parts(workload, n=global_batch, seed=0)], (a, b)


def run_ours(args, dist):
    device = torch.device(f"cuda:{dist.local}")
    torch.cuda.set_device(device)
    stream = torch.cuda.Stream(device)
    steps, warm = args.steps, args.warmup
    cpu_s = 0.0 if args.no_cpu_baseline else args.cpu_seconds

    strong = args.global_batch > 0
    parts_cpu = None
    if strong:
        parts_cpu, _ = split_inputs(args.workload, args.global_batch, dist)
    head = measure(args.workload, dist, device, stream, steps, warm, args.e2e_steps, cpu_s,
                   min(cpu_s, 20.0), math=args.math, parts_cpu=parts_cpu, with_clocks=True,
                   n=args.batch or None)
    batch_rank = (parts_cpu[0].layer.n if strong
                  else parts_meta(args.workload, args.batch or None)[0][0].n)
    global_batch = args.global_batch if strong else batch_rank * dist.world

    secondary = {}
    split = None
    if (not args.no_secondary and args.workload == HEADLINE and not strong and not args.batch
            and not args.math):
        sec_steps = max(20, steps // 20)
        sec_cpu = min(cpu_s, 4.0)
        # the headline layer with the fp32 sampler (one rounding per column value)
        r = measure(HEADLINE, dist, device, stream, sec_steps, 5, 0, 0.0, 0.0, math=1)
        r.pop("_clocks")
        r["math"] = "DCNV2_MATH_PRECISE (fp32 sampler arithmetic, the reference's rounding)"
        secondary[HEADLINE + "_precise"] = r
        secondary[HEADLINE + "_with_head"] = measure_head(dist, device, stream, sec_steps,
                                                          sec_cpu)
        for name in ("int8_n64_256c_64", "fp32_n1_256c_64", "fpn_fp16_b32", "big_512c_128_dg8",
                     "big_512c_128_dg8_int8"):
            big = name.startswith("big")
            r = measure(name, dist, device, stream, max(10, sec_steps // (8 if big else 1)), 5,
                        5 if big else 10, sec_cpu, min(sec_cpu, 3.0))
            r.pop("_clocks")
            r["config"] = config_of(name, dist.world, parts_meta(name)[0][0].n,
                                    parts_meta(name)[0][0].n * dist.world, "weak")
            secondary[name] = r
        # one batch of 64 images split evenly over the ranks (strong scaling)
        if dist.world > 1:
            sp_cpu, (a, b) = split_inputs(HEADLINE, SPLIT_GLOBAL_BATCH, dist)
            r = measure(HEADLINE, dist, device, stream, max(100, steps // 5), 10, 10, 0.0, 0.0,
                        parts_cpu=sp_cpu)
            r.pop("_clocks")
            sizes = [shard_range(SPLIT_GLOBAL_BATCH, dist.world, k) for k in range(dist.world)]
            # value is per rank batch x world in measure(); restate it for the global batch
            flops_global = wl.Layer(SPLIT_GLOBAL_BATCH, 256, 64, 64, 256).flops
            r["value"] = round(flops_global / (r["ms_per_step"] * 1e-3) / 1e12, 2)
            r["images_per_s"] = round(SPLIT_GLOBAL_BATCH / (r["ms_per_step"] * 1e-3), 1)
            if "e2e" in r:
                r["e2e"]["value"] = round(flops_global / (r["e2e"]["ms_per_step"] * 1e-3) / 1e12, 3)
            r["host_copy"] = host_copy_bound(sp_cpu[0], device, stream, 10, dist)
            r.update({"global_batch": SPLIT_GLOBAL_BATCH, "scaling": "strong",
                      "images_per_rank": [y - x for x, y in sizes]})
            split = r
        else:
            split = {"global_batch": SPLIT_GLOBAL_BATCH, "scaling": "strong",
                     "images_per_rank": [SPLIT_GLOBAL_BATCH], "value": head["value"],
                     "ms_per_step": head["ms_per_step"],
                     "note": "one GPU: the split is the headline measurement itself"}

    if dist.rank == 0:
        if strong:  # value from measure() is per-rank batch x world; restate for the batch
            flops_global = sum(L.flops for L in parts_meta(args.workload, args.global_batch)[0])
            head["value"] = round(flops_global / (head["ms_per_step"] * 1e-3) / 1e12, 2)
            head["images_per_s"] = round(args.global_batch / (head["ms_per_step"] * 1e-3), 1)
            if "e2e" in head:
                head["e2e"]["value"] = round(
                    flops_global / (head["e2e"]["ms_per_step"] * 1e-3) / 1e12, 3)
        prec = parts_meta(args.workload)[1]
        line = {
            "metric": metric_of(args.workload),
            "value": head["value"], "unit": head["unit"], "n_gpus": dist.world,
            "steps": steps, "warmup": warm, "ms_per_step": head["ms_per_step"],
            "higher_is_better": True, "scaling": "strong" if strong else "weak",
            "vs_baseline": None, "dtype": prec,
            "data": "synthetic (seeded torch.Generator, dcnv2_b200/workloads.py)",
            "config": config_of(args.workload, dist.world, batch_rank, global_batch,
                                "strong" if strong else "weak"),
            "images_per_s": head["images_per_s"],
            "roofline": head["roofline"], "cpu_baseline": head.get("cpu_baseline"),
            "e2e": head.get("e2e"), "clocks": head["_clocks"],
            "gpu_launches": head["gpu_launches_per_step"] * steps,
            "secondary": secondary or None, "split": split,
        }
        for k in ("levels", "levels_sequential_ms"):
            if k in head:
                line[k] = head[k]
        print(json.dumps(line), flush=True)


def run_reference(args, dist):
    """The reference's own CPU implementation of the path (oracle port), rank 0 only."""
    if dist.rank != 0:
        return
    sys.path.insert(0, os.path.join(ROOT, "oracle"))
    import oracle
    strong = args.global_batch > 0
    batch_rank = (shard_range(args.global_batch, dist.world, 0)[1] if strong
                  else parts_meta(args.workload)[0][0].n)
    global_batch = args.global_batch if strong else batch_rank * dist.world
    parts = wl.workload_parts(args.workload, seed=0)
    inp_cpu = max(parts, key=lambda p: p.layer.flops)   # the dominant layer of a step
    L = inp_cpu.layer
    threads = os.cpu_count() or 1
    x, off, msk, w, b = [t[:1].float().numpy() if i < 3 else t.float().numpy()
                         for i, t in enumerate(inp_cpu.tensors())]
    prec = "fp16" if inp_cpu.precision == "fp16" else "fp32"
    P = L.ho * L.wo
    per_px = 2 * L.out_c * L.c * L.kernel ** 2
    budget = 150.0 / max(1, args.steps + args.warmup)  # seconds per step
    t0 = time.perf_counter()
    oracle.forward_ref_band(x, off, msk, w, b, 0, 16, L.stride, L.padding, L.dilation, L.groups,
                            precision=prec, threads=threads)
    per16 = time.perf_counter() - t0
    band = int(max(1, min(P, 16 * budget / max(per16, 1e-6))))
    p0 = 0
    for _ in range(args.warmup):
        oracle.forward_ref_band(x, off, msk, w, b, 0, band, L.stride, L.padding, L.dilation,
                                L.groups, precision=prec, threads=threads)
    t0 = time.perf_counter()
    for _ in range(args.steps):
        p1 = min(P, p0 + band)
        oracle.forward_ref_band(x, off, msk, w, b, p0, p1, L.stride, L.padding, L.dilation,
                                L.groups, precision=prec, threads=threads)
        p0 = 0 if p1 >= P else p1
    el = time.perf_counter() - t0
    value = per_px * band * args.steps / el / 1e12
    unit = unit_of(inp_cpu.precision)
    line = {
        "impl": "reference",
        "metric": metric_of(args.workload),
        "value": round(value, 6), "unit": unit, "n_gpus": dist.world, "steps": args.steps,
        "warmup": args.warmup, "ms_per_step": round(el / args.steps * 1e3, 3),
        "higher_is_better": True, "scaling": "strong" if strong else "weak",
        "vs_baseline": None, "dtype": parts_meta(args.workload)[1],
        "data": "synthetic (seeded torch.Generator, dcnv2_b200/workloads.py)",
        "config": config_of(args.workload, dist.world, batch_rank, global_batch,
                            "strong" if strong else "weak"),
        "cpu_baseline": {"value": round(value, 6), "unit": unit, "cores": threads,
                         "kind": "port",
                         "sample": f"{band} output pixels of image 0 per step, "
                                   f"{inp_cpu.precision} reference semantics (the oracle's "
                                   f"restatement of src/dcn_kernel.cu + the GEMM), "
                                   f"{threads} threads"},
        "e2e": {"value": round(value, 6), "unit": unit, "h2d_bytes_per_step": 0,
                "d2h_bytes_per_step": 0},
    }
    # The reference's own GPU path (im2col + cuBLAS), when its sm_100a build is present: one
    # enqueue per image (its N=1 fast path), the cuBLAS handle created once, CUDA events on the
    # stream the launches go to.
    if oracle.ref_gpu_available() and torch.cuda.is_available() and L.groups == 1:
        try:
            dev = torch.device("cuda:0")
            torch.cuda.set_device(dev)
            inp = inp_cpu.to(dev)
            t = list(inp.tensors())
            for _ in range(3):
                oracle.ref_gpu_forward(*t, stride=L.stride, padding=L.padding,
                                       dilation=L.dilation, x_scale=inp.x_scale,
                                       w_scale=inp.w_scale)
            torch.cuda.synchronize()
            reps = 10
            st = torch.cuda.current_stream(dev)
            e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
            e0.record(st)
            for _ in range(reps):
                oracle.ref_gpu_forward(*t, stride=L.stride, padding=L.padding,
                                       dilation=L.dilation, x_scale=inp.x_scale,
                                       w_scale=inp.w_scale)
            e1.record(st)
            torch.cuda.synchronize()
            rms = e0.elapsed_time(e1) / reps
            line["reference_gpu"] = {"value": round(inp.layer.flops / (rms * 1e-3) / 1e12, 2),
                                     "unit": unit, "ms_per_step": round(rms, 3),
                                     "what": "reference im2col + cuBLAS + bias kernels on this "
                                             "B200, one image per enqueue (its N=1 fast path), "
                                             f"{inp.layer.n} images"}
        except Exception as e:  # report, do not fail the CPU arm
            line["reference_gpu"] = {"unavailable": str(e)[:200]}
    print(json.dumps(line), flush=True)


def main():
    args = parse_args()
    dist = Dist()
    if args.impl == "reference":
        run_reference(args, dist)
        return
    dist.init("nccl")
    try:
        if args.head:
            device = torch.device(f"cuda:{dist.local}")
            torch.cuda.set_device(device)
            r = measure_head(dist, device, torch.cuda.Stream(device), args.steps, 0.0,
                             n=args.batch or None)
            if dist.rank == 0:
                print(json.dumps({"metric": "DCNv2 layer with offset/mask head, fp16",
                                  "n_gpus": dist.world, "steps": args.steps, **r}), flush=True)
            return
        run_ours(args, dist)
    finally:
        dist.close()


if __name__ == "__main__":
    main()

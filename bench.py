"""DCNv2 forward benchmark (one JSON line on rank 0).

  python bench.py [--gpus N] [--steps K] [--warmup W] [--impl ours|reference] [--workload NAME]

A step is one forward of the DCNv2 layer over one batch of seeded synthetic input (the
dcnv2_b200.workloads table; default fp16_n64_256c_64: N=64, C=O=256, 64x64, 3x3, fp16). With
N GPUs (torchrun, one process per GPU) every rank runs its own batch of the same size: the
batch-sharded layer has no exchange step, so there is no collective on the data path and the
scaling is weak. Timing: W untimed steps; K steps between barriers and device synchronisation,
CUDA events on the launching stream, max over ranks. The inputs (x 134 MB, y 134 MB in fp16)
exceed the 126 MB L2, so no flush is needed between steps.

Extra keys: roofline (dominant kernel, live CUDA-event timing of each launch), cpu_baseline
(the oracle's CPU restatement on a bounded sample, rank 0 at N=1), e2e (host buffers through the
C ABI's host-buffer forward dcnv2_forward_host: every input uploaded and y downloaded inside the
timed region, in image chunks overlapped with the compute), clocks (nvidia-smi sampled during the
timed region), gpu_launches, secondary (int8 layer of the same shape).

--impl reference times the reference's own CPU implementation of the path (the oracle port of
src/dcn_kernel.cu + the reference GEMM, all host threads) on the same workload, each step a
bounded band of output pixels; it also reports the reference's GPU path (its im2col + cuBLAS
kernels built for sm_100a) under "reference_gpu" when that build is present.
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

from dcnv2_b200 import workloads as wl  # noqa: E402

PROFILE_TRAFFIC = os.path.join(ROOT, "profiles", "traffic.txt")


def parse_args():
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=3000)
    ap.add_argument("--warmup", type=int, default=20)
    ap.add_argument("--impl", default="ours", choices=["ours", "reference"])
    ap.add_argument("--workload", default="fp16_n64_256c_64", choices=list(wl.WORKLOADS))
    ap.add_argument("--e2e-steps", type=int, default=20)
    ap.add_argument("--cpu-seconds", type=float, default=12.0)
    ap.add_argument("--no-cpu-baseline", action="store_true")
    ap.add_argument("--no-secondary", action="store_true")
    return ap.parse_args()


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
            torch.distributed.init_process_group(backend, timeout=datetime.timedelta(seconds=120))
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

    def __init__(self, gpu_index: int):
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
    try:
        with open(os.path.join(ROOT, "MEASURED_PEAKS.json")) as f:
            d = json.load(f)
        return d.get("bf16_tflops", 1590.0), d.get("hbm_gbs", 6650.0), "measured"
    except OSError:
        return 1590.0, 6650.0, "fallback"


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


def flops_of(inp: "wl.Inputs") -> int:
    return inp.layer.flops


def step_fn(inp, ws, out, math=0):
    """One forward through the public C ABI on the current stream."""
    from dcnv2_b200 import capi
    L = inp.layer
    dt = {"fp32": capi.DType.FLOAT, "fp16": capi.DType.HALF, "int8": capi.DType.INT8}[inp.precision]
    desc = capi.make_desc(L.n, L.c, L.h, L.w, L.out_c, L.kernel, L.stride, L.padding, L.dilation,
                          L.groups, dt, math)
    ptrs = [t.data_ptr() for t in inp.tensors()]

    def run(stream):
        st = capi.forward_raw(desc, *ptrs, out.data_ptr(), ws.data_ptr(), ws.numel(),
                              inp.x_scale, inp.w_scale, stream)
        if st != 0:
            raise RuntimeError(f"dcnv2_forward failed: {capi.status_string(st)}")
    return desc, ptrs, run


def alloc_for(inp, device):
    from dcnv2_b200 import capi
    L = inp.layer
    dt = {"fp32": capi.DType.FLOAT, "fp16": capi.DType.HALF, "int8": capi.DType.INT8}[inp.precision]
    desc = capi.make_desc(L.n, L.c, L.h, L.w, L.out_c, L.kernel, L.stride, L.padding, L.dilation,
                          L.groups, dt)
    ws = torch.empty(capi.workspace_size(desc), dtype=torch.uint8, device=device)
    ydt = torch.float16 if inp.precision == "fp16" else torch.float32
    out = torch.empty((L.n, L.out_c, L.ho, L.wo), dtype=ydt, device=device)
    return ws, out


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


def kernel_breakdown(inp, ws, out, stream, steps):
    """Per-launch CUDA-event timing of one forward (events recorded between the launches)."""
    from dcnv2_b200 import capi
    desc, ptrs, _ = step_fn(inp, ws, out)
    n = capi.launch_count(desc)
    evs = [[torch.cuda.Event(enable_timing=True) for _ in range(n + 1)] for _ in range(steps)]
    for row in evs:  # torch creates the cudaEvent_t on first record
        for e in row:
            e.record(stream)
    torch.cuda.synchronize()
    for i in range(steps):
        st = capi.forward_events_raw(desc, *ptrs, out.data_ptr(), ws.data_ptr(), ws.numel(),
                                     inp.x_scale, inp.w_scale, stream.cuda_stream,
                                     [e.cuda_event for e in evs[i]])
        if st != 0:
            raise RuntimeError(capi.status_string(st))
    torch.cuda.synchronize()
    per = np.array([[evs[i][k].elapsed_time(evs[i][k + 1]) for k in range(n)]
                    for i in range(steps)])
    return per.mean(axis=0)  # ms per launch slot


def e2e_measure(inp_host, device, stream, steps, dist):
    """Host buffers in, host buffer out, through the C ABI's host-buffer forward
    (dcnv2_forward_host): per step the weight and bias are copied to the device and x, offset and
    mask are uploaded, computed and y downloaded in chunks of images with the copies overlapped.
    Every byte of every input crosses to the device and y comes back inside the timed region."""
    from dcnv2_b200 import capi
    from dcnv2_b200.plugin import _dtype_of
    L = inp_host.layer
    host = [t.contiguous().pin_memory() for t in inp_host.tensors()]  # x, offset, mask, w, b
    dt = _dtype_of(host[0])
    desc = capi.make_desc(L.n, L.c, L.h, L.w, L.out_c, L.kernel, L.stride, L.padding,
                          L.dilation, L.groups, dt)
    oshape = capi.output_shape(desc)
    ydt = torch.float16 if dt == capi.DType.HALF else torch.float32
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
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    e0.record(stream)
    for _ in range(steps):
        step()
    e1.record(stream)
    torch.cuda.synchronize()
    dist.barrier()
    ms = dist.max(e0.elapsed_time(e1) / steps)
    return ms, h2d, d2h


def cpu_baseline(inp_cpu, seconds: float):
    """The oracle's CPU restatement (reference fast-path semantics), all host threads, on a
    bounded band of output pixels of image 0; returns (TFLOP/s, description, threads)."""
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
    tflops = per_px * done / el / 1e12
    return tflops, f"{done} output pixels of the {wl_name(inp_cpu)} layer (image 0), " \
                   f"{prec} reference semantics, {el:.1f} s", threads


def wl_name(inp):
    L = inp.layer
    return f"{L.c}->{L.out_c} {L.h}x{L.w} k{L.kernel} {inp.precision}"


def torchvision_cpu(inp_cpu, seconds: float):
    """torchvision.ops.deform_conv2d fp32 on the host cores for one image (the reference's
    oracle path), TFLOP/s."""
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
    return {"value": per_img * n / el / 1e12, "unit": "TFLOP/s", "cores": os.cpu_count(),
            "sample": f"{n} x 1 image fp32, {el:.1f} s"}


# ---------------------------------------------------------------- arms
L2_BYTES = 126 * 1024 * 1024


def time_steps_flushed(runs, stream, steps, dist, flush):
    """Per-step CUDA-event timing with the L2 flushed (a write larger than L2) before each step;
    the flush is outside the events. Returns ms per step and ms per part of a step."""
    torch.cuda.synchronize()
    dist.barrier()
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
    for i in range(steps):
        per_part += [evs[i][k].elapsed_time(evs[i][k + 1]) for k in range(len(runs))]
    per_part /= steps
    return float(per_part.sum()), per_part


def run_ours(args, dist):
    device = torch.device(f"cuda:{dist.local}")
    torch.cuda.set_device(device)
    stream = torch.cuda.Stream(device)
    from dcnv2_b200 import capi
    parts_cpu = wl.workload_parts(args.workload, seed=1000 * dist.rank)
    parts = [p.to(device) for p in parts_cpu]
    bufs = [alloc_for(p, device) for p in parts]
    fns = [step_fn(p, ws, out) for p, (ws, out) in zip(parts, bufs)]
    runs = [f[2] for f in fns]
    launches = sum(capi.launch_count(f[0]) for f in fns)
    # the dominant layer (most FLOPs) carries the roofline, the CPU baseline and e2e details
    dom = max(range(len(parts)), key=lambda i: parts[i].layer.flops)
    inp, inp_cpu = parts[dom], parts_cpu[dom]
    (ws, out), (desc, _, _) = bufs[dom], fns[dom]
    step_bytes = sum(p.input_bytes + p.output_bytes for p in parts)
    flush = None
    if step_bytes < 2 * L2_BYTES:  # small working set: flush L2 between timed steps
        flush = torch.empty(2 * L2_BYTES // 4, dtype=torch.float32, device=device)

    def run_all(st):
        for r in runs:
            r(st)

    try:  # nvidia-smi addresses the physical GPU; torch's index may be remapped
        gpu_id = "GPU-" + str(torch.cuda.get_device_properties(device).uuid)
    except Exception:
        gpu_id = str(dist.local)
    clocks = ClockSampler(gpu_id)
    # warm-up, then the timed region with clock sampling around it
    for _ in range(args.warmup):
        run_all(stream.cuda_stream)
    torch.cuda.synchronize()
    clocks.start()
    time.sleep(0.3)
    part_ms = None
    if len(parts) > 1:
        # several layers per step (the FPN levels): one CUDA graph of all of them, each on its
        # own stream so the small levels run beside each other (dcnv2_b200.levels)
        from dcnv2_b200.levels import LevelsRunner
        runner = LevelsRunner([dict(x=p.x, offset=p.offset, mask=p.mask, weight=p.weight,
                                    bias=p.bias, stride=p.layer.stride, padding=p.layer.padding,
                                    dilation=p.layer.dilation,
                                    deformable_groups=p.layer.groups) for p in parts])
        grouped = [lambda _h: runner.run(stream)]
        if flush is None:
            ms = time_steps(grouped[0], stream, args.steps, 0, dist)
        else:
            ms, _ = time_steps_flushed(grouped, stream, args.steps, dist, flush)
    elif flush is None:
        ms = time_steps(run_all, stream, args.steps, 0, dist)
    else:
        ms, _ = time_steps_flushed(runs, stream, args.steps, dist, flush)
    clk = clocks.stop()
    ms = dist.max(ms)
    if len(parts) > 1:  # each level alone, one after another (breakdown only)
        if flush is None:
            flush = torch.empty(2 * L2_BYTES // 4, dtype=torch.float32, device=device)
        _, part_ms = time_steps_flushed(runs, stream, min(args.steps, 200), dist, flush)

    flops = sum(p.layer.flops for p in parts)
    int8 = inp.precision == "int8"
    value = flops * dist.world / (ms * 1e-3) / 1e12

    # per-kernel breakdown (live CUDA events between launches), dominant kernel roofline
    per = kernel_breakdown(inp, ws, out, stream, min(args.steps, 200))
    kname = capi.main_kernel(desc)
    main_ms = float(per[-1])
    peak_tf, peak_hbm, peak_kind = peaks()
    tensor_peak = peak_tf * (2.0 if int8 else 1.0)
    if inp.precision == "fp32":
        tensor_peak = None
    achieved = inp.layer.flops / (main_ms * 1e-3) / 1e12
    traffic = traffic_for(args.workload, kname)
    unit = "TOP/s" if int8 else "TFLOP/s"
    spec_peak = 4500.0 if int8 else 2250.0  # B200 dense tensor peaks (no 2:4 sparsity)
    if tensor_peak:
        roof = {"bound": "tensor", "achieved": round(achieved, 1), "peak": round(tensor_peak, 1),
                "unit": unit, "frac": round(achieved / tensor_peak, 4),
                "frac_spec": round(achieved / spec_peak, 4),
                "traffic": traffic, "kernel": kname, "kernel_ms": round(main_ms, 4),
                "peak_source": f"{peak_kind} bf16 dense"
                               + (" x2 (int8 dense rate)" if int8 else "")}
    else:
        roof = {"bound": "fp32 CUDA cores", "achieved": round(achieved, 1), "peak": None,
                "unit": unit, "frac": None, "traffic": traffic, "kernel": kname,
                "kernel_ms": round(main_ms, 4)}
    roof["launch_ms"] = [round(float(v), 4) for v in per]
    alg_bytes = inp.input_bytes + inp.output_bytes
    roof["hbm_alg_gbs"] = round(alg_bytes / (float(per.sum()) * 1e-3) / 1e9, 1)

    # end to end through the C ABI with host buffers
    e2e_ms, h2d, d2h = 0.0, 0, 0
    for p in parts_cpu:
        m, i_b, o_b = e2e_measure(p, device, stream, args.e2e_steps, dist)
        e2e_ms, h2d, d2h = e2e_ms + m, h2d + i_b, d2h + o_b
    e2e = {"value": round(flops * dist.world / (e2e_ms * 1e-3) / 1e12, 3), "unit": unit,
           "ms_per_step": round(e2e_ms, 3), "h2d_bytes_per_step": h2d, "d2h_bytes_per_step": d2h}

    secondary = {}
    if not args.no_secondary and args.workload == "fp16_n64_256c_64":
        s_inp = wl.workload("int8_n64_256c_64", seed=1000 * dist.rank).to(device)
        s_ws, s_out = alloc_for(s_inp, device)
        _, _, s_run = step_fn(s_inp, s_ws, s_out)
        s_ms = dist.max(time_steps(s_run, stream, max(50, args.steps // 10), 5, dist))
        s_per = kernel_breakdown(s_inp, s_ws, s_out, stream, 50)
        s_ach = flops_of(s_inp) / (float(s_per[-1]) * 1e-3) / 1e12
        secondary["int8_n64_256c_64"] = {
            "value": round(flops_of(s_inp) * dist.world / (s_ms * 1e-3) / 1e12, 1),
            "unit": "TOP/s", "ms_per_step": round(s_ms, 4),
            "fused_kernel_ms": round(float(s_per[-1]), 4),
            "tensor_frac": round(s_ach / (2 * peak_tf), 4)}
        del s_inp, s_ws, s_out

    cpu = None
    if dist.rank == 0 and dist.world == 1 and not args.no_cpu_baseline:
        v, sample, thr = cpu_baseline(inp_cpu, args.cpu_seconds)
        cpu = {"value": round(v, 5), "unit": unit, "cores": thr, "kind": "port",
               "sample": sample}
        tv = torchvision_cpu(inp_cpu, min(args.cpu_seconds, 20.0))
        if tv:
            cpu["torchvision"] = tv

    if dist.rank == 0:
        L = inp.layer
        if args.workload == "fp16_n64_256c_64":
            metric = "DCNv2 fwd TFLOP/s (256ch 64x64 3x3) fp16, 1-8 B200"
        else:
            metric = f"DCNv2 fwd {unit} ({args.workload}), 1-8 B200"
        l2 = ("step working set exceeds L2 (no flush)" if flush is None else
              "L2 flushed before every timed step (a 252 MB write outside the timed events)")
        config = {"workload": args.workload, "batch_per_gpu": L.n,
                  "global_batch": L.n * dist.world, "c": L.c, "out_c": L.out_c,
                  "hw": [L.h, L.w], "kernel": L.kernel, "stride": L.stride,
                  "padding": L.padding, "dilation": L.dilation,
                  "deformable_groups": L.groups, "parallelism": f"batch-shard x{dist.world}",
                  "l2": l2}
        if len(parts) > 1:
            config["levels_hw"] = [p.layer.h for p in parts]
        line = {
            "metric": metric,
            "value": round(value, 2), "unit": unit, "n_gpus": dist.world,
            "steps": args.steps, "warmup": args.warmup, "ms_per_step": round(ms, 4),
            "higher_is_better": True, "scaling": "weak", "vs_baseline": None,
            "dtype": inp.precision, "data": "synthetic (seeded torch.Generator, see workloads.py)",
            "config": config,
            "images_per_s": round(L.n * dist.world / (ms * 1e-3), 1),
            "roofline": roof, "cpu_baseline": cpu, "e2e": e2e, "clocks": clk,
            "gpu_launches": launches * args.steps, "secondary": secondary or None,
        }
        if part_ms is not None and len(parts) > 1:
            line["levels"] = [{"hw": p.layer.h, "ms_alone": round(float(m), 4),
                               "tflops_alone": round(p.layer.flops / (m * 1e-3) / 1e12, 1)}
                              for p, m in zip(parts, part_ms)]
            line["levels_sequential_ms"] = round(float(sum(part_ms)), 4)
            config["step"] = ("the five levels as one CUDA graph, one stream per level "
                              "(dcnv2_b200.levels.LevelsRunner)")
        print(json.dumps(line), flush=True)


def run_reference(args, dist):
    if dist.rank != 0:
        return
    sys.path.insert(0, os.path.join(ROOT, "oracle"))
    import oracle
    inp_cpu = wl.workload(args.workload, seed=0)
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
    line = {
        "impl": "reference",
        "metric": "DCNv2 fwd TFLOP/s (256ch 64x64 3x3) fp16, 1-8 B200",
        "value": round(value, 6), "unit": "TFLOP/s", "n_gpus": dist.world, "steps": args.steps,
        "warmup": args.warmup, "ms_per_step": round(el / args.steps * 1e3, 3),
        "higher_is_better": True, "scaling": "weak", "vs_baseline": None,
        "dtype": inp_cpu.precision, "data": "synthetic (seeded torch.Generator, see workloads.py)",
        "config": {"workload": args.workload, "batch_per_gpu": L.n, "c": L.c, "out_c": L.out_c,
                   "hw": [L.h, L.w], "kernel": L.kernel},
        "cpu_baseline": {"value": round(value, 6), "unit": "TFLOP/s", "cores": threads,
                         "kind": "port",
                         "sample": f"{band} output pixels of image 0 per step, "
                                   f"{prec} reference semantics"},
        "e2e": {"value": round(value, 6), "unit": "TFLOP/s", "h2d_bytes_per_step": 0,
                "d2h_bytes_per_step": 0},
    }
    # The reference's own GPU path (im2col + cuBLAS), when its sm_100a build is present.
    if oracle.ref_gpu_available() and torch.cuda.is_available():
        try:
            dev = torch.device("cuda:0")
            inp = inp_cpu.to(dev)
            t = list(inp.tensors())
            for _ in range(3):
                oracle.ref_gpu_forward(*t, stride=L.stride, padding=L.padding,
                                       dilation=L.dilation, x_scale=inp.x_scale,
                                       w_scale=inp.w_scale)
            torch.cuda.synchronize()
            reps = 10
            e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
            e0.record()
            for _ in range(reps):
                oracle.ref_gpu_forward(*t, stride=L.stride, padding=L.padding,
                                       dilation=L.dilation, x_scale=inp.x_scale,
                                       w_scale=inp.w_scale)
            e1.record()
            torch.cuda.synchronize()
            rms = e0.elapsed_time(e1) / reps
            line["reference_gpu"] = {"value": round(L.flops / (rms * 1e-3) / 1e12, 2),
                                     "unit": "TFLOP/s", "ms_per_step": round(rms, 3),
                                     "what": "reference im2col + cuBLAS + bias kernels on this "
                                             "B200, one image per enqueue (its N=1 fast path)"}
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
        run_ours(args, dist)
    finally:
        dist.close()


if __name__ == "__main__":
    main()

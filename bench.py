"""Benchmark of batched use_model: inference samples/s on 1..8 B200s.

One step = one batched use_model over the workload's batch of synthetic samples
on every GPU (weak scaling: each rank runs the full per-GPU batch on its own
GPU; samples are sharded, weights replicated, no collective on the data path).

  value     samples/s of the whole job, inputs resident in HBM, timed with CUDA
            events on the launching stream (max over ranks)
  e2e       the same through the host-array C-ABI call (rosenna_use_model_f32):
            H2D of the step's inputs from pinned memory, kernels, D2H of outputs
  roofline  the dominant kernel's achieved FLOP/s against the measured FP32 peak
            (cuBLAS SGEMM with TF32 off, timed here), plus DRAM traffic per launch
            from the committed ncu capture
  cpu_baseline  the fp64 oracle (a C restatement of roseNNa's Fortran path,
            use_model once per sample, all host threads) on a bounded sample

Default workload: the wide MLP (16-256x5-8, ReLU), batch 4,194,304 per GPU.
`--impl reference` times roseNNa's algorithm on the host cores instead.
"""
import argparse
import json
import os
import statistics
import threading
import subprocess
import sys
import tempfile
import time

ROOT = os.path.dirname(os.path.abspath(__file__))
sys.path.insert(0, ROOT)

# DRAM bytes (read + write) per launch of the dominant kernel, from the ncu
# capture summarised in profiles/ (None until captured).
# DRAM bytes (read + write) per sample of the dominant kernel, from the
# committed ncu captures (profiles/); scaled by the batch for `traffic`
NCU_TRAFFIC_PER_SAMPLE = {
    ("wide_mlp", "mlp_tc_kernel"): (69.486592e6 + 10.319616e6) / 1048576,
}

DEFAULT_WORKLOAD = "wide_mlp"


def parse():
    p = argparse.ArgumentParser()
    p.add_argument("--gpus", type=int, default=1)
    p.add_argument("--steps", type=int, default=20)
    p.add_argument("--warmup", type=int, default=5)
    p.add_argument("--impl", choices=["ours", "reference"], default="ours")
    p.add_argument("--workload", default=DEFAULT_WORKLOAD)
    p.add_argument("--batch", type=int, default=0, help="per-GPU batch (default: the workload's)")
    p.add_argument("--no-cpu-baseline", action="store_true")
    return p.parse_args()


def cpu_baseline(name, model_dir, target_seconds=12.0, steps=1):
    """fp64 oracle, use_model once per sample over all host threads."""
    from oracle import oracle as O
    from rosenna_b200 import workloads

    m = O.OracleModel(model_dir)
    threads = O.max_threads()
    # calibrate on a small sample, then size the sample for ~target_seconds
    n = max(64, threads * 8)
    ins = workloads.make_inputs(name, n, seed_offset=99)
    t0 = time.perf_counter()
    m.run_batched(n, ins, [1] * len(ins), [1], threads)
    dt = time.perf_counter() - t0
    n = int(max(threads, min(1 << 22, n * target_seconds / max(dt, 1e-6) / steps)))
    ins = workloads.make_inputs(name, n, seed_offset=98)
    rates = []
    for _ in range(steps):
        t0 = time.perf_counter()
        m.run_batched(n, ins, [1] * len(ins), [1], threads)
        rates.append(n / (time.perf_counter() - t0))
    return {"value": statistics.median(rates), "unit": "samples/s", "cores": threads, "kind": "port",
            "sample": f"{n} samples of the workload per step, fp64, use_model per sample (C restatement of "
                      f"fLibrary/layers.f90; no Fortran compiler in the image)"}


class ClockSampler:
    """SM clock and clock-event (throttle) reasons, polled through NVML every
    10 ms on a background thread during the timed region (plus one sample at
    each end), so that even a timed region of a few ms has samples."""

    # NVML clocks-event reason bits
    REASONS = {"hw_slowdown": 0x8, "hw_thermal_slowdown": 0x40, "sw_thermal_slowdown": 0x20, "sw_power_cap": 0x4}

    def __init__(self, dev):
        self.dev = dev
        self.samples = []
        self.stop = threading.Event()
        self.nvml = None
        self.handle = None

    def _open(self):
        try:
            import pynvml
            pynvml.nvmlInit()
            self.nvml = pynvml
            try:
                import torch
                pr = torch.cuda.get_device_properties(self.dev)
                bus = f"{pr.pci_domain_id:08x}:{pr.pci_bus_id:02x}:{pr.pci_device_id:02x}.0"
                self.handle = pynvml.nvmlDeviceGetHandleByPciBusId(bus)
            except Exception:
                self.handle = pynvml.nvmlDeviceGetHandleByIndex(self.dev)
        except Exception:
            self.nvml = self.handle = None

    def _sample(self):
        n, h = self.nvml, self.handle
        try:
            sm = n.nvmlDeviceGetClockInfo(h, n.NVML_CLOCK_SM)
            mx = n.nvmlDeviceGetMaxClockInfo(h, n.NVML_CLOCK_SM)
            try:
                r = n.nvmlDeviceGetCurrentClocksEventReasons(h)
            except AttributeError:
                r = n.nvmlDeviceGetCurrentClocksThrottleReasons(h)
            self.samples.append((sm, mx, r))
        except Exception:
            pass

    def _run(self):
        while not self.stop.wait(0.01):
            self._sample()

    def __enter__(self):
        self._open()
        if self.handle is not None:
            self._sample()
            self.thread = threading.Thread(target=self._run, daemon=True)
            self.thread.start()
        return self

    def __exit__(self, *a):
        if self.handle is not None:
            self.stop.set()
            self.thread.join(timeout=5)
            self._sample()

    def summary(self):
        if not self.samples:
            return {"sm_mhz": None, "sm_max_mhz": None, "reasons": [], "samples": 0, "source": "nvml unavailable"}
        reasons = sorted(k for k, bit in self.REASONS.items() if any(r & bit for _, _, r in self.samples))
        return {"sm_mhz": statistics.median(s for s, _, _ in self.samples),
                "sm_max_mhz": max(m for _, m, _ in self.samples), "reasons": reasons,
                "samples": len(self.samples), "source": "NVML, 10 ms polling"}


def measured_peaks():
    try:
        with open(os.path.join(ROOT, "MEASURED_PEAKS.json")) as f:
            return json.load(f)
    except (OSError, ValueError):
        return {}


def measured_fp32_peak(torch):
    """cuBLAS SGEMM (TF32 off), 8192^3, best of 5: the FP32 FFMA denominator."""
    prev = torch.backends.cuda.matmul.allow_tf32
    torch.backends.cuda.matmul.allow_tf32 = False
    a = torch.randn(8192, 8192, device="cuda")
    b = torch.randn(8192, 8192, device="cuda")
    for _ in range(2):
        torch.mm(a, b)
    best = 0.0
    for _ in range(5):
        e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        e0.record()
        torch.mm(a, b)
        e1.record()
        torch.cuda.synchronize()
        best = max(best, 2 * 8192 ** 3 / (e0.elapsed_time(e1) / 1e3))
    torch.backends.cuda.matmul.allow_tf32 = prev
    del a, b
    torch.cuda.empty_cache()
    return best / 1e12


def run_reference(args):
    from rosenna_b200 import ranks

    rank, _, world = ranks.env()
    if rank != 0:
        return
    from rosenna_b200 import workloads

    w = workloads.WORKLOADS[args.workload]
    with tempfile.TemporaryDirectory() as d:
        workloads.write_model(args.workload, d)
        cb = cpu_baseline(args.workload, d, target_seconds=max(2.0, 60.0 / max(1, args.steps + args.warmup)),
                          steps=max(1, args.steps))
    line = {"metric": "inference samples/sec (batched use_model)", "value": cb["value"], "unit": "samples/s",
            "n_gpus": args.gpus, "steps": args.steps, "warmup": args.warmup, "ms_per_step": None,
            "higher_is_better": True, "scaling": "weak", "vs_baseline": None, "dtype": "f64", "data": "synthetic",
            "impl": "reference",
            "config": {"workload": f"{w.name}: {w.description}", "batch_per_gpu": w.batch,
                       "parallelism": "host cores (use_model per sample)"},
            "cpu_baseline": cb,
            "e2e": {"value": cb["value"], "unit": "samples/s", "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0}}
    print(json.dumps(line), flush=True)


def main():
    args = parse()
    if args.impl == "reference":
        run_reference(args)
        return
    import torch
    import torch.distributed as dist

    from rosenna_b200 import api, ranks, workloads

    rank, local, world = ranks.env()
    torch.cuda.set_device(local)
    if world > 1:
        import datetime

        dist.init_process_group("nccl", timeout=datetime.timedelta(seconds=120),
                                device_id=torch.device("cuda", local))
    w = workloads.WORKLOADS[args.workload]
    n = args.batch or w.batch
    tmp = tempfile.TemporaryDirectory()
    workloads.write_model(args.workload, tmp.name)
    api.set_devices([local])
    api.initialize(tmp.name)
    ins = workloads.make_inputs_torch(args.workload, n, device="cuda", seed_offset=rank)
    outs = [torch.empty((r, n), dtype=torch.float32, device="cuda") for r in w.output_rows]
    in_ptrs, out_ptrs = [x.data_ptr() for x in ins], [o.data_ptr() for o in outs]
    stream = torch.cuda.current_stream()

    def barrier():
        if world > 1:
            dist.barrier()

    # ---- device-resident throughput ----
    for _ in range(max(3, args.warmup)):
        api.use_model_device(n, in_ptrs, out_ptrs, stream.cuda_stream)
    torch.cuda.synchronize()
    barrier()
    torch.cuda.synchronize()
    launches = 0
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    with ClockSampler(local) as clk:
        e0.record(stream)
        for _ in range(args.steps):
            api.use_model_device(n, in_ptrs, out_ptrs, stream.cuda_stream)
            launches += api.last_launch_count()
        e1.record(stream)
        torch.cuda.synchronize()
    t_dev = ranks.max_over_ranks(e0.elapsed_time(e1) / 1e3)
    barrier()
    torch.cuda.synchronize()
    value = world * n * args.steps / t_dev
    plan = api.plan_description()
    launches_per_step = launches // max(1, args.steps)

    # ---- end to end through the host-array C ABI (pinned host buffers) ----
    h_in = [x.cpu().pin_memory() for x in ins]
    h_out = [torch.empty((r, n), dtype=torch.float32).pin_memory() for r in w.output_rows]
    hi, ho = [x.data_ptr() for x in h_in], [o.data_ptr() for o in h_out]
    api.use_model_ptrs(n, hi, ho)
    barrier()
    t0 = time.perf_counter()
    for _ in range(args.steps):
        api.use_model_ptrs(n, hi, ho)
    t_e2e = ranks.max_over_ranks(time.perf_counter() - t0)
    e2e = {"value": world * n * args.steps / t_e2e, "unit": "samples/s",
           "h2d_bytes_per_step": sum(x.numel() * 4 for x in h_in), "d2h_bytes_per_step": sum(o.numel() * 4 for o in h_out),
           "api": "rosenna_use_model_f32 (host arrays, pinned)"}
    ok_out = bool(torch.isfinite(h_out[0]).all())
    # the link's own ceiling for this step: a plain pinned H2D copy of the same inputs
    d_tmp = [torch.empty_like(x) for x in ins]
    torch.cuda.synchronize()
    t0 = time.perf_counter()
    for _ in range(3):
        for dst, src in zip(d_tmp, h_in):
            dst.copy_(src, non_blocking=True)
    torch.cuda.synchronize()
    h2d_gbs = 3 * e2e["h2d_bytes_per_step"] / (time.perf_counter() - t0) / 1e9
    e2e["plain_h2d_gbs"] = h2d_gbs
    e2e["h2d_bound_samples_s"] = h2d_gbs * 1e9 / (e2e["h2d_bytes_per_step"] / n) * world
    del d_tmp

    # ---- roofline of the dominant kernel ----
    kernel_s = t_dev / max(1, args.steps * launches_per_step) if launches_per_step == 1 else None
    achieved = (w.flops_per_sample * n) / kernel_s / 1e12 if kernel_s else None
    if "mlp_tc" in plan:
        # 3xTF32: three TF32 tensor products per fp32 MAC; TF32 runs at half the bf16 rate
        peaks = measured_peaks()
        bf16 = peaks.get("bf16_tflops")
        src = "MEASURED_PEAKS.json" if bf16 else "fallback 1590 TFLOP/s bf16 burst"
        bf16 = bf16 or 1590.0
        peak = bf16 / 2.0 / 3.0
        roof = {"bound": "tensor", "kernel": "mlp_tc_kernel", "achieved": achieved, "peak": peak,
                "unit": "TFLOP/s", "frac": (achieved / peak) if achieved else None,
                "peak_source": f"{src}: bf16 {bf16:.0f} TFLOP/s burst / 2 (TF32 rate) / 3 (3xTF32), of measured",
                "tensor_pipe_frac": (achieved * 6.0 / bf16) if achieved else None}
    else:
        fp32_peak = measured_fp32_peak(torch) if rank == 0 else None
        roof = {"bound": "fp32", "kernel": "mlp_ffma_kernel" if "mlp" in args.workload else "plan",
                "achieved": achieved, "peak": fp32_peak, "unit": "TFLOP/s",
                "frac": (achieved / fp32_peak) if (achieved and fp32_peak) else None,
                "peak_source": "measured here: cuBLAS SGEMM 8192^3, TF32 off (MEASURED_PEAKS.json has no FP32 figure)"}
    per_sample = NCU_TRAFFIC_PER_SAMPLE.get((args.workload, roof["kernel"]))
    roof["traffic"] = per_sample * n if per_sample else None
    roof["traffic_unit"] = "bytes per launch (ncu capture at a smaller batch, scaled by samples)"
    roof["algorithmic_flops_per_launch"] = w.flops_per_sample * n if kernel_s else None

    if rank == 0:
        cb = None
        if world == 1 and not args.no_cpu_baseline:
            cb = cpu_baseline(args.workload, tmp.name)
        line = {"metric": "inference samples/sec (batched use_model)", "value": value, "unit": "samples/s",
                "n_gpus": world, "steps": args.steps, "warmup": args.warmup, "ms_per_step": 1e3 * t_dev / args.steps,
                "higher_is_better": True, "scaling": "weak", "vs_baseline": None, "dtype": "f32", "data": "synthetic",
                "config": {"workload": f"{w.name}: {w.description}", "batch_per_gpu": n, "global_batch": world * n,
                           "parallelism": f"dp{world} (contiguous sample shards, weights replicated, no collective)",
                           "l2": f"inputs {sum(x.numel() * 4 for x in ins) / 1e6:.0f} MB + outputs "
                                 f"{sum(o.numel() * 4 for o in outs) / 1e6:.0f} MB per step exceed the 126 MB L2",
                           "plan": plan.strip().splitlines()},
                "e2e": e2e, "gpu_launches": launches, "roofline": roof, "cpu_baseline": cb,
                "clocks": clk.summary(), "outputs_finite": ok_out}
        print(json.dumps(line), flush=True)
    api.finalize()
    if world > 1:
        dist.destroy_process_group()


if __name__ == "__main__":
    main()

"""Benchmark of batched use_model: inference samples/s on 1..8 B200s.

One step = one batched use_model over a workload's batch of synthetic samples
on every GPU (weak scaling: each rank runs the full per-GPU batch on its own
GPU; samples are sharded, weights replicated, no collective on the data path).

The JSON line's top level is the headline workload (default: the wide MLP,
16-256x5-8 ReLU, 4,194,304 samples per GPU); `workloads` holds the same
measurements for all five workloads at their full batches.  Per workload:

  value     samples/s of the whole job, inputs resident in HBM, timed with CUDA
            events on the launching stream (max over ranks)
  e2e       the same through the host-array C-ABI call (rosenna_use_model_f32):
            H2D of the step's inputs from pinned memory, kernels, D2H of outputs
  roofline  the dominant kernel (the plan step with the largest device time,
            from CUDA events the C ABI records around every step during the
            timed region): its algorithmic FLOP/s against the measured peak of
            its pipe -- tcgen05 3xTF32: the measured bf16 burst / 2 / 3; CUDA-core
            FP32: 148 SMs x 128 FMA/clk x 2 x the SM clock sampled during the
            timed region (cuBLAS SGEMM measured here is reported beside it)
  cpu_baseline  the fp64 oracle (a C restatement of roseNNa's Fortran path,
            use_model once per sample, every host core) on a bounded sample of
            the bench's own batch (N=1, rank 0)
  parity    that sample's engine outputs (device and host entry points) against
            the oracle's: max abs (limit 1e-5) and max rel (limit 1e-4, where
            |ref| >= 0.1)

`--impl reference` times roseNNa's algorithm (the oracle) on the host cores.
"""
import argparse
import json
import os
import statistics
import sys
import tempfile
import threading
import time

ROOT = os.path.dirname(os.path.abspath(__file__))
sys.path.insert(0, ROOT)

# DRAM bytes (read + write) per sample of a workload's dominant kernel, from the
# committed ncu captures (profiles/), at batches whose inputs and outputs exceed
# the 126 MB L2; `traffic` = this x the batch.
NCU_TRAFFIC_PER_SAMPLE = {
    ("wide_mlp", "mlp_tc_kernel"): (69.464576e6 + 12.883968e6) / 1048576,
    ("small_mlp", "mlp_narrow_tc_kernel"): (42.096896e6 + 0.306944e6) / 1048576,
    ("lstm", "lstm_dual_tc_kernel"): (105.0368e6 + 5.318144e6) / 65536,
    ("cnn", "conv_tc_kernel"): (769.880064e6 + 190.848768e6) / 65536,  # conv2, the dominant step
    ("lstm2", "lstm2_tc_kernel"): (383.717632e6 + 14.7328e6) / 65536,
}
NCU_TRAFFIC_NOTE = {
    ("wide_mlp", "mlp_tc_kernel"): "capture at 1,048,576 samples: its 33.5 MB of outputs stayed in L2, so writes are "
                                   "under-counted",
    ("small_mlp", "mlp_narrow_tc_kernel"): "capture at 1,048,576 samples: its 21 MB of outputs stayed in L2, so "
                                           "writes are under-counted",
    ("lstm", "lstm_dual_tc_kernel"): "capture at 65,536 samples (105 MB of inputs), scaled per sample",
    ("cnn", "conv_tc_kernel"): "conv2 (8->16 channels) at the bench batch; reads are 1.9x its input because "
                               "neighbouring blocks' patches overlap and part of that reuse misses L2",
    ("lstm2", "lstm2_tc_kernel"): "capture at 65,536 samples (381 MB of inputs), scaled per sample",
}

DEFAULT_WORKLOAD = "wide_mlp"
ORDER = ["wide_mlp", "small_mlp", "lstm", "cnn", "lstm2"]
SMS, FMA_PER_CLK = 148, 128


def parse():
    p = argparse.ArgumentParser()
    p.add_argument("--gpus", type=int, default=1)
    p.add_argument("--steps", type=int, default=20)
    p.add_argument("--warmup", type=int, default=5)
    p.add_argument("--impl", choices=["ours", "reference"], default="ours")
    p.add_argument("--workload", default=DEFAULT_WORKLOAD, help="headline workload")
    p.add_argument("--workloads", default="all", help="'all', 'none' or a comma list measured besides the headline")
    p.add_argument("--batch", type=int, default=0, help="per-GPU batch of the headline (default: the workload's)")
    p.add_argument("--no-cpu-baseline", action="store_true")
    return p.parse_args()


def others(args):
    if args.workloads == "none":
        return []
    names = ORDER if args.workloads == "all" else args.workloads.split(",")
    return [x for x in names if x != args.workload]


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


def tensor_peak():
    """3xTF32 tcgen05 denominator: the measured bf16 burst / 2 (TF32 rate) / 3."""
    bf16 = measured_peaks().get("bf16_tflops")
    if bf16:
        return bf16 / 6.0, f"MEASURED_PEAKS.json bf16 burst {bf16:.1f} TFLOP/s / 2 (TF32 rate) / 3 (3xTF32), of measured"
    return 1590.0 / 6.0, ("bf16 1590 TFLOP/s (the recipe's fallback: MEASURED_PEAKS.json is absent) / 2 (TF32 rate) "
                          "/ 3 (3xTF32), of fallback")


def sgemm_tflops(torch):
    """cuBLAS SGEMM (TF32 off), 8192^3, best of 5: reported beside the FFMA pipe peak."""
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


def oracle_leg(name, model_dir, host_in, outs_by_path, target_seconds):
    """The cpu_baseline leg: the fp64 oracle on a bounded sample of the bench's
    own batch (every host core), timed, and the parity of the engine's outputs
    on that sample.  host_in: (rows, n) fp32 inputs; outs_by_path: {path: (rows,
    n) fp32 outputs of the engine}."""
    import numpy as np

    from oracle import oracle as O
    from oracle import parity

    m = O.OracleModel(model_dir)
    threads = O.host_cores()
    n = host_in[0].shape[1]
    w_key = sum(map(ord, name))
    # calibrate on the first checked indices, then size the sample for ~target_seconds
    idx0 = parity.check_indices(n, 512, seed=w_key)
    sub = [np.ascontiguousarray(x[:, idx0], dtype=np.float64) for x in host_in]
    t0 = time.perf_counter()
    m.run_batched(len(idx0), sub, threads=threads)
    rate = len(idx0) / max(time.perf_counter() - t0, 1e-6)
    count = int(min(n, max(4096, rate * target_seconds)))
    idx = parity.check_indices(n, count, seed=w_key)
    sub = [np.ascontiguousarray(x[:, idx], dtype=np.float64) for x in host_in]
    t0 = time.perf_counter()
    ref = m.run_batched(len(idx), sub, threads=threads)[0].reshape(-1, len(idx))
    dt = time.perf_counter() - t0
    par = {"samples_checked": int(len(idx)), "limits": {"max_abs": parity.ABS_TOL, "max_rel": parity.REL_TOL,
                                                        "rel_where_abs_ref_ge": parity.REL_FLOOR}}
    ok = True
    for path, out in outs_by_path.items():
        r = parity.compare(out[:, idx], ref)
        par[path] = {"max_abs": r["max_abs"], "max_rel": r["max_rel"]}
        ok = ok and r["ok"]
    par["ok"] = ok
    par["max_abs"] = max(v["max_abs"] for k, v in par.items() if k in outs_by_path)
    par["max_rel"] = max(v["max_rel"] for k, v in par.items() if k in outs_by_path)
    cb = {"value": len(idx) / dt, "unit": "samples/s", "cores": threads, "kind": "port",
          "sample": f"{len(idx)} samples of the bench batch of {n} (first/last tiles, chunk and shard boundaries, "
                    f"seeded uniform indices), fp64, use_model once per sample, {dt:.1f} s (C restatement of "
                    f"fLibrary/layers.f90; no Fortran compiler in the image)"}
    return cb, par


def measure(name, n, args, rank, local, world, want_cpu, fp32_ref):
    """Device and end-to-end samples/s of one workload, its dominant kernel's
    roofline, and (rank 0, N=1) the cpu_baseline leg with parity."""
    import numpy as np
    import torch
    import torch.distributed as dist

    from rosenna_b200 import api, ranks, workloads

    w = workloads.WORKLOADS[name]
    tmp = tempfile.TemporaryDirectory()
    workloads.write_model(name, tmp.name)
    api.initialize(tmp.name)
    ins = workloads.make_inputs_torch(name, n, device="cuda", seed_offset=rank)
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
    steps_info = api.step_info()
    api.step_timing_begin(args.steps * len(steps_info))
    launches = 0
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    with ClockSampler(local) as clk:
        e0.record(stream)
        for _ in range(args.steps):
            api.use_model_device(n, in_ptrs, out_ptrs, stream.cuda_stream)
            launches += api.last_launch_count()
        e1.record(stream)
        torch.cuda.synchronize()
    step_times = api.step_timing_end()
    t_ranks = ranks.values_over_ranks(e0.elapsed_time(e1) / 1e3)
    t_dev = max(t_ranks)
    barrier()
    torch.cuda.synchronize()
    value = world * n * args.steps / t_dev
    clocks = clk.summary()
    dev_out = [o.cpu().numpy() for o in outs] if want_cpu else None

    # ---- dominant kernel: the plan step with the most device time ----
    dom = max(range(len(step_times)), key=lambda i: step_times[i][0])
    kname, fps = steps_info[dom]
    k_ms, k_runs = step_times[dom]
    # a call may split the batch into chunks (intermediates beyond the scratch
    # budget): the step then runs once per chunk; per call it processes all n samples
    k_call_s = k_ms / 1e3 / max(1, args.steps)
    achieved = fps * n / k_call_s / 1e12 if fps > 0 else None
    if "_tc" in kname:
        peak, src = tensor_peak()
        bound = "tensor"
    else:
        mhz = clocks.get("sm_mhz") or measured_peaks().get("sm_max_mhz") or 1965.0
        peak = SMS * FMA_PER_CLK * 2 * mhz * 1e6 / 1e12
        src = (f"FP32 FFMA pipe: {SMS} SMs x {FMA_PER_CLK} FMA/clk x 2 flop x {mhz:.0f} MHz (SM clock sampled during "
               f"the timed region)")
        bound = "fp32"
    total_ms = sum(t for t, _ in step_times)
    per_sample = NCU_TRAFFIC_PER_SAMPLE.get((name, kname))
    roof = {"bound": bound, "kernel": kname, "achieved": achieved, "peak": peak, "unit": "TFLOP/s",
            "frac": achieved / peak if achieved else None, "peak_source": src,
            "kernel_ms_per_call": k_call_s * 1e3, "launches_per_call": k_runs / max(1, args.steps),
            "kernel_share": k_ms / total_ms if total_ms else None,
            "algorithmic_flops_per_launch": fps * n,
            "traffic": per_sample * n if per_sample else None,
            "traffic_unit": "DRAM bytes per launch (ncu dram__bytes_read.sum + dram__bytes_write.sum, per sample x batch)",
            "traffic_note": NCU_TRAFFIC_NOTE.get((name, kname))}
    if fp32_ref and bound == "fp32":
        roof["cublas_sgemm_tflops"] = fp32_ref
    steps_desc = [{"kernel": k, "flops_per_sample": f, "ms_per_step": t / max(1, args.steps)}
                  for (k, f), (t, _) in zip(steps_info, step_times)]

    # ---- end to end through the host-array C ABI (pinned host buffers) ----
    h_in = [torch.empty(tuple(x.shape), dtype=torch.float32, pin_memory=True).copy_(x) for x in ins]
    h_out = [torch.empty((r, n), dtype=torch.float32, pin_memory=True) for r in w.output_rows]
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
    # the link's own ceiling for this step: a plain pinned H2D copy of the same inputs
    d_tmp = [torch.empty_like(x) for x in ins]
    torch.cuda.synchronize()
    t0 = time.perf_counter()
    for _ in range(3):
        for dst, src_ in zip(d_tmp, h_in):
            dst.copy_(src_, non_blocking=True)
    torch.cuda.synchronize()
    h2d_gbs = 3 * e2e["h2d_bytes_per_step"] / (time.perf_counter() - t0) / 1e9
    e2e["plain_h2d_gbs"] = h2d_gbs
    e2e["plain_h2d_gbs_max_over_ranks"] = ranks.max_over_ranks(h2d_gbs)
    e2e["h2d_bound_samples_s"] = h2d_gbs * 1e9 / (e2e["h2d_bytes_per_step"] / n) * world
    del d_tmp

    res = {"workload": f"{w.name}: {w.description}", "batch_per_gpu": n, "value": value, "unit": "samples/s",
           "ms_per_step": 1e3 * t_dev / args.steps,
           "ms_per_step_by_rank": [round(1e3 * t / args.steps, 4) for t in t_ranks] if world > 1 else None,
           "e2e": e2e, "roofline": roof, "steps": steps_desc,
           "gpu_launches": launches, "clocks": clocks, "plan": api.plan_description().strip().splitlines(),
           "l2": f"inputs {sum(x.numel() * 4 for x in ins) / 1e6:.0f} MB + outputs "
                 f"{sum(o.numel() * 4 for o in outs) / 1e6:.0f} MB per step"}
    api.finalize()
    if want_cpu:
        host_in = [x.numpy() for x in h_in]
        cb, par = oracle_leg(name, tmp.name, host_in, {"device": dev_out[0], "host": h_out[0].numpy()},
                             12.0 if name == args.workload else 8.0)
        res["cpu_baseline"], res["parity"] = cb, par
    else:
        res["cpu_baseline"] = res["parity"] = None
    del ins, outs, h_in, h_out
    torch.cuda.empty_cache()
    tmp.cleanup()
    return res


def run_reference(args):
    from rosenna_b200 import ranks

    rank, _, world = ranks.env()
    if rank != 0:
        return
    import numpy as np

    from oracle import oracle as O
    from rosenna_b200 import workloads

    def time_oracle(name, seconds, steps):
        w = workloads.WORKLOADS[name]
        with tempfile.TemporaryDirectory() as d:
            workloads.write_model(name, d)
            m = O.OracleModel(d)
            threads = O.host_cores()
            k = max(64, threads * 8)
            ins = workloads.make_inputs(name, k, seed_offset=99)
            t0 = time.perf_counter()
            m.run_batched(k, ins, threads=threads)
            rate = k / max(time.perf_counter() - t0, 1e-6)
            k = int(max(threads, min(1 << 22, rate * seconds)))
            ins = workloads.make_inputs(name, k, seed_offset=98)
            rates = []
            for _ in range(steps):
                t0 = time.perf_counter()
                m.run_batched(k, ins, threads=threads)
                rates.append(k / (time.perf_counter() - t0))
        return {"value": statistics.median(rates), "unit": "samples/s", "cores": threads, "kind": "port",
                "sample": f"{k} samples of the workload per step (batch {w.batch}), fp64, use_model once per "
                          f"sample (C restatement of fLibrary/layers.f90; no Fortran compiler in the image)"}

    w = workloads.WORKLOADS[args.workload]
    cb = time_oracle(args.workload, max(2.0, 60.0 / max(1, args.steps + args.warmup)), max(1, args.steps))
    extra = {}
    for name in others(args):
        extra[name] = time_oracle(name, 4.0, 1)
    line = {"metric": "inference samples/sec (batched use_model)", "value": cb["value"], "unit": "samples/s",
            "n_gpus": args.gpus, "steps": args.steps, "warmup": args.warmup, "ms_per_step": None,
            "higher_is_better": True, "scaling": "weak", "vs_baseline": None, "dtype": "f64", "data": "synthetic",
            "impl": "reference",
            "config": {"workload": f"{w.name}: {w.description}", "batch_per_gpu": w.batch,
                       "parallelism": "host cores (use_model per sample)"},
            "cpu_baseline": cb,
            "e2e": {"value": cb["value"], "unit": "samples/s", "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0},
            "workloads": {k: {"value": v["value"], "unit": "samples/s", "cpu_baseline": v} for k, v in extra.items()}}
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
    # pinned host buffers on the GPU's own NUMA node when several ranks share the host
    numa = ranks.bind_host_to_device(local) if world > 1 else None
    if world > 1:
        import datetime

        dist.init_process_group("nccl", timeout=datetime.timedelta(seconds=120),
                                device_id=torch.device("cuda", local))
    api.set_devices([local])
    want_cpu = rank == 0 and world == 1 and not args.no_cpu_baseline
    fp32_ref = sgemm_tflops(torch) if rank == 0 else None
    head = measure(args.workload, args.batch or workloads.WORKLOADS[args.workload].batch, args, rank, local, world,
                   want_cpu, fp32_ref)
    rest = {}
    for name in others(args):
        rest[name] = measure(name, workloads.WORKLOADS[name].batch, args, rank, local, world, want_cpu, fp32_ref)

    if rank == 0:
        roof = dict(head["roofline"])
        line = {"metric": "inference samples/sec (batched use_model)", "value": head["value"], "unit": "samples/s",
                "n_gpus": world, "steps": args.steps, "warmup": args.warmup, "ms_per_step": head["ms_per_step"],
                "higher_is_better": True, "scaling": "weak", "vs_baseline": None, "dtype": "f32", "data": "synthetic",
                "config": {"workload": head["workload"], "batch_per_gpu": head["batch_per_gpu"],
                           "global_batch": world * head["batch_per_gpu"],
                           "parallelism": f"dp{world} (contiguous sample shards, weights replicated, no collective)",
                           "l2": head["l2"] + " exceed the 126 MB L2 (no flush needed)", "plan": head["plan"],
                           "numa_binding": numa},
                "e2e": head["e2e"], "gpu_launches": head["gpu_launches"], "roofline": roof,
                "cpu_baseline": head["cpu_baseline"], "parity": head["parity"], "clocks": head["clocks"],
                "steps_detail": head["steps"],
                "workloads": {head["workload"].split(":")[0]: {k: head[k] for k in (
                    "workload", "batch_per_gpu", "value", "ms_per_step", "ms_per_step_by_rank", "e2e", "roofline",
                    "parity", "cpu_baseline", "clocks", "gpu_launches")}}}
        for name, r in rest.items():
            line["workloads"][name] = {k: r[k] for k in ("workload", "batch_per_gpu", "value", "ms_per_step",
                                                          "ms_per_step_by_rank", "e2e",
                                                          "roofline", "parity", "cpu_baseline", "clocks",
                                                          "gpu_launches", "steps", "l2")}
        print(json.dumps(line), flush=True)
    if world > 1:
        dist.barrier()
        dist.destroy_process_group()


if __name__ == "__main__":
    main()

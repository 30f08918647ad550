"""Benchmark of the sparse submanifold convolution path on B200.

Default workload (every N): BASELINE config 5, the largest configuration that
fits one GPU -- a 1024^3 union of 32 ellipsoid shells (7,067,536 voxels,
seed 0) through SubM 64->64, 64->256, 256->256, 256->256 in bf16.  At N > 1 the
same grid is cut into N Morton row ranges, one per GPU, and every layer
exchanges its halo rows over NCCL (strong scaling: total work fixed).
``--workload cfg4|cfg2|cfg3|cfg1|convnext`` runs another configuration
(bevy_synth_b200/workloads.py).

A step is one forward pass of the workload's conv layers.  The neighbor map,
its conv schedule and (N > 1) the halo plan are built once per grid at set-up,
as the reference caches its maps per grid; their device time is reported in
``config.setup_ms``.

metric  = sparse-conv voxel-outputs/s (sum over conv layers of N_out / time),
          with TFLOP/s (algorithmic 2*P*Cin*Cout, P = valid neighbor pairs) and
          the fraction of the measured bf16 peak alongside.
value   = inputs resident in HBM, L2 flushed (256 MiB write) before every
          step, steps timed with CUDA events on the launching stream; max of
          the time over ranks, units summed over ranks.
e2e     = the same through the public API with pinned host buffers: every
          step copies its input features in (H2D) and its output features out
          (D2H), pipelined over H2D / compute / D2H streams with two buffer
          slots, timed from the first H2D to the last D2H.
roofline = the conv kernel (conv_tc_kernel): the step's algorithmic FLOPs over
          the CUDA-event time of its conv launches, against the measured bf16
          peak (MEASURED_PEAKS.json, burst).
cpu_baseline = the reference's CPU path (burn_flex_gmm's flex gather+SGEMM,
          restated in oracle/) on a Morton-contiguous window of the same grid,
          every layer of the workload, on all host cores and on one core.
--impl reference: the same CPU path and sample as cpu_baseline, one sample
          round per step, on all host cores (rank 0 only).
"""
from __future__ import annotations

import argparse
import json
import os
import sys
import threading
import time

import numpy as np

ROOT = os.path.dirname(os.path.abspath(__file__))
sys.path.insert(0, ROOT)

L2_FLUSH_BYTES = 256 << 20
CPU_ROWS_PER_CALL = 8192
CPU_WINDOW_ROWS = 65536


FP32_NOMINAL_TFLOPS = 148 * 128 * 2 * 1.965e9 / 1e12


def load_peaks():
    p = os.path.join(ROOT, "MEASURED_PEAKS.json")
    if os.path.exists(p):
        d = json.load(open(p))
        return (d.get("bf16_tflops", 1590.0), d.get("bf16_tflops_sustained"), d.get("hbm_gbs", 6650.0),
                "measured")
    return 1590.0, 1400.0, 6650.0, "fallback"


def read_traffic(workload: str):
    """DRAM bytes per conv launch (ncu) from the committed profile summary, if any."""
    p = os.path.join(ROOT, "profiles", f"conv_tc_{workload}_traffic.txt")
    if not os.path.exists(p):
        return None
    for line in open(p):
        if line.startswith("bytes_per_launch:"):
            return float(line.split(":")[1])
    return None


class ClockSampler:
    """Samples SM clocks and clock-event reasons through NVML while running."""

    REASONS = {
        "gpu_idle": 0x1, "applications_clocks_setting": 0x2, "sw_power_cap": 0x4, "hw_slowdown": 0x8,
        "sync_boost": 0x10, "sw_thermal_slowdown": 0x20, "hw_thermal_slowdown": 0x40,
        "hw_power_brake_slowdown": 0x80, "display_clock_setting": 0x100,
    }

    def __init__(self, index: int):
        self.samples, self.reasons, self.max_mhz = [], 0, None
        self._stop = threading.Event()
        try:
            import pynvml

            pynvml.nvmlInit()
            self.nv = pynvml
            self.h = pynvml.nvmlDeviceGetHandleByIndex(index)
            self.max_mhz = pynvml.nvmlDeviceGetMaxClockInfo(self.h, pynvml.NVML_CLOCK_SM)
        except Exception:  # noqa: BLE001 -- clocks are reported as unavailable
            self.nv = None

    def _run(self):
        while not self._stop.is_set():
            try:
                self.samples.append(self.nv.nvmlDeviceGetClockInfo(self.h, self.nv.NVML_CLOCK_SM))
                self.reasons |= self.nv.nvmlDeviceGetCurrentClocksEventReasons(self.h)
            except Exception:  # noqa: BLE001
                pass
            time.sleep(0.01)

    def __enter__(self):
        if self.nv:
            self.t = threading.Thread(target=self._run, daemon=True)
            self.t.start()
        return self

    def __exit__(self, *a):
        self._stop.set()
        if self.nv:
            self.t.join()

    def report(self):
        if not self.nv or not self.samples:
            return {"sm_mhz": None, "sm_max_mhz": self.max_mhz, "reasons": ["unavailable"]}
        rs = [k for k, v in self.REASONS.items() if self.reasons & v and k != "gpu_idle"]
        return {"sm_mhz": float(np.median(self.samples)), "sm_max_mhz": self.max_mhz, "reasons": rs,
                "samples": len(self.samples)}


# ------------------------------------------------------------------ CPU sample
class CpuSample:
    """The reference's CPU conv path (burn_flex_gmm flex gather + SGEMM,
    lib.rs:242-375, restated in oracle/) on a Morton-contiguous window of the
    workload's grid: the window's rows, their neighbor map against the grid
    cells around them, and every conv layer of the workload, in slices of
    CPU_ROWS_PER_CALL rows.  Features are seeded N(0, 1) (the CPU's values do
    not change its speed)."""

    def __init__(self, coords: np.ndarray, layers: list, window: int = CPU_WINDOW_ROWS):
        import oracle

        self.oracle = oracle
        n = coords.shape[0]
        w = min(window, n)
        a = max(0, n // 2 - w // 2)
        self.window = coords[a:a + w]
        lo = self.window[:, 1:].min(0) - 1
        hi = self.window[:, 1:].max(0) + 1
        inb = np.all((coords[:, 1:] >= lo) & (coords[:, 1:] <= hi), axis=1) & np.isin(coords[:, 0],
                                                                                   np.unique(self.window[:, 0]))
        cand = np.ascontiguousarray(coords[inb])
        cfg0 = oracle.OracleConfig(1, 1)
        self.nbr = oracle.build_neighbor_rows(cfg0, cand.astype(np.uint32), oracle.DUP_LOWEST,
                                              self.window.astype(np.uint32))
        rng = np.random.default_rng(7)
        self.layers = []
        for cin, cout, wt, b in layers:
            cfg = oracle.OracleConfig(cin, cout)
            x = rng.standard_normal((cand.shape[0], cin)).astype(np.float32)
            self.layers.append((cfg, np.asarray(wt, np.float32), np.asarray(b, np.float32), x,
                                oracle.pack_flex_weight(cfg, wt)))
        self.pos = 0
        self.desc = (f"{w} Morton-contiguous rows of the grid (rows {a}..{a + w}), their neighbor map, "
                     f"{len(layers)} conv layer(s) "
                     f"{[f'{c.in_channels}->{c.out_channels}' for c, *_ in self.layers]} in slices of "
                     f"{CPU_ROWS_PER_CALL} rows")

    def round(self, threads: int) -> tuple[int, float]:
        """One slice through every layer: (voxel outputs, seconds)."""
        w = self.nbr.shape[0]
        s = self.pos
        rows = slice(s, min(s + CPU_ROWS_PER_CALL, w))
        self.pos = rows.stop % w
        t0 = time.perf_counter()
        for cfg, wt, b, x, packed in self.layers:
            self.oracle.subm_conv_flex(cfg, wt, b, x, self.nbr[rows], packed=packed, threads=threads)
        return (rows.stop - rows.start) * len(self.layers), time.perf_counter() - t0

    def rate(self, seconds: float, threads: int) -> tuple[float, float]:
        """Voxel-outputs/s over whole rounds lasting about ``seconds``."""
        units, spent = 0, 0.0
        while spent < seconds:
            u, dt = self.round(threads)
            units += u
            spent += dt
        return units / spent, spent


def run_reference(args, rank: int, world: int):
    """The reference arm: the reference's CPU path on the host cores, same
    workload and sample as cpu_baseline, one sample round per step."""
    if rank != 0:
        return
    from bevy_synth_b200 import synth

    wl_name = args.workload
    if wl_name == "cfg5":
        coords = synth.config5_coords(0)
        p = synth.config5_params(0)
        layers = [(ci, co, w, b) for (ci, co), w, b in zip(p["chans"], p["w"], p["b"])]
        name = "cfg5_sharded_grid_bf16"
    elif wl_name == "cfg4":
        wl = synth.config4(0, feats=False)
        coords, layers, name = wl.coords, [(512, 512, wl.params["w"][0], wl.params["b"][0])], wl.name
    elif wl_name == "cfg2":
        wl = synth.config2(0)
        coords, layers, name = wl.coords, [(256, 256, wl.params[0]["w1"], wl.params[0]["b1"])], wl.name
    elif wl_name == "cfg1":
        wl = synth.config1(0)
        coords, layers, name = wl.coords, [(64, 64, wl.params["w"], wl.params["b"])], wl.name
    else:
        print(json.dumps({"impl": "reference", "unavailable": f"no CPU sample defined for {wl_name}"}))
        return
    threads = os.cpu_count() or 1
    cs = CpuSample(coords, layers)
    times, units = [], 0
    for i in range(args.warmup + args.steps):
        u, dt = cs.round(threads)
        if i >= args.warmup:
            times.append(dt)
            units += u
    total = sum(times)
    v = units / total
    line = {
        "impl": "reference", "metric": "sparse conv voxel-outputs/s", "value": v, "unit": "voxel-outputs/s",
        "n_gpus": world, "steps": args.steps, "warmup": args.warmup, "ms_per_step": 1e3 * total / len(times),
        "higher_is_better": True, "scaling": "strong" if wl_name == "cfg5" else "weak", "vs_baseline": None,
        "dtype": "f32", "data": "synthetic",
        "config": {"workload": name, "voxels": int(coords.shape[0]), "sample": cs.desc},
        "cpu_baseline": {"value": v, "unit": "voxel-outputs/s", "cores": threads, "kind": "port",
                         "sample": cs.desc + "; restatement of burn_flex_gmm flex gather+SGEMM "
                                             "(the reference's Rust is not buildable here)"},
        "e2e": {"value": v, "unit": "voxel-outputs/s", "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0},
    }
    print(json.dumps(line), flush=True)


# ------------------------------------------------------------------ GPU arm
class LaunchTimer:
    """Conv-launch observer (flex_gmm.set_conv_observer): CUDA events around
    every conv launch on the launching stream."""

    def __init__(self):
        import torch

        self.torch = torch
        self.events = []
        self._open = None

    def before(self, config, n_rows):
        e = self.torch.cuda.Event(enable_timing=True)
        e.record()
        self._open = (config, n_rows, e)

    def after(self, config, n_rows):
        e = self.torch.cuda.Event(enable_timing=True)
        e.record()
        cfg, rows, e0 = self._open
        self.events.append((f"{cfg.in_channels}->{cfg.out_channels}", rows, e0, e))

    def times(self):
        return [(lbl, rows, a.elapsed_time(b)) for lbl, rows, a, b in self.events]


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=20)
    ap.add_argument("--warmup", type=int, default=5)
    ap.add_argument("--impl", default="ours", choices=["ours", "reference"])
    ap.add_argument("--workload", default="cfg5", choices=["cfg5", "cfg4", "cfg2", "cfg3", "cfg1", "convnext"])
    ap.add_argument("--cpu-seconds", type=float, default=12.0)
    ap.add_argument("--no-cpu", action="store_true")
    ap.add_argument("--no-e2e", action="store_true")
    ap.add_argument("--cfg5-shells", type=int, default=32,
                    help="shells of the config-5 grid (32 = BASELINE; fewer give a smaller case for ncu captures)")
    args = ap.parse_args()
    args.warmup = max(args.warmup, 3)

    rank = int(os.environ.get("RANK", 0))
    world = int(os.environ.get("WORLD_SIZE", 1))
    local = int(os.environ.get("LOCAL_RANK", 0))

    if args.impl == "reference":
        run_reference(args, rank, world)
        return

    import torch
    import torch.distributed as dist

    from bevy_synth_b200 import _lib
    from bevy_synth_b200 import flex_gmm as F
    from bevy_synth_b200.workloads import WORKLOADS

    torch.cuda.set_device(local)
    dev = torch.device("cuda", local)
    if world > 1:
        import datetime

        dist.init_process_group("nccl", timeout=datetime.timedelta(seconds=300), device_id=dev)
    kw = {"shells": args.cfg5_shells} if args.workload == "cfg5" else {}
    wl = WORKLOADS[args.workload](dev, rank, world, **kw)
    flush = torch.empty(L2_FLUSH_BYTES // 4, dtype=torch.float32, device=dev)
    stream = torch.cuda.current_stream(dev)

    def barrier():
        if world > 1:
            dist.barrier()
        torch.cuda.synchronize()

    # ---- warm-up ---------------------------------------------------------------
    for _ in range(args.warmup):
        y = wl.step(0)
    barrier()
    assert _lib.device_fault() == 0, "device fault during warm-up"
    assert bool(torch.isfinite(y.float()).all()), "non-finite output"

    # ---- device-resident timing ------------------------------------------------
    timer = LaunchTimer()
    sampler = ClockSampler(local)
    steps = []
    barrier()
    F.set_conv_observer(timer)
    with sampler:
        for _ in range(args.steps):
            flush.zero_()
            s0, s1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
            s0.record(stream)
            wl.step(0)
            s1.record(stream)
            steps.append((s0, s1))
        barrier()
    F.set_conv_observer(None)
    t_dev = sum(a.elapsed_time(b) for a, b in steps) / 1e3
    launches = timer.times()
    assert _lib.device_fault() == 0, "device fault during the timed region"

    # ---- end-to-end through the public API with host buffers --------------------
    t_e2e, h2d, d2h = None, 0, 0
    if not args.no_e2e:
        host_in = [t.cpu().pin_memory() for t in wl.inputs(0)]
        out0 = wl.output(0)
        host_out = [torch.empty(out0.shape, dtype=out0.dtype).pin_memory() for _ in range(2)]
        h2d = int(sum(t.numel() * t.element_size() for t in host_in))
        d2h = int(out0.numel() * out0.element_size())
        s_h2d, s_d2h = torch.cuda.Stream(dev), torch.cuda.Stream(dev)
        in_free, out_free = [None, None], [None, None]

        def e2e_step(i, first=None):
            k = i % 2
            with torch.cuda.stream(s_h2d):
                if first is not None:
                    first.record(s_h2d)
                if in_free[k] is not None:
                    s_h2d.wait_event(in_free[k])
                for hsrc, ddst in zip(host_in, wl.inputs(k)):
                    ddst.copy_(hsrc, non_blocking=True)
                h2d_done = torch.cuda.Event()
                h2d_done.record(s_h2d)
            stream.wait_event(h2d_done)
            if out_free[k] is not None:
                stream.wait_event(out_free[k])
            flush.zero_()
            y = wl.step(k)
            done = torch.cuda.Event()
            done.record(stream)
            in_free[k] = done
            with torch.cuda.stream(s_d2h):
                s_d2h.wait_event(done)
                host_out[k].copy_(y, non_blocking=True)
                y.record_stream(s_d2h)
                ev = torch.cuda.Event(enable_timing=True)
                ev.record(s_d2h)
                out_free[k] = ev
            return ev

        for i in range(2):  # untimed: first use of both slots
            e2e_step(i)
        barrier()
        e_first = torch.cuda.Event(enable_timing=True)
        e_last = None
        for i in range(args.steps):
            e_last = e2e_step(i, e_first if i == 0 else None)
        barrier()
        t_e2e = e_first.elapsed_time(e_last) / 1e3
        assert _lib.device_fault() == 0, "device fault during the end-to-end leg"

    # ---- max over ranks ---------------------------------------------------------
    units = float(wl.units * args.steps)
    flops = float(wl.flops * args.steps)
    vec = torch.tensor([t_dev, t_e2e or 0.0, units, flops], dtype=torch.float64, device=dev)
    if world > 1:
        tmax = vec[:2].clone()
        dist.all_reduce(tmax, op=dist.ReduceOp.MAX)
        tot = vec[2:].clone()
        dist.all_reduce(tot, op=dist.ReduceOp.SUM)
        t_dev, t_e2e = float(tmax[0]), (float(tmax[1]) if t_e2e is not None else None)
        units, flops = float(tot[0]), float(tot[1])

    if rank == 0:
        peak_tf, peak_sus, hbm, peak_kind = load_peaks()
        conv_ms_step = sum(t for _, _, t in launches) / args.steps
        achieved = wl.flops / (conv_ms_step / 1e3) / 1e12
        n_launch_step = len(launches) // args.steps
        per_layer = []
        lpl = getattr(wl, "launches_per_layer", 1)
        flops_l = getattr(wl, "layer_flops", None)
        for j in range(0, n_launch_step, lpl):
            ms = sum(launches[s * n_launch_step + j + q][2] for s in range(args.steps)
                     for q in range(lpl)) / args.steps
            d = {"layer": launches[j][0], "ms": round(ms, 4)}
            if flops_l is not None and j // lpl < len(flops_l):
                tf = flops_l[j // lpl] / (ms / 1e3) / 1e12
                d.update({"tflops": round(tf, 1), "frac_bf16_peak": round(tf / peak_tf, 4)})
            per_layer.append(d)
        cpu = None
        if world == 1 and not args.no_cpu and wl.cpu_layers() is not None:
            threads = os.cpu_count() or 1
            cs = CpuSample(wl.coords_np, wl.cpu_layers())
            v_all, spent = cs.rate(args.cpu_seconds, threads)
            v_one, spent1 = cs.rate(args.cpu_seconds / 3, 1)
            cpu = {"value": v_all, "unit": "voxel-outputs/s", "cores": threads, "kind": "port",
                   "sample": f"{cs.desc}; {spent:.1f} s on {threads} threads; oracle restatement of "
                             "burn_flex_gmm flex gather+SGEMM (the reference's CPU path)",
                   "single_thread": {"value": v_one, "cores": 1, "seconds": round(spent1, 1),
                                     "note": "the reference's own configuration (matrixmultiply without "
                                             "threading)"}}
        cfgd = wl.describe()
        cfgd.update({"l2": "flushed before every step (256 MiB write); inputs also larger than L2"
                     if args.workload == "cfg5" else "flushed before every step (256 MiB write)",
                     "conv_launches_per_step": n_launch_step, "per_layer": per_layer})
        line = {
            "metric": "sparse conv voxel-outputs/s", "value": units / t_dev, "unit": "voxel-outputs/s",
            "n_gpus": world, "steps": args.steps, "warmup": args.warmup,
            "ms_per_step": 1e3 * t_dev / args.steps, "higher_is_better": True,
            "scaling": "strong" if args.workload == "cfg5" else "weak",
            "vs_baseline": None, "dtype": wl.dtype, "data": "synthetic (seeded; BASELINE shapes and distributions)",
            "tflops": flops / t_dev / 1e12, "pct_bf16_peak": flops / t_dev / 1e12 / (peak_tf * world),
            "config": cfgd,
            "roofline": ({"bound": "tensor", "kernel": "conv_tc_kernel", "achieved": achieved,
                          "peak": peak_tf, "unit": "TFLOP/s", "frac": achieved / peak_tf,
                          "frac_of_sustained": (achieved / peak_sus) if peak_sus else None,
                          "peak_source": f"{peak_kind} bf16 (burst); frac_of_sustained against the sustained figure",
                          "traffic": read_traffic(args.workload),
                          "flops_per_step_rank0": wl.flops, "conv_ms_per_step_rank0": conv_ms_step}
                         if wl.dtype != "f32" else
                         # fp32 runs on the CUDA cores: no measured FP32 peak exists, so the nominal FFMA
                         # peak at the maximum SM clock (148 SMs x 128 FMA/clock x 2 x 1.965 GHz)
                         {"bound": "fp32", "kernel": "conv_f32_tiled_kernel", "achieved": achieved,
                          "peak": FP32_NOMINAL_TFLOPS, "unit": "TFLOP/s", "frac": achieved / FP32_NOMINAL_TFLOPS,
                          "frac_of_sustained": None, "peak_source": "nominal FP32 FFMA peak (no measured figure)",
                          "traffic": None, "flops_per_step_rank0": wl.flops, "conv_ms_per_step_rank0": conv_ms_step}),
            "cpu_baseline": cpu,
            "e2e": ({"value": units / t_e2e, "unit": "voxel-outputs/s", "h2d_bytes_per_step": h2d * world,
                     "d2h_bytes_per_step": d2h * world} if t_e2e else None),
            "gpu_launches": int(args.steps * wl.kernels_per_step),
            "clocks": sampler.report(),
        }
        print(json.dumps(line), flush=True)
    if world > 1:
        dist.barrier()
        dist.destroy_process_group()


if __name__ == "__main__":
    main()

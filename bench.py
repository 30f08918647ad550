"""Benchmark of the sparse submanifold convolution path on B200.

Workload (N=1): BASELINE config 2 -- a stack of 4 SparseResBlock3d at C=256,
bf16, on a 128^3 union of 4 ellipsoid shells (seed = rank, one independent
asset per GPU).  One step = neighbor map build from the coordinates + the
first LN1/SiLU + 8 fused tcgen05 convs (conv1: +bias, LN2, SiLU; conv2:
+bias, +residual, next block's LN1/SiLU as a second output).

metric  = sparse-conv voxel-outputs/s (sum over conv layers of N_out / time),
          with TFLOP/s (algorithmic 2*P*Cin*Cout, P = valid neighbor pairs) and
          the fraction of the measured bf16 peak alongside.
value   = inputs resident in HBM, L2 flushed (256 MiB write) before every
          step, each step timed with CUDA events on the launching stream.
e2e     = the same through the public API with pinned host buffers: every
          step copies its coordinates and features in (H2D) and its output
          features out (D2H); steps are pipelined over H2D / compute / D2H
          streams with two buffer slots, timed from the first H2D to the
          last D2H.
--impl reference: the reference's CPU path (burn_flex_gmm's flex
          gather+SGEMM, restated in oracle/) on the host cores.
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


def load_peaks():
    p = os.path.join(ROOT, "MEASURED_PEAKS.json")
    if os.path.exists(p):
        d = json.load(open(p))
        return d.get("bf16_tflops", 1590.0), d.get("hbm_gbs", 6650.0), "measured"
    return 1590.0, 6650.0, "fallback"


def read_traffic():
    """DRAM bytes per conv launch from the committed ncu summary, if any."""
    p = os.path.join(ROOT, "profiles", "conv_tc_cfg2_traffic.txt")
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


def cpu_sample(wl, seconds: float, threads: int, rows_per_step: int = 8192):
    """Times the oracle's flex conv (the reference's CPU path) on Morton-
    contiguous row slices of the workload's first C=256 layer."""
    import oracle

    c = wl.feats.shape[1]
    cfg = oracle.OracleConfig(c, c)
    nbr = oracle.build_neighbor_rows(cfg, wl.coords.astype(np.uint32), oracle.DUP_LOWEST)
    packed = oracle.pack_flex_weight(cfg, wl.params[0]["w1"])
    n = nbr.shape[0]
    done, pairs, t0 = 0, 0, time.perf_counter()
    start = 0
    while True:
        rows = slice(start, min(start + rows_per_step, n))
        oracle.subm_conv_flex(cfg, wl.params[0]["w1"], wl.params[0]["b1"], wl.feats, nbr[rows], packed=packed,
                              threads=threads)
        done += rows.stop - rows.start
        pairs += int((nbr[rows] >= 0).sum())
        start = rows.stop % n
        if time.perf_counter() - t0 >= seconds:
            break
    dt = time.perf_counter() - t0
    return done / dt, 2.0 * pairs * c * c / dt / 1e12, done


def run_reference(args, rank: int, world: int):
    if rank != 0:
        return
    from bevy_synth_b200 import synth

    wl = synth.config2(0)
    threads = os.cpu_count() or 1
    # each step: one bounded slice of the config-2 C=256 layer
    import oracle

    c = wl.feats.shape[1]
    cfg = oracle.OracleConfig(c, c)
    nbr = oracle.build_neighbor_rows(cfg, wl.coords.astype(np.uint32), oracle.DUP_LOWEST)
    packed = oracle.pack_flex_weight(cfg, wl.params[0]["w1"])
    rows_per_step = 4096
    times, rows_done = [], 0
    for i in range(args.warmup + args.steps):
        s = (i * rows_per_step) % nbr.shape[0]
        sl = slice(s, min(s + rows_per_step, nbr.shape[0]))
        t0 = time.perf_counter()
        oracle.subm_conv_flex(cfg, wl.params[0]["w1"], wl.params[0]["b1"], wl.feats, nbr[sl], packed=packed,
                              threads=threads)
        dt = time.perf_counter() - t0
        if i >= args.warmup:
            times.append(dt)
            rows_done += sl.stop - sl.start
    total = sum(times)
    v = rows_done / total
    line = {
        "impl": "reference", "metric": "sparse conv voxel-outputs/s", "value": v, "unit": "voxel-outputs/s",
        "n_gpus": world, "steps": args.steps, "warmup": args.warmup, "ms_per_step": 1e3 * total / len(times),
        "higher_is_better": True, "scaling": "weak", "vs_baseline": None, "dtype": "f32", "data": "synthetic",
        "config": {"workload": wl.name, "voxels": int(nbr.shape[0]), "channels": c,
                   "sample": f"{rows_per_step} Morton-contiguous rows of one C=256 SubM layer per step"},
        "cpu_baseline": {"value": v, "unit": "voxel-outputs/s", "cores": threads, "kind": "port",
                         "sample": f"{rows_per_step}-row slices of the config-2 C=256 layer; restatement of "
                                   "burn_flex_gmm flex gather+SGEMM (reference Rust not buildable here)"},
        "e2e": {"value": v, "unit": "voxel-outputs/s", "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0},
    }
    print(json.dumps(line), flush=True)


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=30)
    ap.add_argument("--warmup", type=int, default=5)
    ap.add_argument("--impl", default="ours", choices=["ours", "reference"])
    ap.add_argument("--cpu-seconds", type=float, default=12.0)
    ap.add_argument("--no-cpu", action="store_true")
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

    from bevy_synth_b200 import _lib, blocks, synth
    from bevy_synth_b200 import flex_gmm as F

    torch.cuda.set_device(local)
    dev = torch.device("cuda", local)
    if world > 1:
        import datetime

        dist.init_process_group("nccl", timeout=datetime.timedelta(seconds=120), device_id=dev)

    wl = synth.config2(seed=rank)
    c = 256
    cfg = F.SparseSubmConvConfig.subm3(c, c)
    stack = blocks.ResBlockStack([blocks.ResBlockParams.from_numpy(p, dev) for p in wl.params])
    n = wl.coords.shape[0]
    coords_d = torch.as_tensor(wl.coords, device=dev)
    feats_d = torch.as_tensor(wl.feats, device=dev).to(torch.bfloat16)
    ws = F.NeighborWorkspace(dev, n)
    bufs: dict = {}
    flush = torch.empty(L2_FLUSH_BYTES // 4, dtype=torch.float32, device=dev)
    stream = torch.cuda.current_stream(dev)
    conv_events: list = []

    use_order = os.environ.get("SC_ROW_ORDER", "1") == "1"

    def step(coords_t, feats_t, record=False):
        nbr = F.neighbor_rows_tensor_from_coords_tensor(cfg, coords_t, check_status=False, workspace=ws)
        order = F.neighbor_schedule(cfg, nbr) if use_order else None
        if record:
            return stack_forward_timed(feats_t, nbr, order)
        return stack.forward(feats_t, nbr, bufs, order), nbr

    def stack_forward_timed(x, nbr, order):
        # identical to ResBlockStack.forward, with events around each conv launch
        b0 = stack.blocks[0]
        h = F.layer_norm_affine_silu_forward(x, b0.ln1_g, b0.ln1_b, b0.eps, out=bufs["h"])
        h1 = bufs["h1"]
        ping = [bufs["x0"], bufs["x1"]]
        cur = x
        for i, p in enumerate(stack.blocks):
            e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
            e0.record(stream)
            F.sparse_subm_conv_forward(cfg, h, nbr, p.w1, p.b1, F.Epilogue(layer_norm=True, ln_eps=p.eps,
                                       ln_gamma=p.ln2_g, ln_beta=p.ln2_b, silu=True, schedule=order), out=h1)
            e1.record(stream)
            conv_events.append((e0, e1))
            nxt = ping[i % 2]
            if i + 1 < len(stack.blocks):
                q = stack.blocks[i + 1]
                e = F.Epilogue(residual=cur, layer_norm=True, ln_eps=q.eps, ln_gamma=q.ln1_g, ln_beta=q.ln1_b,
                               silu=True, out2=h, schedule=order)
            else:
                e = F.Epilogue(residual=cur, schedule=order)
            e2, e3 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
            e2.record(stream)
            F.sparse_subm_conv_forward(cfg, h1, nbr, p.w2, p.b2, e, out=nxt)
            e3.record(stream)
            conv_events.append((e2, e3))
            cur = nxt
        return cur, nbr

    # warm-up (also checks the map's status once)
    for _ in range(args.warmup):
        y, nbr = step(coords_d, feats_d)
    ws.status(dev)
    torch.cuda.synchronize()
    P = int((nbr >= 0).sum().item())
    convs = stack.conv_count()
    flops_per_conv = 2.0 * P * c * c
    assert torch.isfinite(y.float()).all().item(), "non-finite output"

    # ---- device-resident timing ---------------------------------------------
    def barrier():
        if world > 1:
            dist.barrier()
        torch.cuda.synchronize()

    sampler = ClockSampler(local)
    step_ms = []
    barrier()
    with sampler:
        for _ in range(args.steps):
            flush.zero_()
            s0, s1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
            s0.record(stream)
            step(coords_d, feats_d, record=True)
            s1.record(stream)
            step_ms.append((s0, s1))
        barrier()
    t_dev = sum(a.elapsed_time(b) for a, b in step_ms) / 1e3
    conv_ms = [a.elapsed_time(b) for a, b in conv_events]
    assert _lib.device_fault() == 0, "device fault during the timed region"

    # ---- end-to-end through the public API with host buffers -----------------
    # Steps are pipelined over three streams (H2D, compute, D2H) and two slots
    # of device inputs / outputs, so the copies of one step overlap the convs of
    # its neighbours; every step still copies its inputs in and its result out.
    # The time is the span from the first H2D to the last D2H.
    coords_h = torch.as_tensor(wl.coords).pin_memory()
    feats_h = torch.as_tensor(wl.feats).to(torch.bfloat16).pin_memory()
    out_h = [torch.empty((n, c), dtype=torch.bfloat16).pin_memory() for _ in range(2)]
    cd = [torch.empty_like(coords_d) for _ in range(2)]
    fd = [torch.empty((n, c), dtype=torch.bfloat16, device=dev) for _ in range(2)]
    slot_bufs = [dict(bufs), {}]
    s_h2d, s_d2h = torch.cuda.Stream(dev), torch.cuda.Stream(dev)
    in_free = [None, None]
    out_free = [None, None]

    def e2e_step(i, first=None):
        k = i % 2
        with torch.cuda.stream(s_h2d):
            if first is not None:
                first.record(s_h2d)
            if in_free[k] is not None:
                s_h2d.wait_event(in_free[k])
            cd[k].copy_(coords_h, non_blocking=True)
            fd[k].copy_(feats_h, non_blocking=True)
            h2d_done = torch.cuda.Event()
            h2d_done.record(s_h2d)
        stream.wait_event(h2d_done)
        if out_free[k] is not None:
            stream.wait_event(out_free[k])
        flush.zero_()
        nbr_k = F.neighbor_rows_tensor_from_coords_tensor(cfg, cd[k], check_status=False, workspace=ws)
        order_k = F.neighbor_schedule(cfg, nbr_k) if use_order else None
        y = stack.forward(fd[k], nbr_k, slot_bufs[k], order_k)
        done = torch.cuda.Event()
        done.record(stream)
        in_free[k] = done
        with torch.cuda.stream(s_d2h):
            s_d2h.wait_event(done)
            out_h[k].copy_(y, non_blocking=True)
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

    # ---- max over ranks -------------------------------------------------------
    units = float(n * convs * args.steps)
    flops = flops_per_conv * convs * args.steps
    vec = torch.tensor([t_dev, t_e2e, units, flops, n], dtype=torch.float64, device=dev)
    if world > 1:
        tmax = vec[:2].clone()
        dist.all_reduce(tmax, op=dist.ReduceOp.MAX)
        tot = vec[2:].clone()
        dist.all_reduce(tot, op=dist.ReduceOp.SUM)
        t_dev, t_e2e = float(tmax[0]), float(tmax[1])
        units, flops, n_all = float(tot[0]), float(tot[1]), int(tot[2])
    else:
        n_all = n

    if rank == 0:
        peak_tf, hbm, peak_kind = load_peaks()
        avg_conv_s = float(np.mean(conv_ms)) / 1e3
        achieved = flops_per_conv / avg_conv_s / 1e12
        tflops = flops / t_dev / 1e12
        cpu = None
        if world == 1 and not args.no_cpu:
            threads = os.cpu_count() or 1
            v, tf, rows = cpu_sample(wl, args.cpu_seconds, threads)
            cpu = {"value": v, "unit": "voxel-outputs/s", "cores": threads, "kind": "port",
                   "tflops": tf,
                   "sample": f"{rows} rows of one C=256 SubM layer of this workload (Morton-contiguous slices, "
                             f"~{args.cpu_seconds:.0f} s); oracle restatement of burn_flex_gmm flex gather+SGEMM"}
        line = {
            "metric": "sparse conv voxel-outputs/s", "value": units / t_dev, "unit": "voxel-outputs/s",
            "n_gpus": world, "steps": args.steps, "warmup": args.warmup,
            "ms_per_step": 1e3 * t_dev / args.steps, "higher_is_better": True, "scaling": "weak",
            "vs_baseline": None, "dtype": "bf16", "data": "synthetic",
            "tflops": tflops, "pct_bf16_peak": tflops / (peak_tf * world),
            "config": {"workload": wl.name, "voxels_per_gpu": n, "voxels_total": n_all, "blocks": len(wl.params),
                       "channels": c, "convs_per_step": convs, "valid_pairs_P": P,
                       "step": "neighbor map + row order + LN1/SiLU + 8 fused SubM convs",
                       "row_order": "mask-sorted" if use_order else "morton",
                       "l2": "flushed before every step (256 MiB write); per-step CUDA events",
                       "parallelism": f"asset-sharded x{world} (one independent asset per GPU, no collective)"},
            "roofline": {"bound": "tensor", "kernel": "conv_tc_kernel", "achieved": achieved,
                         "peak": peak_tf, "unit": "TFLOP/s", "frac": achieved / peak_tf,
                         "peak_source": f"{peak_kind} bf16 (burst)", "traffic": read_traffic(),
                         "flops_per_launch": flops_per_conv, "avg_launch_ms": avg_conv_s * 1e3},
            "cpu_baseline": cpu,
            "e2e": {"value": units / t_e2e, "unit": "voxel-outputs/s",
                    "h2d_bytes_per_step": int(coords_h.numel() * 4 + feats_h.numel() * 2),
                    "d2h_bytes_per_step": int(out_h[0].numel() * 2)},
            "gpu_launches": int(args.steps * (2 + (2 if use_order else 0) + 1 + convs)),
            "clocks": sampler.report(),
        }
        print(json.dumps(line), flush=True)
    if world > 1:
        dist.barrier()
        dist.destroy_process_group()


if __name__ == "__main__":
    main()

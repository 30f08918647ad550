"""Per-workload device timing of the sparse-conv path (one GPU).

``python -m bevy_synth_b200.perf [names...]`` prints one JSON line per
workload: BASELINE configs 1, 3, 4, 5 (config 2 is ``bench.py``'s headline)
and the ConvNeXt decoder stage.  Inputs are resident in HBM; L2 is flushed
(256 MiB write) before every timed repetition; each repetition is bracketed
by CUDA events on the launching stream; the median of the repetitions is
reported.  FLOPs are algorithmic (2*P*Cin*Cout per SubM layer with P the
valid (row, tap) pairs; 2*N*Cin*Cout per linear layer), and the fraction is
of the measured dense bf16 peak (MEASURED_PEAKS.json, burst) -- or of the
measured HBM copy bandwidth for the fp32 CUDA-core layer, which is HBM- or
FP32-bound rather than tensor-bound.
"""
from __future__ import annotations

import json
import os
import sys
import time

import numpy as np
import torch

from . import blocks, synth
from . import flex_gmm as F

_ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))


def _peaks():
    try:
        with open(os.path.join(_ROOT, "MEASURED_PEAKS.json")) as f:
            d = json.load(f)
        return float(d["bf16_tflops"]), float(d["hbm_gbs"]), "measured"
    except (OSError, KeyError, ValueError):
        return 1590.0, 6650.0, "fallback"


class _Timer:
    def __init__(self, dev, reps=5, warmup=3):
        self.dev, self.reps, self.warmup = dev, reps, warmup
        self.flush = torch.empty(256 * 2 ** 20 // 4, dtype=torch.float32, device=dev)

    def __call__(self, fn) -> float:
        """Median milliseconds of fn() over the repetitions."""
        for _ in range(self.warmup):
            fn()
        torch.cuda.synchronize(self.dev)
        ts = []
        for _ in range(self.reps):
            self.flush.zero_()
            a = torch.cuda.Event(enable_timing=True)
            b = torch.cuda.Event(enable_timing=True)
            a.record()
            fn()
            b.record()
            torch.cuda.synchronize(self.dev)
            ts.append(a.elapsed_time(b))
        return float(np.median(ts))


def _line(name, ms, flops, voxel_outputs, layers, extra=None):
    peak, _, kind = _peaks()
    tf = flops / ms / 1e9
    d = {"workload": name, "ms": round(ms, 4), "tflops": round(tf, 1),
         "frac_bf16_peak": round(tf / peak, 4), "peak_source": f"{kind} bf16 (burst)",
         "voxel_outputs_per_s": voxel_outputs / ms * 1e3, "layers": layers}
    if extra:
        d.update(extra)
    return d


def run_cfg1(dev, t):
    wl = synth.config1(0)
    cfg = F.SparseSubmConvConfig.subm3(64, 64)
    ct = torch.as_tensor(wl.coords, device=dev)
    nbr = F.neighbor_rows_tensor_from_coords_tensor(cfg, ct)
    P = float((nbr >= 0).sum())
    n = ct.shape[0]
    w = torch.as_tensor(np.asarray(wl.params["w"]), device=dev)
    b = torch.as_tensor(np.asarray(wl.params["b"]), device=dev)
    x = torch.as_tensor(wl.feats, device=dev)
    out = []
    ms = t(lambda: F.sparse_subm_conv_forward(cfg, x, nbr, w, b))
    _, hbm, kind = _peaks()
    byts = 4.0 * (n * 64 * 2) + 4 * 27 * 64 * 64 + 4 * 27 * n
    sms = torch.cuda.get_device_properties(dev).multi_processor_count
    fp32_peak = sms * 128 * 2 * 1.965e9 / 1e12  # nominal FFMA TFLOP/s at the maximum SM clock
    out.append(_line("cfg1_fp32_cuda_core", ms, 2 * P * 64 * 64, n, 1,
                     {"dtype": "f32", "frac_hbm": round(byts / ms / 1e6 / hbm, 4), "hbm_source": kind,
                      "frac_fp32_nominal": round(2 * P * 64 * 64 / ms / 1e9 / fp32_peak, 4)}))
    xb, wb = x.to(torch.bfloat16), w.to(torch.bfloat16)
    sched = F.neighbor_schedule(cfg, nbr)
    ms = t(lambda: F.sparse_subm_conv_forward(cfg, xb, nbr, wb, b, F.Epilogue(schedule=sched)))
    out.append(_line("cfg1_bf16_tensor", ms, 2 * P * 64 * 64, n, 1, {"dtype": "bf16"}))
    return out


def run_cfg3(dev, t):
    wl = synth.config3(0)
    pyr = blocks.UpsamplePyramid(wl.params, dev)
    coords = torch.as_tensor(wl.coords, device=dev)
    x = torch.as_tensor(wl.feats, device=dev).to(torch.bfloat16)
    out = []
    for li, (c2s, res, mseed) in enumerate(pyr.levels):
        m = torch.as_tensor(synth.child_mask(mseed, coords.shape[0]), device=dev)
        keep = {}

        def level():
            cc, y, nb = c2s.forward(coords, x, m)
            keep["r"] = (cc, res.forward(y, nb), nb)

        ms = t(level)
        cc, y, nb = keep["r"]
        nbp = F.neighbor_rows_tensor_from_coords_tensor(c2s.cfg1, coords)
        fl = c2s.flops(nbp, nb, m) + res.conv_count() * 2.0 * float((nb >= 0).sum()) * res.channels ** 2
        out.append(_line(f"cfg3_level{li}", ms, fl, 2 * cc.shape[0] + res.conv_count() * cc.shape[0],
                         2 + res.conv_count(),
                         {"parents": int(coords.shape[0]), "children": int(cc.shape[0]),
                          "channels": [c2s.cin, c2s.cout], "note": "includes subdivision and both neighbor maps"}))
        coords, x = cc, y
    return out


def run_cfg4(dev, t):
    wl = synth.config4(0)
    st = blocks.SubmStack(wl.params["w"], wl.params["b"], True, dev)
    ct = torch.as_tensor(wl.coords, device=dev)
    nbr = F.neighbor_rows_tensor_from_coords_tensor(st.cfgs[0], ct)
    x = torch.as_tensor(wl.feats, device=dev).to(torch.bfloat16)
    sched = F.neighbor_schedule(st.cfgs[0], nbr)
    n = ct.shape[0]
    ms = t(lambda: st.forward(x, nbr, sched))
    return [_line("cfg4_64_assets_8x512", ms, st.flops(nbr), 8 * n, 8, {"voxels": int(n)})]


def run_cfg5(dev, t):
    wl = synth.config5(0)
    st = blocks.SubmStack(wl.params["w"], wl.params["b"], False, dev)
    ct = torch.as_tensor(wl.coords, device=dev)
    nbr = F.neighbor_rows_tensor_from_coords_tensor(st.cfgs[0], ct)
    x = torch.as_tensor(wl.feats, device=dev).to(torch.bfloat16)
    sched = F.neighbor_schedule(st.cfgs[0], nbr)
    n = ct.shape[0]
    P = float((nbr >= 0).sum())
    out = []
    total_ms, total_fl = 0.0, 0.0
    for i, (cfg, w, b) in enumerate(zip(st.cfgs, st.w, st.b)):
        xi = torch.randn(n, cfg.in_channels, device=dev).to(torch.bfloat16)
        ms = t(lambda: F.sparse_subm_conv_forward(cfg, xi, nbr, w, b, F.Epilogue(schedule=sched)))
        fl = 2 * P * cfg.in_channels * cfg.out_channels
        total_ms += ms
        total_fl += fl
        out.append(_line(f"cfg5_layer{i}_{cfg.in_channels}to{cfg.out_channels}", ms, fl, n, 1,
                         {"voxels": int(n)}))
    out.append(_line("cfg5_all_layers_1gpu", total_ms, total_fl, 4 * n, 4, {"voxels": int(n)}))
    return out


def run_convnext(dev, t):
    wl = synth.convnext_stage(0)
    stack = blocks.ConvNeXtStack([blocks.ConvNeXtParams.from_numpy(p, dev) for p in wl.params])
    ct = torch.as_tensor(wl.coords, device=dev)
    nbr = F.neighbor_rows_tensor_from_coords_tensor(stack.cfg, ct)
    sched = F.neighbor_schedule(stack.cfg, nbr)
    x = torch.as_tensor(wl.feats, device=dev).to(torch.bfloat16)
    bufs: dict = {}
    n = ct.shape[0]
    ms = t(lambda: stack.forward(x, nbr, sched, bufs))
    return [_line("convnext_stage_2x_c256_h1024", ms, stack.flops(nbr), n * len(stack.blocks),
                  stack.launches(), {"voxels": int(n)})]


def run_gather(dev, t):
    """Random 128-byte row gather bandwidth by copy method (micro/gather_bw.cu), the
    bound of the gather-limited small-channel layers."""
    import re
    import subprocess

    from .build import nvcc
    here = os.path.dirname(os.path.abspath(__file__))
    src = os.path.join(here, "micro", "gather_bw.cu")
    exe = os.path.join(here, "micro", "gather_bw")
    if not os.path.exists(exe) or os.path.getmtime(exe) < os.path.getmtime(src):
        subprocess.run([nvcc(), "-gencode", "arch=compute_100a,code=sm_100a", "-O3", "-std=c++17",
                        "-I" + os.path.join(_ROOT, "include"), "-o", exe, src, "-lcuda"], check=True)
    txt = subprocess.run([exe], check=True, capture_output=True, text=True).stdout
    out = []
    for line in txt.splitlines():
        m = re.match(r"(.+?)\s+([\d.]+) TB/s\s+([\d.]+) B/clk", line)
        if m:
            out.append({"workload": "gather_bw", "method": m.group(1).strip(), "tb_per_s": float(m.group(2)),
                        "bytes_per_clk_per_sm_at_1.9ghz": float(m.group(3))})
    return out


WORKLOADS = {"cfg1": run_cfg1, "cfg3": run_cfg3, "cfg4": run_cfg4, "cfg5": run_cfg5, "convnext": run_convnext,
             "gather": run_gather}


def main(argv=None):
    names = (argv if argv is not None else sys.argv[1:]) or list(WORKLOADS)
    dev = torch.device("cuda", 0)
    torch.cuda.set_device(dev)
    t = _Timer(dev)
    for name in names:
        t0 = time.time()
        for d in WORKLOADS[name](dev, t):
            d["wall_s"] = round(time.time() - t0, 1)
            print(json.dumps(d), flush=True)


if __name__ == "__main__":
    main()

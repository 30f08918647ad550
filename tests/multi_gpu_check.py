"""Run under torchrun (one process per GPU): checks the multi-GPU paths
against the same computation on the whole input on one GPU.

* Morton-range sharding with halo exchange (config-5 structure, reduced size):
  each rank's rows of the sharded 3-layer stack vs the whole-grid stack.
* Asset sharding (config-4 structure, reduced size): each rank's assets alone
  vs all assets together.
Prints one JSON line per rank; exit code 0 when every check passes."""
import datetime
import json
import os
import sys

import numpy as np
import torch
import torch.distributed as dist

sys.path.insert(0, os.path.dirname(os.path.dirname(os.path.abspath(__file__))))
from bevy_synth_b200 import _lib, blocks, sharding, synth  # noqa: E402
from bevy_synth_b200 import flex_gmm as F  # noqa: E402


def rel(a, b):
    return float(torch.linalg.norm((a - b).float()) / max(float(torch.linalg.norm(b.float())), 1e-30))


def main():
    rank, world = int(os.environ["RANK"]), int(os.environ["WORLD_SIZE"])
    local = int(os.environ.get("LOCAL_RANK", rank))
    torch.cuda.set_device(local)
    dev = torch.device("cuda", local)
    dist.init_process_group("nccl", timeout=datetime.timedelta(seconds=60), device_id=dev)
    out = {"rank": rank}
    try:
        # --- Morton-range sharding + halo -----------------------------------
        coords = synth.config5_coords(seed=3, shells=6, grid=256, axes_range=(20.0, 50.0))
        n = coords.shape[0]
        rng = np.random.default_rng(5)
        chans = [(64, 64), (64, 256), (256, 256)]
        ws = [synth.normal_weight(rng, co, ci) for ci, co in chans]
        bs = [(0.1 * rng.standard_normal(co)).astype(np.float32) for _, co in chans]
        x = torch.as_tensor(rng.standard_normal((n, 64)).astype(np.float32), device=dev).to(torch.bfloat16)
        stack = blocks.SubmStack(ws, bs, silu=False, device=dev)
        ct = torch.as_tensor(coords, device=dev)
        cfg = F.SparseSubmConvConfig.subm3(64, 64)
        full_nbr = F.neighbor_rows_tensor_from_coords_tensor(cfg, ct)
        full = stack.forward(x, full_nbr)
        ranges = sharding.morton_ranges(n, world)
        lo, hi = ranges[rank]
        plan = sharding.HaloPlan.build_local(ct[lo:hi].contiguous(), cfg)
        # the local map, with plan rows and halo rows put back to global ids, is the global map's rows
        glob_of = torch.cat([lo + plan.order.to(torch.int64), plan.halo_global])
        nl = plan.nbr_local.to(torch.int64)
        remapped = torch.where(nl >= 0, glob_of[nl.clamp(min=0)], torch.full_like(nl, -1))
        maps_equal = bool(torch.equal(remapped.to(torch.int32), full_nbr[lo + plan.order.to(torch.int64)]))
        sharded = sharding.ShardedSubmStack(stack, plan)
        y = sharded.forward(x[lo:hi].contiguous()).clone()
        y2 = sharded.forward(x[lo:hi].contiguous())   # second pass reuses the buffers
        torch.cuda.synchronize()
        out["morton"] = {"rows": hi - lo, "halo": plan.n_halo, "interior": plan.n_interior,
                         "rel": rel(y, full[lo:hi]), "repeat_equal": bool(torch.equal(y, y2)),
                         "maps_equal": maps_equal}
        # --- asset sharding ---------------------------------------------------
        n_assets = 4 * world
        wl_all = synth.config4(seed=2, assets=n_assets, layers=2, channels=128)
        mine = sharding.asset_shard(n_assets, rank, world)
        wl = synth.config4(seed=2, assets=n_assets, layers=2, channels=128, asset_ids=mine)
        st4 = blocks.SubmStack(wl.params["w"], wl.params["b"], silu=True, device=dev)
        c4 = F.SparseSubmConvConfig.subm3(128, 128)
        ca = torch.as_tensor(wl_all.coords, device=dev)
        ya = st4.forward(torch.as_tensor(wl_all.feats, device=dev).to(torch.bfloat16),
                         F.neighbor_rows_tensor_from_coords_tensor(c4, ca))
        cm = torch.as_tensor(wl.coords, device=dev)
        ym = st4.forward(torch.as_tensor(wl.feats, device=dev).to(torch.bfloat16),
                         F.neighbor_rows_tensor_from_coords_tensor(c4, cm))
        sel = torch.as_tensor(np.isin(wl_all.coords[:, 0], mine), device=dev)
        out["assets"] = {"assets": mine, "rows": int(cm.shape[0]), "rel": rel(ym, ya[sel])}
        out["fault"] = _lib.device_fault()
        ok = (out["morton"]["rel"] <= 1e-6 and out["morton"]["repeat_equal"] and out["morton"]["maps_equal"]
              and out["assets"]["rel"] <= 1e-6
              and out["fault"] == 0)
        out["ok"] = ok
    finally:
        dist.barrier()
        dist.destroy_process_group()
    # one write of the whole line (<= PIPE_BUF bytes: atomic), so the ranks' lines do not interleave
    sys.stdout.write(json.dumps(out) + "\n")
    sys.stdout.flush()
    sys.exit(0 if out.get("ok") else 1)


if __name__ == "__main__":
    main()

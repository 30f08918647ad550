"""The BASELINE configurations as runnable workloads on the sparse-conv path.

A workload is set up once per grid -- coordinates, weights, the neighbor map,
its conv schedule and, on several GPUs, the shard's halo plan -- and then runs
steps: one forward pass of the configuration's conv layers over inputs that
are already on the device.  Keeping the map per grid is what the reference
does too (its thread-local neighbor-map cache, burn_flex_gmm src/wgpu.rs:128,
379-382); the set-up time is measured and reported beside the steps.

==========  ===============================================  ===============================
name        BASELINE configuration                           on N > 1 GPUs
==========  ===============================================  ===============================
cfg5        1024^3 union of 32 shells, SubM 64->64, 64->256,   Morton row ranges + halo
            256->256, 256->256 (bf16)                          exchange (strong scaling)
cfg4        64 assets, 8 x (SubM 512->512 + SiLU) (bf16)       64/N assets per rank (weak)
cfg2        4 SparseResBlock3d, C=256 (bf16)                   one grid per GPU (replicas)
cfg3        3-level C2S upsample pyramid 768->384->192->96     replicas
cfg1        one SubM 64->64, fp32, 64^3 sphere shell           replicas
convnext    2 ConvNeXt blocks C=256 / hidden 1024 (bf16)       replicas
==========  ===============================================  ===============================

``bench.py`` times the steps.  Every workload exposes:

* ``units`` -- conv voxel outputs of one step on this rank (the metric's unit);
* ``flops`` -- algorithmic FLOPs of one step on this rank (2*P*Cin*Cout per SubM
  layer, P = valid neighbor pairs; 2*N*Cin*Cout per linear layer);
* ``step(slot)`` -- one forward pass on the resident inputs of ``slot``;
* ``inputs(slot)`` / ``output(slot)`` -- the tensors an end-to-end step copies in
  from and out to host memory;
* ``kernels_per_step`` -- launches of this library's kernels in one step.
"""
from __future__ import annotations

import numpy as np
import torch

from . import blocks, sharding, synth
from . import flex_gmm as F
from .sparse_tensor import SparseTensor

BF16 = torch.bfloat16


def _events_ms(fn, dev) -> float:
    """Device time of fn() in ms (CUDA events on the current stream)."""
    s = torch.cuda.current_stream(dev)
    a, b = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    a.record(s)
    fn()
    b.record(s)
    b.synchronize()
    return a.elapsed_time(b)


def _broadcast(tensors, world: int, group=None):
    """Rank 0's parameter tensors to every rank (one NCCL broadcast each, at set-up)."""
    if world > 1:
        import torch.distributed as dist

        for t in tensors:
            dist.broadcast(t, src=0, group=group)


def _pairs(nbr: torch.Tensor) -> int:
    return int((nbr >= 0).sum().item())


class _Slots:
    """Per-slot objects (slot 0 built at set-up, slot 1 on first use)."""

    def __init__(self, make):
        self._make = make
        self._slots: dict = {}

    def __getitem__(self, k):
        if k not in self._slots:
            self._slots[k] = self._make(k)
        return self._slots[k]


class _Base:
    launches_per_layer = 1
    setup_ms = 0.0

    def inputs(self, slot: int = 0) -> list:
        return [self._x[slot]]

    def output(self, slot: int = 0) -> torch.Tensor:
        return self._out[slot]


# ---------------------------------------------------------------------------- cfg5
class Cfg5(_Base):
    """1024^3 union of 32 ellipsoid shells (~7.07M voxels),
    SubM 64->64, 64->256, 256->256, 256->256, bf16, no activation.  On N GPUs
    the Morton-sorted rows are cut into N equal ranges; each layer exchanges
    the boundary rows another rank reads (sharding.HaloPlan)."""

    name = "cfg5_sharded_grid_bf16"
    dtype = "bf16"

    def __init__(self, dev, rank: int = 0, world: int = 1, group=None, seed: int = 0, coords=None, shells: int = 32,
                 tile_sources: bool = True):
        self.dev, self.rank, self.world = dev, rank, world
        self.shells = shells
        coords_np = synth.config5_coords(seed, shells=shells) if coords is None else coords
        self.coords_np = coords_np
        self.params = synth.config5_params(seed)
        self.stack = blocks.SubmStack(self.params["w"], self.params["b"], False, dev)
        _broadcast(self.stack.w + self.stack.b, world, group)
        n = coords_np.shape[0]
        self.n_total = n
        ct = torch.as_tensor(coords_np, device=dev)
        cfg = self.stack.cfgs[0]
        x_all = synth.device_normal(seed + 1, n, 64, dev, BF16)
        holder = {}
        if world == 1:
            self.lo, self.hi = 0, n

            def setup():
                holder["nbr"] = F.neighbor_rows_tensor_from_coords_tensor(cfg, ct)
                holder["sched"] = F.neighbor_schedule(cfg, holder["nbr"])
                holder["ts"] = F.neighbor_tile_sources(cfg, holder["nbr"]) if tile_sources else None

            self.setup_ms = _events_ms(setup, dev)
            self.nbr, self.sched, self.tile_sources = holder["nbr"], holder["sched"], holder["ts"]
            self._x = _Slots(lambda k: x_all if k == 0 else x_all.clone())
            self.plan = None
        else:
            self.lo, self.hi = sharding.morton_ranges(n, world)[rank]

            def setup():
                holder["plan"] = sharding.HaloPlan.build_local(ct[self.lo:self.hi].contiguous(), cfg, group)
                holder["stack"] = sharding.ShardedSubmStack(self.stack, holder["plan"], tile_sources=tile_sources)

            self.setup_ms = _events_ms(setup, dev)
            self.plan = holder["plan"]
            self.nbr = self.plan.nbr_local
            self.tile_sources = None
            x_mine = x_all[self.lo:self.hi].contiguous()
            del x_all
            self._x = _Slots(lambda k: x_mine if k == 0 else x_mine.clone())
            first = holder["stack"]
            self._sharded = _Slots(lambda k: first if k == 0 else first.twin())
        P = _pairs(self.nbr)
        self.n_local = self.hi - self.lo
        self.valid_pairs = P
        self.layer_flops = [2.0 * P * c.in_channels * c.out_channels for c in self.stack.cfgs]
        self.flops = float(sum(self.layer_flops))
        self.units = 4 * self.n_local
        self.launch_labels = [f"{c.in_channels}->{c.out_channels}" for c in self.stack.cfgs]
        # sharded: two conv launches a layer (interior, boundary rows); per layer also the halo pack
        # gather, plus the gathers into and out of plan order
        self.launches_per_layer = 1 if world == 1 else 2
        self.kernels_per_step = 4 if world == 1 else 4 * 3 + 2
        self._out: dict = {}

    def step(self, slot: int = 0) -> torch.Tensor:
        x = self._x[slot]
        if self.world == 1:
            y = self.stack.forward(x, self.nbr, self.sched, self.tile_sources)
        else:
            y = self._sharded[slot].forward(x)
        self._out[slot] = y
        return y

    def describe(self) -> dict:
        d = {"workload": self.name, "voxels_total": int(self.n_total), "voxels_this_rank": int(self.n_local),
             "layers": self.launch_labels, "valid_pairs_P_this_rank": int(self.valid_pairs),
             "grid": f"1024^3, union of {self.shells} ellipsoid shells (seed 0)",
             "step": "4 SubM conv layers (tcgen05, bf16); neighbor map, conv schedule and tile-source plan "
                     "built once per grid",
             "tile_sources": "64-channel layers stage each tile's distinct source rows once, A built in TMEM"
             if (self.tile_sources is not None or (self.plan is not None and self._sharded[0].ts_int is not None))
             else "off",
             "setup_ms": round(self.setup_ms, 3)}
        if self.plan is not None:
            d["halo_rows_this_rank"] = int(self.plan.n_halo)
            d["interior_rows_this_rank"] = int(self.plan.n_interior)
            d["parallelism"] = (f"Morton-range sharded x{self.world}; per layer NCCL all-to-all halo exchange "
                                "on a second stream, overlapped with the interior rows' conv")
        else:
            d["parallelism"] = "one GPU"
        return d

    def cpu_layers(self):
        return [(c.in_channels, c.out_channels, w, b) for c, w, b in
                zip(self.stack.cfgs, self.params["w"], self.params["b"])]


# ---------------------------------------------------------------------------- cfg4
class Cfg4(_Base):
    """64 assets (64^3 sphere shells, batch index in
    coord[0]), 8 x (SubM 512->512 + SiLU), bf16.  On N GPUs each rank takes a
    contiguous block of 64/N assets (no neighbor crosses an asset)."""

    name = "cfg4_batched_assets_bf16_512"
    dtype = "bf16"

    def __init__(self, dev, rank: int = 0, world: int = 1, group=None, seed: int = 0, assets: int = 64,
                 layers: int = 8, channels: int = 512):
        self.dev, self.rank, self.world = dev, rank, world
        self.assets = sharding.asset_shard(assets, rank, world)
        wl = synth.config4(seed, assets=assets, layers=layers, channels=channels, asset_ids=self.assets,
                           feats=False)
        self.coords_np = wl.coords
        self.params = wl.params
        self.stack = blocks.SubmStack(wl.params["w"], wl.params["b"], True, dev)
        _broadcast(self.stack.w + self.stack.b, world, group)
        ct = torch.as_tensor(wl.coords, device=dev)
        cfg = self.stack.cfgs[0]
        parts = [synth.device_normal(s, r, channels, dev, BF16) for s, r in
                 zip(wl.extra["feat_seeds"], wl.extra["rows"])]
        x = torch.cat(parts) if parts else torch.empty((0, channels), dtype=BF16, device=dev)
        # the rank's assets as one batch-grouped sparse tensor (batch index = asset id)
        self.sparse = SparseTensor.new(ct, x, 64)
        assert self.sparse.layout.batch_size() == len(self.assets)
        self.setup_ms = _events_ms(lambda: self.sparse.neighbor_rows(cfg), dev)
        self.nbr, self.sched = self.sparse.neighbor_rows(cfg)
        self._x = _Slots(lambda k: x if k == 0 else x.clone())
        self.n_local = int(ct.shape[0])
        self.valid_pairs = _pairs(self.nbr)
        self.flops = self.stack.flops(self.nbr)
        self.units = layers * self.n_local
        self.kernels_per_step = layers
        self._out: dict = {}

    def step(self, slot: int = 0) -> torch.Tensor:
        y = self.stack.forward(self._x[slot], self.nbr, self.sched)
        self._out[slot] = y
        return y

    def describe(self) -> dict:
        return {"workload": self.name, "assets_this_rank": len(self.assets), "voxels_this_rank": self.n_local,
                "valid_pairs_P_this_rank": self.valid_pairs, "layers": "8 x SubM 512->512 + SiLU",
                "step": "8 fused SubM conv launches; neighbor map + schedule built once per grid",
                "setup_ms": round(self.setup_ms, 3),
                "parallelism": f"asset-sharded x{self.world} ({len(self.assets)} assets per rank, no collective)"}

    def cpu_layers(self):
        return [(512, 512, self.params["w"][0], self.params["b"][0])]


# ---------------------------------------------------------------------------- cfg2
class Cfg2(_Base):
    """4 SparseResBlock3d at C=256, bf16, on a 128^3 union of
    4 ellipsoid shells.  One independent grid per GPU (seed = rank)."""

    name = "cfg2_resblock_stack_bf16_256"
    dtype = "bf16"

    def __init__(self, dev, rank: int = 0, world: int = 1, group=None, seed: int | None = None):
        self.dev, self.rank, self.world = dev, rank, world
        seed = rank if seed is None else seed
        wl = synth.config2(seed)
        self.coords_np, self.params = wl.coords, wl.params
        self.stack = blocks.ResBlockStack([blocks.ResBlockParams.from_numpy(p, dev) for p in wl.params])
        ct = torch.as_tensor(wl.coords, device=dev)
        holder = {}

        def setup():
            holder["nbr"] = F.neighbor_rows_tensor_from_coords_tensor(self.stack.cfg, ct)
            holder["sched"] = F.neighbor_schedule(self.stack.cfg, holder["nbr"])

        self.setup_ms = _events_ms(setup, dev)
        self.nbr, self.sched = holder["nbr"], holder["sched"]
        x = torch.as_tensor(wl.feats, device=dev).to(BF16)
        self._x = _Slots(lambda k: x if k == 0 else x.clone())
        self._bufs = _Slots(lambda k: {})
        self.n_local = int(ct.shape[0])
        self.valid_pairs = _pairs(self.nbr)
        self.flops = 2.0 * self.valid_pairs * 256 * 256 * self.stack.conv_count()
        self.units = self.stack.conv_count() * self.n_local
        self.kernels_per_step = 1 + self.stack.conv_count()
        self._out: dict = {}

    def step(self, slot: int = 0) -> torch.Tensor:
        y = self.stack.forward(self._x[slot], self.nbr, self._bufs[slot], self.sched)
        self._out[slot] = y
        return y

    def describe(self) -> dict:
        return {"workload": self.name, "voxels_this_rank": self.n_local, "blocks": len(self.params),
                "channels": 256, "valid_pairs_P_this_rank": self.valid_pairs,
                "step": "LN1/SiLU + 8 fused SubM conv launches; neighbor map + schedule built once per grid",
                "setup_ms": round(self.setup_ms, 3),
                "parallelism": f"replicas x{self.world} (one independent grid per GPU, no collective)"}

    def cpu_layers(self):
        return [(256, 256, self.params[0]["w1"], self.params[0]["b1"])]


# ---------------------------------------------------------------------------- cfg3
class Cfg3(_Base):
    """32^3 grid at 20% occupancy, C=768, three levels of
    [C2S upsample (seeded Bernoulli(0.5) child mask) + 2 SparseResBlock3d],
    768->384->192->96, bf16.  Replicas on N GPUs."""

    name = "cfg3_upsample_pyramid_bf16"
    dtype = "bf16"

    def __init__(self, dev, rank: int = 0, world: int = 1, group=None, seed: int = 0):
        self.dev, self.rank, self.world = dev, rank, world
        wl = synth.config3(seed)
        self.pyr = blocks.UpsamplePyramid(wl.params, dev)
        self.coords = torch.as_tensor(wl.coords, device=dev)
        x = torch.as_tensor(wl.feats, device=dev).to(BF16)
        # the child masks, and the per-level counts, from one untimed pass
        self.masks, units, flops = [], 0, 0.0
        coords, h = self.coords, x
        self.level_rows = []
        for c2s, res, mseed in self.pyr.levels:
            m = torch.as_tensor(synth.child_mask(mseed, coords.shape[0]), device=dev)
            self.masks.append(m)
            nbp = F.neighbor_rows_tensor_from_coords_tensor(c2s.cfg1, coords)
            cc, h, nb = c2s.forward(coords, h, m, nbr_parent=nbp)
            h = res.forward(h, nb)
            n_child = int(cc.shape[0])
            self.level_rows.append((int(coords.shape[0]), n_child))
            units += (2 + res.conv_count()) * n_child
            flops += c2s.flops(nbp, nb, m) + res.conv_count() * 2.0 * _pairs(nb) * res.channels ** 2
            coords = cc
        self._x = _Slots(lambda k: x if k == 0 else x.clone())
        self.units, self.flops = units, flops
        # per level: LN, subdivision count + write, 2 maps (build + query each), grouped schedule (key +
        # permute), C2S conv1 + conv2, and the ResBlock stack (LN + 2 convs a block)
        self.kernels_per_step = sum(1 + 2 + 4 + 2 + 2 + 1 + 2 * len(res.blocks) for _, res, _ in self.pyr.levels)
        self.n_local = int(self.coords.shape[0])
        self._out: dict = {}

    def step(self, slot: int = 0) -> torch.Tensor:
        _, y, _ = self.pyr.forward(self.coords, self._x[slot], self.masks)
        self._out[slot] = y
        return y

    def describe(self) -> dict:
        return {"workload": self.name, "levels": [{"parents": p, "children": c} for p, c in self.level_rows],
                "channels": [768, 384, 192, 96],
                "step": "per level: subdivision (child count read back), 2 neighbor maps, C2S conv1 + conv2, "
                        "2 SparseResBlock3d",
                "parallelism": f"replicas x{self.world}"}

    def cpu_layers(self):
        return None


# ---------------------------------------------------------------------------- cfg1
class Cfg1(_Base):
    """one SubM 64->64, fp32, on the 64^3 sphere shell
    (~21.7k voxels), on the fp32 CUDA-core kernel."""

    name = "cfg1_subm_fp32_64"
    dtype = "f32"

    def __init__(self, dev, rank: int = 0, world: int = 1, group=None, seed: int = 0):
        self.dev, self.rank, self.world = dev, rank, world
        wl = synth.config1(seed)
        self.coords_np, self.params = wl.coords, wl.params
        self.cfg = F.SparseSubmConvConfig.subm3(64, 64)
        ct = torch.as_tensor(wl.coords, device=dev)
        self.nbr = F.neighbor_rows_tensor_from_coords_tensor(self.cfg, ct)
        self.w = torch.as_tensor(np.asarray(wl.params["w"]), device=dev)
        self.b = torch.as_tensor(np.asarray(wl.params["b"]), device=dev)
        x = torch.as_tensor(wl.feats, device=dev)
        self._x = _Slots(lambda k: x if k == 0 else x.clone())
        self.n_local = int(ct.shape[0])
        self.valid_pairs = _pairs(self.nbr)
        self.flops = 2.0 * self.valid_pairs * 64 * 64
        self.units = self.n_local
        self.kernels_per_step = 1
        self._out: dict = {}

    def step(self, slot: int = 0) -> torch.Tensor:
        y = F.sparse_subm_conv_forward(self.cfg, self._x[slot], self.nbr, self.w, self.b)
        self._out[slot] = y
        return y

    def describe(self) -> dict:
        return {"workload": self.name, "voxels_this_rank": self.n_local, "valid_pairs_P_this_rank": self.valid_pairs,
                "step": "1 SubM conv launch (fp32, CUDA cores)", "parallelism": f"replicas x{self.world}"}

    def cpu_layers(self):
        return [(64, 64, self.params["w"], self.params["b"])]


# ---------------------------------------------------------------------------- ConvNeXt
class ConvNeXt(_Base):
    """Two ConvNeXt decoder blocks (C=256, hidden 1024) on config 2's grid: the
    production TRELLIS.2 decoder block (not a BASELINE configuration)."""

    name = "convnext_stage_bf16_256"
    dtype = "bf16"

    def __init__(self, dev, rank: int = 0, world: int = 1, group=None, seed: int = 0):
        self.dev, self.rank, self.world = dev, rank, world
        wl = synth.convnext_stage(seed)
        self.stack = blocks.ConvNeXtStack([blocks.ConvNeXtParams.from_numpy(p, dev) for p in wl.params])
        ct = torch.as_tensor(wl.coords, device=dev)
        self.nbr = F.neighbor_rows_tensor_from_coords_tensor(self.stack.cfg, ct)
        self.sched = F.neighbor_schedule(self.stack.cfg, self.nbr)
        x = torch.as_tensor(wl.feats, device=dev).to(BF16)
        self._x = _Slots(lambda k: x if k == 0 else x.clone())
        self._bufs = _Slots(lambda k: {})
        self.n_local = int(ct.shape[0])
        self.flops = self.stack.flops(self.nbr)
        self.units = self.n_local * len(self.stack.blocks) * 3
        self.kernels_per_step = 3 * len(self.stack.blocks)
        self._out: dict = {}

    def step(self, slot: int = 0) -> torch.Tensor:
        y = self.stack.forward(self._x[slot], self.nbr, self.sched, self._bufs[slot])
        self._out[slot] = y
        return y

    def describe(self) -> dict:
        return {"workload": self.name, "voxels_this_rank": self.n_local,
                "step": "2 x (SubM + LN, linear 256->1024 + SiLU, linear 1024->256 + residual)",
                "parallelism": f"replicas x{self.world}"}

    def cpu_layers(self):
        return None


WORKLOADS = {"cfg5": Cfg5, "cfg4": Cfg4, "cfg2": Cfg2, "cfg3": Cfg3, "cfg1": Cfg1, "convnext": ConvNeXt}

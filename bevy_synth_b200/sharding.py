"""Multi-GPU partitioning of the sparse-conv path (one process per GPU).

The reference has no multi-GPU support; its own test shows why a single grid
cannot simply be cut into row chunks -- a chunk rebuilt on its own loses the
neighbors across the cut (burn_trellis/src/runtime_model/
sparse_decoder_tests.rs:238-292), which is why its decoder disables
coordinate-chunked streaming (sparse_decoder_runtime_impl.rs:2135-2177).
Two partitions are built here:

* Assets: independent grids, batch index in coord[0].
  Each rank takes a contiguous block of assets; no neighbor crosses a batch,
  so there is no data-path collective.
* Morton ranges (config 5): one large grid, rows Morton-sorted, rank r owns
  rows [lo_r, hi_r).  Every rank holds the (small) coordinate list, queries
  its own rows against the whole grid, and a one-time plan exchanges the
  requested boundary rows' ids.  Per layer each rank packs the rows others
  need (sc_gather_rows) and one all_to_all delivers the halo rows into its
  own [n_local + n_halo, C] buffer; the local neighbor map addresses halo rows
  as ids >= n_local, which the conv accepts because query rows <= input rows.
"""
from __future__ import annotations

from dataclasses import dataclass
from typing import Callable

import torch
import torch.distributed as dist


def asset_shard(n_assets: int, rank: int, world: int) -> list[int]:
    """Contiguous block of assets for `rank` (sizes differ by at most one)."""
    base, extra = divmod(n_assets, world)
    lo = rank * base + min(rank, extra)
    return list(range(lo, lo + base + (1 if rank < extra else 0)))


def morton_ranges(n_rows: int, world: int) -> list[tuple[int, int]]:
    """Equal contiguous row ranges of a Morton-sorted grid."""
    base, extra = divmod(n_rows, world)
    out, lo = [], 0
    for r in range(world):
        hi = lo + base + (1 if r < extra else 0)
        out.append((lo, hi))
        lo = hi
    return out


MapFn = Callable[[torch.Tensor, torch.Tensor], torch.Tensor]  # (all coords, query coords) -> [n_q, K] global ids
GatherFn = Callable[[torch.Tensor, torch.Tensor], torch.Tensor]


def _default_gather(src: torch.Tensor, idx: torch.Tensor) -> torch.Tensor:
    if src.is_cuda:
        from . import flex_gmm as F

        return F.gather_rows(src, idx)
    return src.index_select(0, idx.to(torch.int64))


@dataclass
class HaloPlan:
    """Exchange plan of one rank for a Morton-range-sharded grid."""

    rank: int
    world: int
    lo: int
    hi: int
    n_halo: int
    nbr_local: torch.Tensor      # [n_local, K] int32: own rows [0, n_local), halo rows [n_local, n_local + n_halo)
    halo_global: torch.Tensor    # [n_halo] int64 global ids, in receive order
    send_idx: torch.Tensor       # [n_send] int32 local ids to pack, grouped by destination rank
    send_counts: list
    recv_counts: list
    group: object = None

    @property
    def n_local(self) -> int:
        return self.hi - self.lo

    @staticmethod
    def build(coords_all: torch.Tensor, ranges: list, rank: int, map_fn: MapFn, group=None) -> "HaloPlan":
        world = len(ranges)
        lo, hi = ranges[rank]
        dev = coords_all.device
        g = map_fn(coords_all, coords_all[lo:hi].contiguous()).to(torch.int64)
        valid = g >= 0
        own = valid & (g >= lo) & (g < hi)
        halo_mask = valid & ~own
        halo_ids = torch.unique(g[halo_mask])                       # sorted == receive order
        n_halo = int(halo_ids.numel())
        local = torch.full_like(g, -1)
        local[own] = g[own] - lo
        local[halo_mask] = (hi - lo) + torch.searchsorted(halo_ids, g[halo_mask])
        # requests per owner (contiguous ranges -> the sorted ids split by owner)
        bounds = torch.tensor([r[1] for r in ranges], dtype=torch.int64, device=dev)
        owner = torch.searchsorted(bounds, halo_ids, right=True)
        req_counts = torch.bincount(owner, minlength=world).to(torch.int64)
        cnt_in = torch.zeros(world, dtype=torch.int64, device=dev)
        dist.all_to_all_single(cnt_in, req_counts, group=group)
        recv_counts = req_counts.tolist()             # rows each owner will send me
        send_counts = cnt_in.tolist()                 # rows I must send to each rank
        req_in = torch.empty(int(sum(send_counts)), dtype=torch.int64, device=dev)
        dist.all_to_all_single(req_in, halo_ids.contiguous(), output_split_sizes=send_counts,
                               input_split_sizes=recv_counts, group=group)
        if req_in.numel() and (int(req_in.min()) < lo or int(req_in.max()) >= hi):
            raise RuntimeError("halo plan: a peer requested rows this rank does not own")
        return HaloPlan(rank, world, lo, hi, n_halo, local.to(torch.int32).contiguous(), halo_ids,
                        (req_in - lo).to(torch.int32).contiguous(), send_counts, recv_counts, group)

    def buffer(self, channels: int, dtype, device) -> torch.Tensor:
        """A [n_local + n_halo, C] layer buffer: the conv writes rows [0, n_local)."""
        return torch.empty((self.n_local + self.n_halo, channels), dtype=dtype, device=device)

    def exchange(self, buf: torch.Tensor, gather_fn: GatherFn = _default_gather) -> torch.Tensor:
        """Fills buf[n_local:] with the halo rows, packing buf[:n_local] rows for the peers."""
        n = self.n_local
        send = gather_fn(buf[:n], self.send_idx) if self.send_idx.numel() else buf.new_empty((0,) + buf.shape[1:])
        recv = buf[n:]
        dist.all_to_all_single(recv, send.contiguous(), output_split_sizes=self.recv_counts,
                               input_split_sizes=self.send_counts, group=self.group)
        return buf


class ShardedSubmStack:
    """SubM layer stack on a Morton-range-sharded grid: per layer one halo
    exchange (pack + all_to_all into the layer buffer), then the local conv
    over [n_local + n_halo] input rows writing the next buffer's own rows."""

    def __init__(self, stack, plan: HaloPlan, schedule=None):
        self.stack = stack      # blocks.SubmStack
        self.plan = plan
        self.schedule = schedule
        self.bufs = None

    def forward(self, x_local: torch.Tensor) -> torch.Tensor:
        from . import flex_gmm as F

        plan, n = self.plan, self.plan.n_local
        if self.bufs is None:
            self.bufs = [plan.buffer(c.in_channels, x_local.dtype, x_local.device) for c in self.stack.cfgs]
        self.bufs[0][:n].copy_(x_local)
        out = None
        for i, (cfg, w, b) in enumerate(zip(self.stack.cfgs, self.stack.w, self.stack.b)):
            buf = self.bufs[i]
            plan.exchange(buf)
            dst = self.bufs[i + 1][:n] if i + 1 < len(self.bufs) else None
            out = F.sparse_subm_conv_forward(cfg, buf, plan.nbr_local, w, b,
                                             F.Epilogue(silu=self.stack.silu, schedule=self.schedule), out=dst)
        return out

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
* Morton ranges (config 5): one large grid, rows sorted by (batch, Morton
  code), rank r owns the r-th contiguous range.  A rank holds only its own
  coordinates.  ``HaloPlan.build_local`` finds, from the rank's own rows, the
  neighbor coordinates that fall in another rank's key range, asks their
  owners (one all-to-all of coordinates, one of answers) and numbers the rows
  that exist as halo rows n_local, n_local + 1, ...  Per layer each owner
  packs the rows others read (sc_gather_rows) and one all-to-all delivers
  them into the receiver's [n_local + n_halo, C] layer buffer; the local map
  addresses halo rows as ids >= n_local, which the conv accepts because query
  rows <= input rows.  Local rows are kept in plan order [interior | boundary]
  (boundary = reads a halo row or is sent to a peer), so each layer runs the
  interior rows while the exchange is in flight on a second stream and the
  boundary rows after it.
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


# ------------------------------------------------------------------ Morton keys
_SPREAD = ((32, 0x1F00000000FFFF), (16, 0x1F0000FF0000FF), (8, 0x100F00F00F00F00F),
           (4, 0x10C30C30C30C30C3), (2, 0x1249249249249249))


def _spread3(v: torch.Tensor) -> torch.Tensor:
    """Bit i of v (< 2^21) moved to bit 3i, int64."""
    v = v.to(torch.int64) & 0x1FFFFF
    for sh, mask in _SPREAD:
        v = (v | (v << sh)) & mask
    return v


def morton_key(batch: torch.Tensor, xyz: torch.Tensor) -> torch.Tensor:
    """Sort key of a coordinate: (batch << 48) | interleave(x, y, z), x in bit 0.
    Components lie in [0, 65534], so the interleave fits 48 bits and the key
    orders rows exactly as a (batch, Morton code) sort does."""
    code = _spread3(xyz[:, 0]) | (_spread3(xyz[:, 1]) << 1) | (_spread3(xyz[:, 2]) << 2)
    return (batch.to(torch.int64) << 48) | code


QueryFn = Callable[[torch.Tensor, torch.Tensor, object], torch.Tensor]
GatherFn = Callable[[torch.Tensor, torch.Tensor], torch.Tensor]


def _device_query(table: torch.Tensor, query: torch.Tensor, cfg) -> torch.Tensor:
    """[n_query, K] rows of ``table`` at query + offset (the library's map)."""
    from . import flex_gmm as F

    return F.neighbor_rows_query_tensor(cfg, table, query)


def _default_gather(src: torch.Tensor, idx: torch.Tensor) -> torch.Tensor:
    if src.is_cuda:
        from . import flex_gmm as F

        return F.gather_rows(src, idx)
    return src.index_select(0, idx.to(torch.int64))


def _kernel_offsets(cfg) -> torch.Tensor:
    from . import flex_gmm as F

    return F.kernel_offsets(cfg)


def _point_config():
    """The 1x1x1 config of a point lookup (offset 0)."""
    from . import flex_gmm as F

    return F.SparseSubmConvConfig(1, 1, 1, 1, 1)


@dataclass
class HaloPlan:
    """Exchange plan of one rank for a Morton-range-sharded grid.

    Local rows are numbered in plan order: ``order[p]`` is the rank's own
    (Morton-local) row at plan row p; rows [0, n_interior) read no halo row
    and are sent to no peer, rows [n_interior, n_local) are the boundary."""

    rank: int
    world: int
    lo: int                      # first global row of this rank
    n_local: int
    n_halo: int
    n_interior: int
    order: torch.Tensor          # [n_local] int32: plan row -> Morton-local row
    nbr_local: torch.Tensor      # [n_local, K] int32 in plan numbering; halo rows n_local + h
    halo_global: torch.Tensor    # [n_halo] int64 global ids, in receive order
    send_idx: torch.Tensor       # [n_send] int32 plan rows to pack, grouped by destination rank
    send_counts: list
    recv_counts: list
    group: object = None

    @property
    def hi(self) -> int:
        return self.lo + self.n_local

    @staticmethod
    def build_local(coords_local: torch.Tensor, cfg, group=None, query_fn: QueryFn = _device_query) -> "HaloPlan":
        """The plan from this rank's own [n_local, 4] coordinates (the rank's
        contiguous range of the grid's (batch, Morton)-sorted rows; every rank
        holds at least one row).  Collective: every rank of ``group`` calls it."""
        rank, world = dist.get_rank(group), dist.get_world_size(group)
        dev = coords_local.device
        n = int(coords_local.shape[0])
        if n == 0:
            raise ValueError("halo plan: every rank needs at least one row")
        keys = morton_key(coords_local[:, 0], coords_local[:, 1:])
        if n > 1 and bool((keys[1:] <= keys[:-1]).any()):
            raise ValueError("halo plan: rows must be unique and sorted by (batch, Morton code)")
        meta = torch.tensor([n, int(keys[0]), int(keys[-1])], dtype=torch.int64, device=dev)
        metas = [torch.empty_like(meta) for _ in range(world)]
        dist.all_gather(metas, meta, group=group)
        metas = torch.stack(metas).cpu()
        counts, firsts, lasts = metas[:, 0], metas[:, 1], metas[:, 2]
        if world > 1 and bool((firsts[1:] <= lasts[:-1]).any()):
            raise ValueError("halo plan: ranks' row ranges overlap or are out of order")
        starts = torch.cumsum(counts, 0) - counts
        lo = int(starts[rank])
        splitters = firsts.to(dev)

        # own rows first: a tap that finds no local row may lie in another rank's key range
        nbr = query_fn(coords_local, coords_local, cfg).to(torch.int32).clone()
        offs = _kernel_offsets(cfg).to(dev).to(torch.int64)
        rows, taps = (nbr < 0).nonzero(as_tuple=True)
        nc = coords_local[rows, 1:].to(torch.int64) + offs[taps]
        ok = ((nc >= 0) & (nc <= 65534)).all(1)
        rows, taps, nc = rows[ok], taps[ok], nc[ok]
        b = coords_local[rows, 0].to(torch.int64)
        key = morton_key(b, nc)
        owner = torch.searchsorted(splitters, key, right=True) - 1
        remote = (owner >= 0) & (owner != rank)
        rows, taps, nc, b, key = rows[remote], taps[remote], nc[remote], b[remote], key[remote]
        ukey, inv = torch.unique(key, sorted=True, return_inverse=True)
        ucoord = torch.empty((ukey.numel(), 4), dtype=torch.int32, device=dev)
        ucoord[inv] = torch.cat([b[:, None], nc], 1).to(torch.int32)
        uowner = torch.searchsorted(splitters, ukey, right=True) - 1
        req_counts = torch.bincount(uowner, minlength=world).to(torch.int64)
        cnt_in = torch.empty_like(req_counts)
        dist.all_to_all_single(cnt_in, req_counts, group=group)
        req_l, in_l = req_counts.tolist(), cnt_in.tolist()
        req_in = torch.empty((int(sum(in_l)), 4), dtype=torch.int32, device=dev)
        dist.all_to_all_single(req_in, ucoord, output_split_sizes=in_l, input_split_sizes=req_l, group=group)
        # the owner's answers: its local row of each requested coordinate, or -1
        if req_in.shape[0]:
            ans = query_fn(coords_local, req_in, _point_config())[:, 0].to(torch.int64).contiguous()
        else:
            ans = torch.empty(0, dtype=torch.int64, device=dev)
        back = torch.empty(int(sum(req_l)), dtype=torch.int64, device=dev)
        dist.all_to_all_single(back, ans, output_split_sizes=req_l, input_split_sizes=in_l, group=group)
        exists = back >= 0
        n_halo = int(exists.sum())
        hid = torch.where(exists, n + torch.cumsum(exists.to(torch.int64), 0) - 1, torch.full_like(back, -1))
        nbr[rows, taps] = hid[inv].to(torch.int32)
        recv_counts = torch.bincount(uowner[exists], minlength=world).tolist()
        halo_global = (starts.to(dev)[uowner] + back)[exists]
        sent = ans >= 0
        send_local = ans[sent]
        src_rank = torch.repeat_interleave(torch.arange(world, device=dev), cnt_in)
        send_counts = torch.bincount(src_rank[sent], minlength=world).tolist()

        # plan order: interior rows first, then the boundary (reads a halo row, or is sent)
        bnd = (nbr >= n).any(1)
        if send_local.numel():
            bnd[send_local] = True
        order = torch.cat([(~bnd).nonzero()[:, 0], bnd.nonzero()[:, 0]])
        rank_of = torch.empty(n, dtype=torch.int64, device=dev)
        rank_of[order] = torch.arange(n, device=dev)
        nb = nbr[order].to(torch.int64)
        own = (nb >= 0) & (nb < n)
        nb = torch.where(own, rank_of[nb.clamp(0, n - 1)], nb)
        return HaloPlan(rank, world, lo, n, n_halo, int((~bnd).sum()), order.to(torch.int32).contiguous(),
                        nb.to(torch.int32).contiguous(), halo_global.contiguous(),
                        rank_of[send_local].to(torch.int32).contiguous(), send_counts, recv_counts, group)

    def buffer(self, channels: int, dtype, device) -> torch.Tensor:
        """A [n_local + n_halo, C] layer buffer in plan order: the convs write rows [0, n_local)."""
        return torch.empty((self.n_local + self.n_halo, channels), dtype=dtype, device=device)

    def pack(self, buf: torch.Tensor, gather_fn: GatherFn = _default_gather) -> torch.Tensor:
        """The rows of buf[:n_local] the peers read, grouped by destination rank.  They are
        all boundary rows (plan rows >= n_interior)."""
        n = self.n_local
        if not self.send_idx.numel():
            return buf.new_empty((0,) + buf.shape[1:])
        return gather_fn(buf[:n], self.send_idx).contiguous()

    def exchange(self, buf: torch.Tensor, gather_fn: GatherFn = _default_gather, send=None) -> torch.Tensor:
        """Fills buf[n_local:] with the halo rows, packing buf[:n_local] rows for the peers
        (or sending ``send``, an earlier ``pack`` of buf)."""
        if send is None:
            send = self.pack(buf, gather_fn)
        dist.all_to_all_single(buf[self.n_local:], send, output_split_sizes=self.recv_counts,
                               input_split_sizes=self.send_counts, group=self.group)
        return buf

    def inverse_order(self) -> torch.Tensor:
        """[n_local] int32: Morton-local row -> plan row."""
        inv = torch.empty_like(self.order)
        inv[self.order.to(torch.int64)] = torch.arange(self.n_local, dtype=torch.int32, device=self.order.device)
        return inv


class ShardedSubmStack:
    """SubM layer stack on a Morton-range-sharded grid.  Per layer: the halo
    exchange (pack + all-to-all) on a second stream while the interior rows'
    conv runs on the compute stream, then the boundary rows' conv once the halo
    has arrived.  Input and output rows are in Morton-local order.

    Measured on two B200s (config 5, 20 steps, one job, max over ranks): this
    order 22.71 / 22.88 ms a step; boundary rows first with the next layer's
    exchange beside the interior conv, 23.01 / 23.21 (all-to-all enqueued before
    the interior conv) and 22.78 / 23.08 (after it).  NCCL's kernel gets SMs only
    when a conv leaves them, so the exchange lands after the interior conv in
    every order, and boundary-first adds a dependency step per layer."""

    def __init__(self, stack, plan: HaloPlan, schedule: bool = True, _scheds=None, tile_sources: bool = True):
        from . import flex_gmm as F

        self.stack = stack      # blocks.SubmStack
        self.plan = plan
        cfg = stack.cfgs[0]
        ni = plan.n_interior
        # separate allocations: a row slice of the [n, 27] map starts 108 * ni bytes in, which is not
        # 16-byte aligned in general, and the tensor-core kernel reads the map in 16-byte vectors
        self.nbr_int = plan.nbr_local[:ni].clone()
        self.nbr_bnd = plan.nbr_local[ni:].clone()
        if _scheds is not None:
            self.sched_int, self.sched_bnd, self.ts_int, self.ts_bnd = _scheds
        else:
            # conv schedules of the two row sets (tap-mask row order, computed once), and their
            # tile-source plans for the 64-input-channel layers
            n_in = plan.n_local + plan.n_halo
            self.sched_int = F.neighbor_schedule(cfg, self.nbr_int) if ni and schedule else None
            self.sched_bnd = F.neighbor_schedule(cfg, self.nbr_bnd) if plan.n_local > ni and schedule else None
            want_ts = tile_sources and any(c.in_channels == 64 for c in stack.cfgs)
            self.ts_int = F.neighbor_tile_sources(cfg, self.nbr_int, n_in) if ni and want_ts else None
            self.ts_bnd = F.neighbor_tile_sources(cfg, self.nbr_bnd, n_in) if plan.n_local > ni and want_ts else None
        # the last layer writes Morton-local rows directly (epilogue row map: plan row p -> order[p])
        self.order_int = plan.order[:ni].clone()
        self.order_bnd = plan.order[ni:].clone()
        self.bufs = None
        self.comm = None

    def twin(self) -> "ShardedSubmStack":
        """A second instance on the same plan and schedules with its own layer
        buffers (e.g. for a second pipelined input slot)."""
        return ShardedSubmStack(self.stack, self.plan, _scheds=(self.sched_int, self.sched_bnd, self.ts_int, self.ts_bnd))

    def forward(self, x_local: torch.Tensor) -> torch.Tensor:
        """One pass; returns this instance's [n_local, Cout] output buffer (Morton-local rows),
        which the next call on the same instance overwrites."""
        from . import flex_gmm as F

        plan, n, ni = self.plan, self.plan.n_local, self.plan.n_interior
        dev = x_local.device
        if self.bufs is None:
            self.bufs = [plan.buffer(c.in_channels, x_local.dtype, dev) for c in self.stack.cfgs]
            self.out = torch.empty((n, self.stack.cfgs[-1].out_channels), dtype=x_local.dtype, device=dev)
            self.comm = torch.cuda.Stream(dev)
        compute = torch.cuda.current_stream(dev)
        F.gather_rows(x_local, plan.order, out=self.bufs[0][:n])

        def pack(buf):
            """Packs ``buf``'s rows for the peers on the comm stream, after the compute
            stream's work so far; returns (send rows, packed event)."""
            ready = torch.cuda.Event()
            ready.record(compute)
            with torch.cuda.stream(self.comm):
                self.comm.wait_event(ready)
                send = plan.pack(buf)
                packed = torch.cuda.Event()
                packed.record(self.comm)
            return send, packed

        def all_to_all(buf, send):
            """The all-to-all of packed rows into ``buf``'s halo, on the comm stream;
            returns the event of the halo's arrival."""
            with torch.cuda.stream(self.comm):
                plan.exchange(buf, send=send)
                arrived = torch.cuda.Event()
                arrived.record(self.comm)
            return arrived

        from .blocks import layer_epilogue

        layers = list(zip(self.stack.cfgs, self.stack.w, self.stack.b))
        for i, (cfg, w, b) in enumerate(layers):
            buf = self.bufs[i]
            last = i + 1 == len(layers)
            dst = self.out if last else self.bufs[i + 1][:n]
            # this layer's halo on the comm stream, beside the interior rows' conv
            halo = all_to_all(buf, pack(buf)[0])
            for rows, nbr, sched, ts, order, boundary in (
                    (slice(0, ni), self.nbr_int, self.sched_int, self.ts_int, self.order_int, False),
                    (slice(ni, n), self.nbr_bnd, self.sched_bnd, self.ts_bnd, self.order_bnd, True)):
                if boundary:
                    compute.wait_event(halo)
                if rows.stop <= rows.start:
                    continue
                if last:  # rows go straight to their Morton-local place
                    F.sparse_subm_conv_forward(cfg, buf, nbr, w, b, F.Epilogue(
                        silu=self.stack.silu, schedule=sched, out_row_map=order, out_row_map_cols=1),
                        out=dst, out_rows=n)
                else:
                    F.sparse_subm_conv_forward(cfg, buf, nbr, w, b, layer_epilogue(cfg, self.stack.silu, sched, ts),
                                               out=dst[rows])
        return self.out

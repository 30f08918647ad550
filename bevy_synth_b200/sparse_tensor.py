"""Sparse tensor types of the decoder path, mirroring burn_trellis's runtime
types (crates/burn_trellis/src/runtime_model/types/):

=========================  ==================================================
this module                reference
=========================  ==================================================
``SparseBatchLayout``      ``SparseBatchLayoutDevice{offsets, lengths, rows}``
                           (sparse_batch_layout_device.rs:4-26)
``VarLenTensor``           ``VarLenTensorDevice{values, layout, channels}``
                           (varlen_tensor_device.rs:6-28)
``SparseTensor``           ``SparseTensorDevice{coords, values,
                           sparse_resolution}`` (sparse_tensor_device.rs:6-32)
=========================  ==================================================

Coordinates are ``[N, 4]`` int32 ``(batch, x, y, z)`` with rows grouped by
batch in ascending batch order (each batch Morton-sorted), so a batch is a
contiguous row range: ``offsets[i]`` / ``lengths[i]`` give the rows of the
i-th batch present, ``batch_ids[i]`` its index in ``coords[:, 0]``.  A
``SparseTensor`` also caches the neighbor map (and conv schedule) of each
kernel geometry it is convolved with, as the reference caches maps per grid
(burn_flex_gmm src/wgpu.rs:128, 379-382).
"""
from __future__ import annotations

from dataclasses import dataclass, field

import torch

from . import flex_gmm as F


@dataclass
class SparseBatchLayout:
    """Per-batch row ranges of a batch-grouped sparse tensor."""

    offsets: torch.Tensor      # [B] int64: first row of each batch
    lengths: torch.Tensor      # [B] int64: rows of each batch
    rows: int
    batch_ids: torch.Tensor | None = None  # [B] int64: coord[0] of each batch (None: 0..B-1)

    def batch_size(self) -> int:
        return int(self.offsets.shape[0])

    @staticmethod
    def from_coords(coords: torch.Tensor) -> "SparseBatchLayout":
        """The layout of ``coords`` (rows grouped by ascending batch index)."""
        if coords.dim() != 2 or coords.shape[1] != 4:
            raise F.SparseConvError(F._lib.SC_ERR_INVALID,
                                    f"sparse coords must have shape [N, 4], got {list(coords.shape)}")
        n = int(coords.shape[0])
        if n == 0:
            z = torch.zeros(0, dtype=torch.int64, device=coords.device)
            return SparseBatchLayout(z, z.clone(), 0, z.clone())
        b = coords[:, 0].to(torch.int64)
        if n > 1 and bool((b[1:] < b[:-1]).any()):
            raise F.SparseConvError(F._lib.SC_ERR_INVALID, "sparse coords must be grouped by ascending batch index")
        ids, lengths = torch.unique_consecutive(b, return_counts=True)
        offsets = torch.cumsum(lengths, 0) - lengths
        return SparseBatchLayout(offsets, lengths, n, ids)

    def rows_of(self, i: int) -> slice:
        o, n = int(self.offsets[i]), int(self.lengths[i])
        return slice(o, o + n)

    def split(self, t: torch.Tensor) -> list[torch.Tensor]:
        """Row slices of ``t`` (views), one per batch."""
        return [t[self.rows_of(i)] for i in range(self.batch_size())]


@dataclass
class VarLenTensor:
    """Row values of a batch-grouped sparse tensor with their batch layout."""

    values: torch.Tensor       # [rows, channels]
    layout: SparseBatchLayout
    channels: int

    def rows(self) -> int:
        return int(self.values.shape[0])


@dataclass
class SparseTensor:
    """Coordinates, per-row values and the grid resolution of a sparse tensor."""

    coords: torch.Tensor       # [N, 4] int32
    values: VarLenTensor
    sparse_resolution: int
    _maps: dict = field(default_factory=dict, repr=False)

    @staticmethod
    def new(coords: torch.Tensor, feats: torch.Tensor, sparse_resolution: int) -> "SparseTensor":
        if feats.dim() != 2 or feats.shape[0] != coords.shape[0]:
            raise F.SparseConvError(F._lib.SC_ERR_INVALID,
                                    f"sparse values must be [{coords.shape[0]}, C], got {list(feats.shape)}")
        layout = SparseBatchLayout.from_coords(coords)
        return SparseTensor(coords, VarLenTensor(feats, layout, int(feats.shape[1])), sparse_resolution)

    @staticmethod
    def from_batches(parts: list, sparse_resolution: int, batch_ids=None) -> "SparseTensor":
        """One sparse tensor from per-batch ``(coords_xyz [n, 3] or [n, 4], feats [n, C])``
        pairs; batch i gets index ``batch_ids[i]`` (default i) in coord[0]."""
        ids = list(range(len(parts))) if batch_ids is None else list(batch_ids)
        cs, fs = [], []
        for bid, (c, f) in zip(ids, parts):
            c = c[:, -3:] if c.shape[1] == 4 else c
            col = torch.full((c.shape[0], 1), int(bid), dtype=torch.int32, device=c.device)
            cs.append(torch.cat([col, c.to(torch.int32)], 1))
            fs.append(f)
        return SparseTensor.new(torch.cat(cs).contiguous(), torch.cat(fs).contiguous(), sparse_resolution)

    def rows(self) -> int:
        return int(self.coords.shape[0])

    @property
    def feats(self) -> torch.Tensor:
        return self.values.values

    @property
    def layout(self) -> SparseBatchLayout:
        return self.values.layout

    def with_values(self, feats: torch.Tensor) -> "SparseTensor":
        """Same coordinates (and cached maps), new [N, C'] values."""
        if feats.shape[0] != self.rows():
            raise F.SparseConvError(F._lib.SC_ERR_INVALID,
                                    f"sparse values must have {self.rows()} rows, got {feats.shape[0]}")
        return SparseTensor(self.coords, VarLenTensor(feats, self.layout, int(feats.shape[1])),
                            self.sparse_resolution, self._maps)

    def batch(self, i: int) -> "SparseTensor":
        """The i-th batch as its own sparse tensor (row views, batch index kept)."""
        r = self.layout.rows_of(i)
        return SparseTensor.new(self.coords[r], self.feats[r], self.sparse_resolution)

    def neighbor_rows(self, config: F.SparseSubmConvConfig, schedule: bool = True):
        """(map [N, K], conv schedule or None) of this grid for ``config``'s kernel
        geometry, built once and cached on the tensor."""
        key = (config.kernel_d, config.kernel_h, config.kernel_w, tuple(config.axis_order),
               tuple(config.axis_sign), schedule)
        hit = self._maps.get(key)
        if hit is None:
            nbr = F.neighbor_rows_tensor_from_coords_tensor(config, self.coords)
            sched = F.neighbor_schedule(config, nbr) if schedule and F.kernel_rows(config) <= 32 else None
            hit = (nbr, sched)
            self._maps[key] = hit
        return hit


def sparse_subm_conv3d(x: SparseTensor, config: F.SparseSubmConvConfig, weight: torch.Tensor,
                       bias: torch.Tensor | None = None, epilogue: F.Epilogue | None = None) -> SparseTensor:
    """SubM conv of a sparse tensor: same coordinates, new values [N, Cout]
    (the map of the tensor's grid is built on first use and reused)."""
    nbr, sched = x.neighbor_rows(config)
    e = epilogue or F.Epilogue()
    if sched is not None and e.schedule is None and e.row_order is None:
        e.schedule = sched
    y = F.sparse_subm_conv_forward(config, x.feats, nbr, weight, bias, e)
    return x.with_values(y)

"""Seeded synthetic inputs for the five BASELINE configurations.

The reference ships no decoder weights or activations (its hook fixtures are
missing), so every workload is synthetic: ``numpy.random.default_rng(seed)``
drives occupancy, features and weights.  Coordinates are ``[batch, x, y, z]``
int32, sorted by Morton code (x in bit 0) within each batch, batches in
ascending order.  A cell's centre is ``index + 0.5``.
"""
from __future__ import annotations

from dataclasses import dataclass

import numpy as np


# --------------------------------------------------------------------------
# Morton order
# --------------------------------------------------------------------------
def _spread3(v: np.ndarray) -> np.ndarray:
    """Spread the low 21 bits of v so that bit i lands at bit 3i."""
    v = v.astype(np.uint64) & np.uint64(0x1FFFFF)
    v = (v | (v << np.uint64(32))) & np.uint64(0x1F00000000FFFF)
    v = (v | (v << np.uint64(16))) & np.uint64(0x1F0000FF0000FF)
    v = (v | (v << np.uint64(8))) & np.uint64(0x100F00F00F00F00F)
    v = (v | (v << np.uint64(4))) & np.uint64(0x10C30C30C30C30C3)
    v = (v | (v << np.uint64(2))) & np.uint64(0x1249249249249249)
    return v


def morton_code(coords: np.ndarray) -> np.ndarray:
    """Interleaved (x, y, z) code with x in bit 0 (batch not included)."""
    c = np.asarray(coords)
    return _spread3(c[:, 1]) | (_spread3(c[:, 2]) << np.uint64(1)) | (_spread3(c[:, 3]) << np.uint64(2))


def morton_sort(coords: np.ndarray) -> np.ndarray:
    c = np.asarray(coords, np.int32).reshape(-1, 4)
    order = np.lexsort((morton_code(c), c[:, 0]))
    return np.ascontiguousarray(c[order])


def _sorted_unique(key: np.ndarray) -> np.ndarray:
    """Sorted unique values of a 1-D array (sort + adjacent difference: the same
    result as np.unique, whose hash-based path is ~80x slower on 7M int64 keys)."""
    s = np.sort(key)
    if s.size == 0:
        return s
    keep = np.empty(s.size, bool)
    keep[0] = True
    np.not_equal(s[1:], s[:-1], out=keep[1:])
    return s[keep]


def _unique_xyz(xyz: np.ndarray) -> np.ndarray:
    """Unique rows of non-negative [M,3] int coordinates (< 2^21 each), via 1-D keys."""
    xyz = np.asarray(xyz, np.int64).reshape(-1, 3)
    key = _sorted_unique((xyz[:, 0] << 42) | (xyz[:, 1] << 21) | xyz[:, 2])
    mask = (1 << 21) - 1
    return np.stack([key >> 42, (key >> 21) & mask, key & mask], axis=1).astype(np.int32)


def unique_cells(batch: int, xyz: np.ndarray) -> np.ndarray:
    xyz = _unique_xyz(xyz)
    b = np.full((xyz.shape[0], 1), batch, np.int32)
    return np.concatenate([b, xyz], axis=1)


# --------------------------------------------------------------------------
# Shell occupancy
# --------------------------------------------------------------------------
def sphere_shell(grid: int, centre, radius: float, half_thickness: float) -> np.ndarray:
    """Cells whose centre lies within ``half_thickness`` of a sphere."""
    ax = np.arange(grid, dtype=np.float64) + 0.5
    x, y, z = np.meshgrid(ax, ax, ax, indexing="ij")
    d = np.sqrt((x - centre[0]) ** 2 + (y - centre[1]) ** 2 + (z - centre[2]) ** 2)
    m = np.abs(d - radius) <= half_thickness
    return np.argwhere(m).astype(np.int32)


def ellipsoid_shell(grid: int, centre, axes, half_thickness: float) -> np.ndarray:
    """Cells within ``half_thickness`` of an axis-aligned ellipsoid surface,
    using the first-order distance d = (rho - 1) / |grad rho| with
    rho = |(q - centre) / axes|.  Enumerates only candidate cells near the
    surface (column by column), so 1024^3 grids stay cheap."""
    p = np.asarray(centre, np.float64)
    a = np.asarray(axes, np.float64)
    h = half_thickness
    band = (h + 1.0) / a.min()                       # |rho-1| <= h/min(a) is necessary
    lo2, hi2 = max(0.0, 1.0 - band) ** 2, (1.0 + band) ** 2
    x0, x1 = max(0, int(np.floor(p[0] - a[0] - h - 1))), min(grid, int(np.ceil(p[0] + a[0] + h + 2)))
    y0, y1 = max(0, int(np.floor(p[1] - a[1] - h - 1))), min(grid, int(np.ceil(p[1] + a[1] + h + 2)))
    if x0 >= x1 or y0 >= y1:
        return np.zeros((0, 3), np.int32)
    xs, ys = np.meshgrid(np.arange(x0, x1), np.arange(y0, y1), indexing="ij")
    xs, ys = xs.ravel(), ys.ravel()
    X2 = ((xs + 0.5 - p[0]) / a[0]) ** 2
    Y2 = ((ys + 0.5 - p[1]) / a[1]) ** 2
    r2 = X2 + Y2
    keep = r2 <= hi2
    xs, ys, r2 = xs[keep], ys[keep], r2[keep]
    zhi = np.sqrt(np.maximum(hi2 - r2, 0.0)) * a[2]
    zlo = np.sqrt(np.maximum(lo2 - r2, 0.0)) * a[2]
    cand = []
    # the |z - pz| interval [zlo, zhi] on both sides of the centre
    for sign in (-1.0, 1.0):
        if sign < 0:
            za, zb = p[2] - zhi, p[2] - zlo
        else:
            za, zb = p[2] + zlo, p[2] + zhi
        s = np.clip(np.floor(za - 0.5).astype(np.int64) - 1, 0, grid)
        e = np.clip(np.ceil(zb - 0.5).astype(np.int64) + 2, 0, grid)
        n = np.maximum(e - s, 0)
        tot = int(n.sum())
        if tot == 0:
            continue
        idx = np.repeat(np.arange(len(n)), n)
        start = np.repeat(np.cumsum(n) - n, n)
        zz = s[idx] + (np.arange(tot) - start)
        cand.append(np.stack([xs[idx], ys[idx], zz], axis=1))
    if not cand:
        return np.zeros((0, 3), np.int32)
    c = _unique_xyz(np.concatenate(cand)).astype(np.int64)
    u = (c + 0.5 - p) / a
    rho = np.sqrt((u ** 2).sum(1))
    g = np.sqrt(((u / a) ** 2).sum(1)) / np.maximum(rho, 1e-12)
    d = (rho - 1.0) / np.maximum(g, 1e-12)
    return c[np.abs(d) <= h].astype(np.int32)


# --------------------------------------------------------------------------
# Weights and parameters
# --------------------------------------------------------------------------
def kaiming_uniform(rng, cout: int, cin: int, k: int = 3) -> np.ndarray:
    """[Cout, k, k, k, Cin], bound sqrt(6 / fan_in), fan_in = k^3 * Cin."""
    bound = np.sqrt(6.0 / (k ** 3 * cin))
    return rng.uniform(-bound, bound, size=(cout, k, k, k, cin)).astype(np.float32)


def normal_weight(rng, cout: int, cin: int, std: float = 0.02, k: int = 3) -> np.ndarray:
    return (rng.standard_normal((cout, k, k, k, cin)) * std).astype(np.float32)


def resblock_params(rng, c: int, eps: float = 1e-5) -> dict:
    return {
        "ln1_g": (1.0 + 0.1 * rng.standard_normal(c)).astype(np.float32),
        "ln1_b": (0.1 * rng.standard_normal(c)).astype(np.float32),
        "w1": normal_weight(rng, c, c), "b1": np.zeros(c, np.float32),
        "ln2_g": (1.0 + 0.1 * rng.standard_normal(c)).astype(np.float32),
        "ln2_b": (0.1 * rng.standard_normal(c)).astype(np.float32),
        "w2": normal_weight(rng, c, c), "b2": np.zeros(c, np.float32),
        "eps": eps,
    }


def c2s_params(rng, cin: int, cout: int) -> dict:
    return {
        "ln1_g": (1.0 + 0.1 * rng.standard_normal(cin)).astype(np.float32),
        "ln1_b": (0.1 * rng.standard_normal(cin)).astype(np.float32),
        "w1": normal_weight(rng, 8 * cout, cin), "b1": np.zeros(8 * cout, np.float32),
        "w2": normal_weight(rng, cout, cout), "b2": np.zeros(cout, np.float32),
    }


def convnext_params(rng, c: int, hidden: int) -> dict:
    """A ConvNeXt decoder block: SubM C->C, LayerNorm(g, b), Linear C->hidden,
    Linear hidden->C (PyTorch [out, in] layout), weights N(0, 0.02^2)."""
    return {
        "w": normal_weight(rng, c, c), "b": (0.02 * rng.standard_normal(c)).astype(np.float32),
        "norm_g": (1.0 + 0.1 * rng.standard_normal(c)).astype(np.float32),
        "norm_b": (0.1 * rng.standard_normal(c)).astype(np.float32),
        "w0": (0.02 * rng.standard_normal((hidden, c))).astype(np.float32),
        "b0": (0.02 * rng.standard_normal(hidden)).astype(np.float32),
        "w2": (0.02 * rng.standard_normal((c, hidden))).astype(np.float32),
        "b2": (0.02 * rng.standard_normal(c)).astype(np.float32),
    }


# --------------------------------------------------------------------------
# The five configurations
# --------------------------------------------------------------------------
@dataclass
class Workload:
    name: str
    coords: np.ndarray           # [N,4] int32, Morton-sorted per batch
    feats: np.ndarray            # [N,C] float32
    params: object               # config-specific
    extra: dict


def config1(seed: int = 0) -> Workload:
    """64^3, sphere shell radius 24 at (32,32,32), |d-24| <= 1.5; fp32 C=64->64,
    Kaiming-uniform weights, bias 0."""
    rng = np.random.default_rng(seed)
    coords = morton_sort(unique_cells(0, sphere_shell(64, (32.0, 32.0, 32.0), 24.0, 1.5)))
    feats = rng.standard_normal((coords.shape[0], 64)).astype(np.float32)
    w = kaiming_uniform(rng, 64, 64)
    return Workload("cfg1_subm_fp32_64", coords, feats, {"w": w, "b": np.zeros(64, np.float32)}, {})


def config2(seed: int = 0, blocks: int = 4, channels: int = 256) -> Workload:
    """128^3, union of 4 ellipsoid shells (axes U(20,50), thickness 2, centres
    U[32,96]^3); 4 SparseResBlock3d at C=256, weights N(0, 0.02^2)."""
    rng = np.random.default_rng(seed)
    cells = []
    for _ in range(4):
        axes = rng.uniform(20, 50, 3)
        centre = rng.uniform(32, 96, 3)
        cells.append(ellipsoid_shell(128, centre, axes, 1.0))
    coords = morton_sort(unique_cells(0, np.concatenate(cells)))
    feats = rng.standard_normal((coords.shape[0], channels)).astype(np.float32)
    params = [resblock_params(rng, channels) for _ in range(blocks)]
    return Workload("cfg2_resblock_stack_bf16_256", coords, feats, params, {})


def config3(seed: int = 0, channels=(768, 384, 192, 96), res_blocks: int = 2) -> Workload:
    """32^3 at 20% Bernoulli occupancy, C=768; three levels of [C2S upsample
    with a seeded Bernoulli(0.5) child mask + 2 SparseResBlock3d]."""
    rng = np.random.default_rng(seed)
    occ = rng.random((32, 32, 32)) < 0.2
    coords = morton_sort(unique_cells(0, np.argwhere(occ)))
    feats = rng.standard_normal((coords.shape[0], channels[0])).astype(np.float32)
    levels = []
    for cin, cout in zip(channels[:-1], channels[1:]):
        levels.append({"c2s": c2s_params(rng, cin, cout),
                       "res": [resblock_params(rng, cout) for _ in range(res_blocks)],
                       "mask_seed": int(rng.integers(0, 2**31 - 1))})
    return Workload("cfg3_upsample_pyramid_bf16", coords, feats, levels, {})


def child_mask(seed: int, rows: int, p: float = 0.5) -> np.ndarray:
    return (np.random.default_rng(seed).random((rows, 8)) < p).astype(np.uint8)


def config4(seed: int = 0, assets: int = 64, layers: int = 8, channels: int = 512,
            asset_ids=None, feats: bool = True) -> Workload:
    """64 assets, each a 64^3 sphere shell (radius U(16,28), thickness 2) at
    (32,32,32); batch index in coord[0]; 8 x (SubM 512->512 + SiLU).
    ``asset_ids`` selects a subset (a rank's shard) with identical content.
    With ``feats=False`` no host features are drawn; ``extra["rows"]`` holds
    each selected asset's row count and ``extra["feat_seeds"]`` its feature
    seed (for ``device_normal``)."""
    rng = np.random.default_rng(seed)
    radii = rng.uniform(16, 28, assets)
    ws = [normal_weight(rng, channels, channels) for _ in range(layers)]
    bs = [np.zeros(channels, np.float32) for _ in range(layers)]
    ids = range(assets) if asset_ids is None else asset_ids
    parts, fs, rows, seeds = [], [], [], []
    for b in ids:
        c = morton_sort(unique_cells(b, sphere_shell(64, (32.0, 32.0, 32.0), radii[b], 1.0)))
        parts.append(c)
        rows.append(c.shape[0])
        seeds.append(seed * 1000003 + 17 + b)
        if feats:
            frng = np.random.default_rng(seeds[-1])
            fs.append(frng.standard_normal((c.shape[0], channels)).astype(np.float32))
    coords = np.concatenate(parts) if parts else np.zeros((0, 4), np.int32)
    f = (np.concatenate(fs) if fs else np.zeros((0, channels), np.float32)) if feats else None
    return Workload("cfg4_batched_assets_bf16_512", coords, f, {"w": ws, "b": bs},
                    {"radii": radii, "rows": rows, "feat_seeds": seeds})


def config5_coords(seed: int = 0, shells: int = 32, grid: int = 1024,
                   axes_range=(50.0, 130.0)) -> np.ndarray:
    """1024^3, seeded union of 32 ellipsoid shells (thickness 2) -> ~6M cells."""
    rng = np.random.default_rng(seed)
    cells = []
    for _ in range(shells):
        axes = rng.uniform(*axes_range, 3)
        centre = rng.uniform(axes.max() + 4, grid - axes.max() - 4, 3)
        cells.append(ellipsoid_shell(grid, centre, axes, 1.0))
    return morton_sort(unique_cells(0, np.concatenate(cells)))


CONFIG5_CHANNELS = [(64, 64), (64, 256), (256, 256), (256, 256)]


def config5_params(seed: int = 0) -> dict:
    """The four SubM layers of config 5, weights N(0, 0.02^2), bias 0.  Drawn
    from their own stream so that they do not depend on the feature draw."""
    rng = np.random.default_rng(seed + 0x5EED)
    ws = [normal_weight(rng, co, ci) for ci, co in CONFIG5_CHANNELS]
    bs = [np.zeros(co, np.float32) for _, co in CONFIG5_CHANNELS]
    return {"w": ws, "b": bs, "chans": list(CONFIG5_CHANNELS)}


def config5(seed: int = 0, grid: int = 1024, shells: int = 32, feats: bool = True) -> Workload:
    """Four SubM layers on the 1024^3 union of shells: two read C=64 features
    (64->64, 64->256) and two read C=256 (256->256, 256->256).  With
    ``feats=False`` the [N, 64] features are left out (the GPU workloads draw
    them on the device with ``device_normal``)."""
    rng = np.random.default_rng(seed)
    coords = config5_coords(seed, shells, grid)
    f = rng.standard_normal((coords.shape[0], 64)).astype(np.float32) if feats else None
    return Workload("cfg5_sharded_grid_bf16", coords, f, config5_params(seed), {})


def device_normal(seed: int, rows: int, cols: int, device, dtype=None):
    """Seeded N(0, 1) features drawn on a CUDA device (torch's Philox stream):
    the large configs' inputs without a host-side draw of billions of values.
    Deterministic for a given seed, shape and device type."""
    import torch

    g = torch.Generator(device=device)
    g.manual_seed(int(seed))
    x = torch.randn((rows, cols), generator=g, device=device, dtype=torch.float32)
    return x.to(dtype) if dtype is not None else x


def convnext_stage(seed: int = 0, channels: int = 256, hidden: int = 1024, blocks: int = 2) -> Workload:
    """A ConvNeXt decoder stage (not a BASELINE configuration; the production
    TRELLIS.2 decoder block): config 2's 128^3 union of shells, C=256 with a
    4x MLP, bf16."""
    w2 = config2(seed, blocks=1, channels=channels)
    rng = np.random.default_rng(seed + 7)
    params = [convnext_params(rng, channels, hidden) for _ in range(blocks)]
    return Workload("convnext_stage_bf16_256", w2.coords, w2.feats, params, {})

"""Sparse 3-D patchify -- TEST INFRASTRUCTURE (numpy restatement).

Restates burn_flex_gmm's ``sparse_patchify3d_forward_flex`` (src/lib.rs:133-240):
each output row starts as the bias; the patch of the dense input
[B, Cin, T, H, W] at (batch, tubelet*tubelet_size + dt, patch_row*patch_h + py,
patch_col*patch_w + px) is gathered in (c, dt, py, px) order and multiplied by
the weight packed to [K, Cout] (pack_sparse_patchify3d_weight, :203-240: the
Conv3d weight [Cout, Cin, tubelet, patch_h, patch_w] flattened per output
channel in the same order), accumulated onto the bias.  Coordinates are
validated as in validate_sparse_patchify3d_coords (:634-667).
"""
from __future__ import annotations

import numpy as np


def patchify_gather(cfg: dict, coords, x) -> np.ndarray:
    """[rows, K] im2col in (c, dt, py, px) order."""
    cin, T, H, W = cfg["in_channels"], cfg["frames"], cfg["height"], cfg["width"]
    tb, ph, pw = cfg["tubelet_size"], cfg["patch_h"], cfg["patch_w"]
    x = np.asarray(x, np.float32).reshape(-1, cin, T, H, W)
    coords = np.asarray(coords, np.int64).reshape(-1, 4)
    rows = coords.shape[0]
    out = np.zeros((rows, cin * tb * ph * pw), np.float32)
    for r, (b, t, py0, px0) in enumerate(coords):
        if not (0 <= b < x.shape[0] and 0 <= t < T // tb and 0 <= py0 < H // ph and 0 <= px0 < W // pw):
            raise ValueError(f"sparse patchify coord row {r} out of bounds")
        blk = x[b, :, t * tb:(t + 1) * tb, py0 * ph:(py0 + 1) * ph, px0 * pw:(px0 + 1) * pw]
        out[r] = blk.reshape(-1)
    return out


def sparse_patchify3d_forward(cfg: dict, weight, bias, coords, x) -> np.ndarray:
    cols = patchify_gather(cfg, coords, x).astype(np.float64)
    w = np.asarray(weight, np.float64).reshape(cfg["out_channels"], -1)  # [Cout, K] in (c, dt, py, px) order
    return (np.asarray(bias, np.float64)[None, :] + cols @ w.T).astype(np.float32)

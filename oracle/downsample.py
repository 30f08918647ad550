"""Stride-2 sparse downsample conv on the CPU -- TEST INFRASTRUCTURE.

The reference has no downsample convolution (its decoders only upsample), so
this restates the operation from its definition (SparseConv3d with kernel 2,
stride 2, no padding): output cells are the distinct (batch, x//2, y//2, z//2)
of the input cells, sorted by (batch, Morton code); each output sums, over its
8 child cells (a, b, c) in {0,1}^3 that are present, in[child] @ W[:, a, b, c, :]^T,
plus the bias.  Pure numpy loops: small cases only.  Parity unpinned against
the reference (it has no such op)."""
from __future__ import annotations

import numpy as np


def _morton(x: int, y: int, z: int) -> int:
    code = 0
    for i in range(21):
        code |= ((x >> i) & 1) << (3 * i) | ((y >> i) & 1) << (3 * i + 1) | ((z >> i) & 1) << (3 * i + 2)
    return code


def downsample_coords(coords) -> np.ndarray:
    cells = {(int(b), int(x) >> 1, int(y) >> 1, int(z) >> 1) for b, x, y, z in np.asarray(coords)}
    return np.array(sorted(cells, key=lambda c: (c[0], _morton(c[1], c[2], c[3]))), np.int32).reshape(-1, 4)


def conv3d_stride2(coords, feats, weight, bias):
    """Returns (out_coords [M, 4], out [M, Cout]) in fp32 (fp64 accumulation)."""
    coords = np.asarray(coords)
    x = np.asarray(feats, np.float64)
    w = np.asarray(weight, np.float64)            # [Cout, 2, 2, 2, Cin]
    row = {tuple(int(v) for v in c): i for i, c in enumerate(coords)}
    oc = downsample_coords(coords)
    out = np.zeros((oc.shape[0], w.shape[0]), np.float64) + np.asarray(bias, np.float64)[None, :]
    for o, (b, X, Y, Z) in enumerate(oc):
        for a in (0, 1):
            for bb in (0, 1):
                for c in (0, 1):
                    r = row.get((int(b), 2 * int(X) + a, 2 * int(Y) + bb, 2 * int(Z) + c))
                    if r is not None:
                        out[o] += w[:, a, bb, c, :] @ x[r]
    return oc, out.astype(np.float32)

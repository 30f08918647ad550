"""Sparse 3-D patchify oracle (burn_flex_gmm src/lib.rs:133-240) against an
independent per-element loop (CPU only)."""
import numpy as np
import pytest

from oracle import patchify as OP


def test_patchify_matches_loops():
    cfg = dict(in_channels=3, out_channels=5, frames=4, height=6, width=4, tubelet_size=2, patch_h=3, patch_w=2)
    rng = np.random.default_rng(0)
    x = rng.standard_normal((2, 3, 4, 6, 4)).astype(np.float32)
    w = rng.standard_normal((5, 3, 2, 3, 2)).astype(np.float32)
    b = rng.standard_normal(5).astype(np.float32)
    coords = np.array([[0, 0, 0, 0], [1, 1, 1, 1], [0, 1, 0, 1], [1, 0, 1, 0]], np.int32)
    got = OP.sparse_patchify3d_forward(cfg, w, b, coords, x)
    ref = np.zeros((4, 5))
    for r, (bb, t, py0, px0) in enumerate(coords):
        for o in range(5):
            acc = float(b[o])
            for c in range(3):
                for dt in range(2):
                    for py in range(3):
                        for px in range(2):
                            acc += x[bb, c, t * 2 + dt, py0 * 3 + py, px0 * 2 + px] * w[o, c, dt, py, px]
            ref[r, o] = acc
    np.testing.assert_allclose(got, ref, rtol=1e-5, atol=1e-5)


def test_patchify_rejects_out_of_grid():
    cfg = dict(in_channels=1, out_channels=1, frames=2, height=2, width=2, tubelet_size=1, patch_h=1, patch_w=1)
    with pytest.raises(ValueError, match="out of bounds"):
        OP.patchify_gather(cfg, np.array([[0, 2, 0, 0]]), np.zeros((1, 1, 2, 2, 2), np.float32))

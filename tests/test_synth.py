"""CPU checks of the seeded synthetic workloads."""
import numpy as np

from bevy_synth_b200 import synth


def test_morton_code_interleaves_x_in_bit0():
    c = np.array([[0, 1, 0, 0], [0, 0, 1, 0], [0, 0, 0, 1], [0, 3, 3, 3]], np.int32)
    assert synth.morton_code(c).tolist() == [1, 2, 4, 63]


def test_config1_shape_and_order():
    w = synth.config1(0)
    n = w.coords.shape[0]
    assert 21000 <= n <= 22500          # BASELINE: ~21k voxels
    assert w.feats.shape == (n, 64) and w.params["w"].shape == (64, 3, 3, 3, 64)
    key = synth.morton_code(w.coords)
    assert np.all(np.diff(key.astype(np.int64)) > 0)   # unique, Morton-sorted
    c = w.coords[:, 1:] + 0.5
    d = np.linalg.norm(c - 32.0, axis=1)
    assert np.all(np.abs(d - 24.0) <= 1.5)
    bound = np.sqrt(6.0 / 1728.0)
    assert np.abs(w.params["w"]).max() <= bound


def test_ellipsoid_shell_matches_dense_evaluation():
    g = 48
    centre, axes = np.array([23.3, 25.1, 22.7]), np.array([14.0, 9.5, 17.2])
    got = synth.ellipsoid_shell(g, centre, axes, 1.0)
    ax = np.arange(g) + 0.5
    x, y, z = np.meshgrid(ax, ax, ax, indexing="ij")
    q = np.stack([x, y, z], -1).reshape(-1, 3)
    u = (q - centre) / axes
    rho = np.linalg.norm(u, axis=1)
    grad = np.linalg.norm(u / axes, axis=1) / np.maximum(rho, 1e-12)
    d = (rho - 1) / np.maximum(grad, 1e-12)
    exp = np.argwhere((np.abs(d) <= 1.0).reshape(g, g, g))
    assert sorted(map(tuple, got.tolist())) == sorted(map(tuple, exp.tolist()))


def test_config4_asset_subset_is_consistent():
    full = synth.config4(0, assets=4, layers=1, channels=8)
    part = synth.config4(0, assets=4, layers=1, channels=8, asset_ids=[2, 3])
    sel = full.coords[:, 0] >= 2
    np.testing.assert_array_equal(full.coords[sel], part.coords)
    np.testing.assert_array_equal(full.feats[sel], part.feats)
    np.testing.assert_array_equal(full.params["w"][0], part.params["w"][0])

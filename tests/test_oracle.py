"""CPU oracle pinned against the reference's own tests.

Known answers and property tests transcribed from the reference:
* burn_trellis/src/runtime_model/sparse_decoder_tests.rs:189-236 -> [201, 12]
* sparse_decoder_tests.rs:238-292 -> full map row 0 = [-1,0,1], chunk map = [-1,0,-1]
* burn_flex_gmm/src/lib.rs:799-839, 841-861, 863-914, 916-972 -> flex==legacy
  with the reference LCG (lib.rs:764-778), tolerances 1e-5 / 2e-5.
"""
import json
import os

import numpy as np
import pytest

import oracle
from oracle import OracleConfig

GOLDEN = os.path.join(os.path.dirname(__file__), "golden")


def line_coords(n):
    return np.array([[0, x, 0, 0] for x in range(n)], np.uint32)


def grid_coords(nx, ny, nz):
    # lib.rs:784-797 (make_sparse_grid_coords): keep cells with (x+y+z) even
    return np.array([[0, x, y, z] for x in range(nx) for y in range(ny) for z in range(nz)
                     if (x + y + z) % 2 == 0], np.uint32)


def test_lcg_matches_reference_golden():
    g = json.load(open(os.path.join(GOLDEN, "lcg_seed42.json")))
    got = oracle.Lcg(42).take(len(g["values"]))
    np.testing.assert_array_equal(got, np.array(g["values"], np.float32))


def test_kat_uses_neighbor_voxels():
    cfg = OracleConfig(1, 1, 3, 1, 1)
    coords = np.array([[0, 0, 0, 0], [0, 1, 0, 0]], np.uint32)
    out = oracle.subm_conv_forward_flex(cfg, np.array([10.0, 1.0, 100.0], np.float32),
                                        np.zeros(1, np.float32), coords, np.array([1.0, 2.0], np.float32))
    kat = json.load(open(os.path.join(GOLDEN, "kat_neighbor_voxels.json")))
    np.testing.assert_allclose(out.reshape(-1), kat["expected"], atol=1e-5)


def test_kat_query_chunks_keep_global_neighbors():
    kat = json.load(open(os.path.join(GOLDEN, "kat_halo_chunk.json")))
    cfg = OracleConfig(1, 1, 3, 1, 1)
    coords = np.array(kat["coords"], np.uint32)
    full = oracle.build_neighbor_rows(cfg, coords, oracle.DUP_LAST)
    chunk = oracle.build_neighbor_rows(cfg, coords[:1], oracle.DUP_LAST)
    assert full.reshape(-1)[:3].tolist() == kat["full_row0"]
    assert chunk.reshape(-1).tolist() == kat["chunk_rows"]
    w = np.array([10.0, 1.0, 100.0], np.float32)
    x = np.array([1.0, 2.0], np.float32)
    full_out = oracle.subm_conv_flex(cfg, w, np.zeros(1, np.float32), x, full)
    q_out = oracle.subm_conv_flex(cfg, w, np.zeros(1, np.float32), x, full[:1])
    assert q_out.tolist() == full_out[:1].tolist()


def _lcg_case(seed, cfg, coords):
    rng = oracle.Lcg(seed)
    x = rng.take(coords.shape[0] * cfg.in_channels)
    wl = cfg.out_channels * cfg.kernel_rows * (cfg.in_channels // cfg.groups)
    w = rng.take(wl)
    b = rng.take(cfg.out_channels)
    return x, w, b


def test_flex_matches_legacy_small_kernel():
    cfg = OracleConfig(4, 6, 3, 1, 1, groups=2)
    coords = line_coords(16)
    x, w, b = _lcg_case(42, cfg, coords)
    a = oracle.subm_conv_legacy(cfg, w, b, coords, x)
    f = oracle.subm_conv_forward_flex(cfg, w, b, coords, x)
    assert np.abs(a - f).max() <= 1e-5


def test_flex_handles_empty_rows():
    cfg = OracleConfig(2, 2, 1, 1, 1)
    out = oracle.subm_conv_forward_flex(cfg, np.array([1, 0, 0, 1], np.float32),
                                        np.array([0.25, -0.5], np.float32),
                                        np.zeros((0, 4), np.uint32), np.zeros(0, np.float32))
    assert out.size == 0


def test_flex_precomputed_matches_default():
    cfg = OracleConfig(8, 12, 3, 1, 1, groups=2)
    coords = line_coords(32)
    x, w, b = _lcg_case(73, cfg, coords)
    exp = oracle.subm_conv_forward_flex(cfg, w, b, coords, x)
    nbr = oracle.build_neighbor_rows(cfg, coords, oracle.DUP_LAST)
    packed = oracle.pack_flex_weight(cfg, w)
    got = oracle.subm_conv_flex(cfg, w, b, x, nbr, packed=packed)
    assert np.abs(exp - got).max() <= 1e-5


@pytest.mark.parametrize("axis_order", [(0, 1, 2), (2, 1, 0), (1, 2, 0)])
@pytest.mark.parametrize("axis_sign", [(1, 1, 1), (-1, 1, 1), (1, -1, -1)])
def test_flex_matches_legacy_axis_permutations(axis_order, axis_sign):
    coords = grid_coords(6, 5, 4)
    base = OracleConfig(6, 8, 3, 3, 3, groups=2)
    x, w, b = _lcg_case(991, base, coords)
    cfg = OracleConfig(6, 8, 3, 3, 3, groups=2, axis_order=axis_order, axis_sign=axis_sign)
    a = oracle.subm_conv_legacy(cfg, w, b, coords, x)
    f = oracle.subm_conv_forward_flex(cfg, w, b, coords, x)
    assert np.abs(a - f).max() <= 2e-5


def test_kernel_offsets_order():
    off = oracle.kernel_offsets(OracleConfig(1, 1))
    assert off[0].tolist() == [-1, -1, -1] and off[13].tolist() == [0, 0, 0]
    assert off[26].tolist() == [1, 1, 1] and off[1].tolist() == [-1, -1, 0]


def test_duplicate_rule_lowest_vs_last():
    cfg = OracleConfig(4, 4, 3, 3, 1)
    coords = np.concatenate([line_coords(128), np.array([[0, 17, 0, 0], [0, 32, 0, 0],
                                                         [0, 17, 0, 0], [0, 32, 0, 0]], np.uint32)])
    lo = oracle.build_neighbor_rows(cfg, coords, oracle.DUP_LOWEST)
    la = oracle.build_neighbor_rows(cfg, coords, oracle.DUP_LAST)
    # centre tap (k=4 of a 3x3x1 kernel) of row 17: lowest is 17, last is 130
    assert lo[17, 4] == 17 and la[17, 4] == 130
    assert lo[129, 4] == 32 and la[129, 4] == 131 and lo[130, 4] == 17


def test_bf16_round_rne():
    x = np.array([1.0, 1.00390625, 1.005859375, -2.5, 3.0e38], np.float32)
    r = oracle.bf16_round(x)
    assert r[0] == 1.0 and r[1] == 1.0 and r[2] == np.float32(1.0078125) and r[3] == -2.5


def test_layer_norm_two_pass():
    x = np.arange(12, dtype=np.float32).reshape(2, 6)
    y = oracle.layer_norm(x, None, None, 1e-5)
    m = x.mean(1, keepdims=True)
    v = ((x - m) ** 2).mean(1, keepdims=True)
    np.testing.assert_allclose(y, (x - m) / np.sqrt(v + 1e-5), rtol=1e-6, atol=1e-6)


def test_channel2spatial_order():
    coords = np.array([[0, 1, 2, 3]], np.uint32)
    feats = np.arange(16, dtype=np.float32).reshape(1, 16)
    mask = np.array([[1, 0, 0, 1, 0, 0, 0, 1]], np.uint8)
    oc, of = oracle.channel2spatial(coords, feats, mask)
    assert oc.tolist() == [[0, 2, 4, 6], [0, 3, 5, 6], [0, 3, 5, 7]]
    assert of.tolist() == [[0, 1], [6, 7], [14, 15]]


def test_duplicate_coords_match_scan_golden():
    g = json.load(open(os.path.join(GOLDEN, "dup_coords.json")))
    cfg = OracleConfig(4, 4, *g["kernel"])
    got = oracle.build_neighbor_rows(cfg, np.array(g["coords"], np.uint32), oracle.DUP_LOWEST)
    assert got.reshape(-1).tolist() == g["expected_lowest"]

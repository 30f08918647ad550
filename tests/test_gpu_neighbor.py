"""Neighbor map on the GPU vs the CPU oracle: bit-exact (lowest row on
duplicates, the rule of the reference's device builders)."""
import json
import os

import numpy as np
import pytest

import oracle
from bevy_synth_b200 import _lib, synth
from bevy_synth_b200 import flex_gmm as F

from gpu_util import assert_no_fault, gpu_map, ocfg

pytestmark = pytest.mark.gpu
GOLDEN = os.path.join(os.path.dirname(__file__), "golden")


def line_coords(n):
    return np.array([[0, x, 0, 0] for x in range(n)], np.int32)


def grid_coords(nx, ny, nz):
    return np.array([[0, x, y, z] for x in range(nx) for y in range(ny) for z in range(nz)
                     if (x + y + z) % 2 == 0], np.int32)


def check(cfg, coords, query=None):
    got = gpu_map(cfg, coords, query)
    exp = oracle.build_neighbor_rows(ocfg(cfg), np.asarray(coords, np.uint32), oracle.DUP_LOWEST,
                                     None if query is None else np.asarray(query, np.uint32))
    np.testing.assert_array_equal(got, exp)
    return got


def test_line_5000_3x3x3(cuda_device):
    check(F.SparseSubmConvConfig(4, 4), line_coords(5000))


@pytest.mark.parametrize("axis_order", [(0, 1, 2), (2, 1, 0), (1, 2, 0)])
@pytest.mark.parametrize("axis_sign", [(1, 1, 1), (-1, 1, 1), (1, -1, -1)])
def test_grid_axis_permutations(cuda_device, axis_order, axis_sign):
    check(F.SparseSubmConvConfig(6, 8, groups=2, axis_order=axis_order, axis_sign=axis_sign),
          grid_coords(6, 5, 4))


def test_duplicates_keep_lowest_row_golden(cuda_device):
    g = json.load(open(os.path.join(GOLDEN, "dup_coords.json")))
    got = gpu_map(F.SparseSubmConvConfig(4, 4, *g["kernel"]), np.array(g["coords"], np.int32))
    assert got.reshape(-1).tolist() == g["expected_lowest"]


def test_kernel_9x9x9(cuda_device):
    check(F.SparseSubmConvConfig(4, 4, 9, 9, 9), line_coords(256))


def test_halo_chunk_kat(cuda_device):
    kat = json.load(open(os.path.join(GOLDEN, "kat_halo_chunk.json")))
    cfg = F.SparseSubmConvConfig(1, 1, 3, 1, 1)
    coords = np.array(kat["coords"], np.int32)
    full = gpu_map(cfg, coords)
    assert full.reshape(-1)[:3].tolist() == kat["full_row0"]
    chunk = gpu_map(cfg, coords[:1])
    assert chunk.reshape(-1).tolist() == kat["chunk_rows"]
    # querying the chunk against the full table restores the neighbor
    q = gpu_map(cfg, coords, coords[:1])
    assert q.reshape(-1).tolist() == kat["full_row0"]


def test_config1_and_config2_coords(cuda_device):
    cfg = F.SparseSubmConvConfig(4, 4)
    check(cfg, synth.config1(0).coords)
    got = check(cfg, synth.config2(0, blocks=1, channels=8).coords)
    # size-independent properties: centre tap is the row itself; maps are symmetric
    n = got.shape[0]
    assert np.array_equal(got[:, 13], np.arange(n))
    r, k = np.nonzero(got >= 0)
    assert np.array_equal(got[got[r, k], 26 - k], r)


def test_batched_assets_do_not_mix(cuda_device):
    w = synth.config4(0, assets=4, layers=1, channels=8)
    got = check(F.SparseSubmConvConfig(4, 4), w.coords)
    r, k = np.nonzero(got >= 0)
    assert np.array_equal(w.coords[r, 0], w.coords[got[r, k], 0])


def test_query_other_coords(cuda_device):
    a = synth.config1(0).coords
    q = a[::7] + np.array([0, 1, 0, 0], np.int32)
    check(F.SparseSubmConvConfig(4, 4), a, q)


def test_empty_inputs(cuda_device):
    cfg = F.SparseSubmConvConfig(4, 4)
    got = gpu_map(cfg, np.zeros((0, 4), np.int32))
    assert got.shape == (0, 27)


def test_out_of_range_coordinate_is_an_error(cuda_device):
    cfg = F.SparseSubmConvConfig(4, 4)
    coords = np.array([[0, 1, 2, 3], [0, 70000, 0, 0]], np.int32)
    with pytest.raises(_lib.SparseConvError, match="outside") as ei:
        gpu_map(cfg, coords)
    assert ei.value.code == _lib.SC_ERR_RANGE
    assert_no_fault()


def test_near_boundary_coordinates(cuda_device):
    # components at the top of the packable range and at 0 (negative offsets)
    coords = np.array([[0, 65534, 65534, 65534], [0, 65533, 65534, 65534], [7, 0, 0, 0], [7, 1, 0, 0]],
                      np.int32)
    check(F.SparseSubmConvConfig(4, 4), coords)


def test_minimum_workspace_gives_the_same_map(cuda_device):
    """A workspace of the minimum size (table of 2n slots, load factor 0.5) and the
    full one (4n slots) give the same, oracle-exact map; one byte less than the
    minimum is refused."""
    import torch

    from gpu_util import to_dev

    coords = synth.config2(0, blocks=1, channels=8).coords
    cfg = F.SparseSubmConvConfig(4, 4)
    n = coords.shape[0]
    ct = to_dev(coords)
    full = F.neighbor_rows_tensor_from_coords_tensor(cfg, ct)
    cap = 1024
    while cap < 2 * n:
        cap <<= 1
    ws = F.NeighborWorkspace(ct.device, n)
    assert ws.bytes >= 256 + 2 * cap * 16
    ws.bytes = 256 + cap * 16
    small = F.neighbor_rows_tensor_from_coords_tensor(cfg, ct, workspace=ws)
    assert torch.equal(small, full)
    exp = oracle.build_neighbor_rows(ocfg(cfg), np.asarray(coords, np.uint32), oracle.DUP_LOWEST, None)
    np.testing.assert_array_equal(full.cpu().numpy(), exp)
    ws.bytes -= 1
    with pytest.raises(F.SparseConvError):
        F.neighbor_rows_tensor_from_coords_tensor(cfg, ct, workspace=ws)
    assert_no_fault()

"""The tile-source conv path (conv_ts.cuh): 64-input-channel bf16 convs that
stage each 128-row tile's distinct source rows once and build the taps' A
operands in tensor memory.  The plan must describe the map exactly, and the
conv must agree with the generic tensor-core kernel to rounding (rel-L2 <= 1e-6:
the same taps in the same order, the same K-steps) and with the oracle within
the bf16 tolerance."""
import numpy as np
import pytest
import torch

import oracle
from bevy_synth_b200 import synth
from bevy_synth_b200 import flex_gmm as F

from gpu_util import assert_no_fault, ocfg, rel_l2, to_dev

pytestmark = pytest.mark.gpu
UMAX = 576


def shell(grid=40, r=15.0):
    return synth.morton_sort(synth.unique_cells(0, synth.sphere_shell(grid, (grid / 2,) * 3, r, 1.0)))


def plan_arrays(ts, n_rows, K):
    """(u_count, tap_mask, u_rows, lidx) views of a plan buffer (layout of conv_ts.cuh)."""
    nt = (n_rows + 127) // 128
    a16 = lambda b: (b + 15) // 16 * 16
    raw = ts.buf.cpu().numpy()
    off = 64
    u_count = raw[off:off + 4 * nt].view(np.int32)
    off += a16(4 * nt)
    mask = raw[off:off + 4 * nt].view(np.uint32)
    off += a16(4 * nt)
    u_rows = raw[off:off + 4 * nt * UMAX].view(np.int32).reshape(nt, UMAX)
    off += 4 * nt * UMAX
    lidx = raw[off:off + 2 * nt * 128 * K].view(np.uint16).reshape(nt, 128, K)
    return u_count, mask, u_rows, lidx


def test_plan_describes_the_map(cuda_device):
    coords = shell()
    cfg = F.SparseSubmConvConfig.subm3(64, 64)
    nbr = F.neighbor_rows_tensor_from_coords_tensor(cfg, to_dev(coords))
    ts = F.neighbor_tile_sources(cfg, nbr)
    assert ts is not None
    nb = nbr.cpu().numpy()
    n = nb.shape[0]
    u_count, mask, u_rows, lidx = plan_arrays(ts, n, 27)
    assert ts.max_sources == u_count.max()
    for t in range(u_count.shape[0]):
        rows = nb[t * 128:(t + 1) * 128]
        want = np.unique(rows[rows >= 0])
        assert u_count[t] == want.size and np.array_equal(u_rows[t, :want.size], want)
        lid = lidx[t, :rows.shape[0]]
        got = np.where(lid == 0xFFFF, -1, u_rows[t][np.minimum(lid, UMAX - 1)])
        assert np.array_equal(got, rows)
        assert np.all(lidx[t, rows.shape[0]:] == 0xFFFF)
        assert mask[t] == int(sum(1 << k for k in range(27) if (rows[:, k] >= 0).any()))
    assert_no_fault()


@pytest.mark.parametrize("cout,silu", [(64, False), (96, True), (128, False), (32, True)])
def test_tile_source_conv_equals_generic_kernel(cuda_device, monkeypatch, cout, silu):
    coords = shell()
    n = coords.shape[0]
    rng = np.random.default_rng(cout)
    x = rng.standard_normal((n, 64)).astype(np.float32)
    w = (0.05 * rng.standard_normal((cout, 3, 3, 3, 64))).astype(np.float32)
    b = rng.standard_normal(cout).astype(np.float32)
    cfg = F.SparseSubmConvConfig.subm3(64, cout)
    nbr = F.neighbor_rows_tensor_from_coords_tensor(cfg, to_dev(coords))
    ts = F.neighbor_tile_sources(cfg, nbr)
    assert ts is not None
    xd, wd, bd = to_dev(x, torch.bfloat16), to_dev(w, torch.bfloat16), to_dev(b)
    got = F.sparse_subm_conv_forward(cfg, xd, nbr, wd, bd, F.Epilogue(silu=silu, tile_sources=ts))
    monkeypatch.setenv("SC_TC_PAIR", "0")   # the single-CTA generic kernel, same tile rows
    ref_gpu = F.sparse_subm_conv_forward(cfg, xd, nbr, wd, bd, F.Epilogue(silu=silu))
    assert rel_l2(got.float().cpu().numpy(), ref_gpu.float().cpu().numpy()) <= 1e-6
    ref = oracle.subm_conv_flex(ocfg(cfg), oracle.bf16_round(w), b, oracle.bf16_round(x), nbr.cpu().numpy(),
                                threads=8)
    if silu:
        ref = oracle.silu(ref)
    assert rel_l2(got.float().cpu().numpy(), oracle.bf16_round(ref)) <= 1e-2
    assert_no_fault()


@pytest.mark.parametrize("env,cout", [({"SC_TS_WIDE": "1"}, 256), ({"SC_TS_WIDE": "2"}, 256),
                                     ({"SC_TS_WIDE": "1", "SC_TS_TMAEPI": "0"}, 192),
                                     ({"SC_TS_TMAEPI": "1"}, 64), ({"SC_TS_G": "2"}, 64),
                                     ({"SC_TS_NSTG": "1", "SC_TS_SMAX": "16"}, 64)])
def test_tile_source_variants_equal_generic_kernel(cuda_device, monkeypatch, env, cout):
    """The opt-in tile-source variants (wide outputs with one single-buffered accumulator or
    128-wide column tiles, the TMA box-store epilogue, the pipeline-shape switches) give the
    generic kernel's result."""
    coords = shell()
    n = coords.shape[0]
    rng = np.random.default_rng(cout + len(env))
    x = rng.standard_normal((n, 64)).astype(np.float32)
    w = (0.05 * rng.standard_normal((cout, 3, 3, 3, 64))).astype(np.float32)
    b = rng.standard_normal(cout).astype(np.float32)
    cfg = F.SparseSubmConvConfig.subm3(64, cout)
    nbr = F.neighbor_rows_tensor_from_coords_tensor(cfg, to_dev(coords))
    ts = F.neighbor_tile_sources(cfg, nbr)
    xd, wd, bd = to_dev(x, torch.bfloat16), to_dev(w, torch.bfloat16), to_dev(b)
    monkeypatch.setenv("SC_TC_PAIR", "0")
    ref_gpu = F.sparse_subm_conv_forward(cfg, xd, nbr, wd, bd, F.Epilogue())
    for k, v in env.items():
        monkeypatch.setenv(k, v)
    got = F.sparse_subm_conv_forward(cfg, xd, nbr, wd, bd, F.Epilogue(tile_sources=ts))
    assert rel_l2(got.float().cpu().numpy(), ref_gpu.float().cpu().numpy()) <= 1e-6
    assert_no_fault()


def test_plan_over_capacity_falls_back(cuda_device):
    """A map whose tiles read more distinct rows than the staging holds gives no plan; the conv
    then runs on the generic kernel."""
    n = 4096
    rng = np.random.default_rng(1)
    nbr = rng.integers(0, n, size=(n, 27)).astype(np.int32)   # scattered rows: ~3456 distinct per tile
    cfg = F.SparseSubmConvConfig.subm3(64, 64)
    assert F.neighbor_tile_sources(cfg, to_dev(nbr)) is None
    assert "distinct source rows" in F._lib.last_error()
    assert_no_fault()


def test_config5_grid_layers_on_tile_sources(cuda_device):
    """Config 5's 64-channel layers (7.07M rows) through the tile-source plan agree with the
    generic kernel's results to rounding (64->64 takes the tile-source kernel; 64->256, wider
    than it takes, runs on the generic kernel with the plan ignored)."""
    from bevy_synth_b200.workloads import Cfg5
    wl = Cfg5(torch.device("cuda:0"))
    assert wl.tile_sources is not None and wl.tile_sources.max_sources <= UMAX
    x = wl.inputs(0)[0]
    for cfg, w, b in list(zip(wl.stack.cfgs, wl.stack.w, wl.stack.b))[:2]:
        a = F.sparse_subm_conv_forward(cfg, x, wl.nbr, w, b, F.Epilogue(tile_sources=wl.tile_sources))
        c = F.sparse_subm_conv_forward(cfg, x, wl.nbr, w, b, F.Epilogue(schedule=wl.sched))
        assert rel_l2(a.float().cpu().numpy(), c.float().cpu().numpy()) <= 1e-6, cfg
        x = a
    assert_no_fault()

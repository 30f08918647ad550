"""Sparse submanifold conv on the GPU vs the CPU oracle.

Tolerances: fp32 rel-L2 <= 1e-4 (and the reference's device-vs-CPU 1e-4
max-abs bar, burn_flex_gmm/src/wgpu/tests.rs:1360-1503); bf16 rel-L2 <= 1e-2
against the oracle run in fp32 on bf16-rounded inputs and weights."""
import json
import os

import numpy as np
import pytest
import torch

import oracle
from bevy_synth_b200 import _lib, synth
from bevy_synth_b200 import flex_gmm as F

from gpu_util import assert_no_fault, gpu_map, ocfg, rel_l2, to_dev

pytestmark = pytest.mark.gpu
GOLDEN = os.path.join(os.path.dirname(__file__), "golden")
BF16 = torch.bfloat16


def conv_gpu(cfg, coords, x, w, b, dtype=torch.float32, epi=None, nbr=None, **kw):
    if nbr is None:
        nbr = F.neighbor_rows_tensor_from_coords_tensor(cfg, to_dev(coords.astype(np.int32)))
    out = F.sparse_subm_conv_forward(cfg, to_dev(x, dtype), nbr, to_dev(w.reshape(cfg.out_channels, cfg.kernel_d,
                                     cfg.kernel_h, cfg.kernel_w, cfg.in_channels_per_group), dtype),
                                     to_dev(b, torch.float32), epi, **kw)
    return out.float().cpu().numpy(), nbr


def shell(grid=32, r=11.0, t=1.0, seed=0):
    return synth.morton_sort(synth.unique_cells(0, synth.sphere_shell(grid, (grid / 2,) * 3, r, t)))


def test_kat_uses_neighbor_voxels(cuda_device):
    kat = json.load(open(os.path.join(GOLDEN, "kat_neighbor_voxels.json")))
    cfg = F.SparseSubmConvConfig(1, 1, 3, 1, 1)
    out, _ = conv_gpu(cfg, np.array(kat["coords"]), np.array(kat["input"], np.float32).reshape(2, 1),
                      np.array(kat["weight"], np.float32), np.array(kat["bias"], np.float32))
    np.testing.assert_allclose(out.reshape(-1), kat["expected"], atol=1e-5)
    assert_no_fault()


def lcg_case(seed, cfg, n_rows):
    rng = oracle.Lcg(seed)
    x = rng.take(n_rows * cfg.in_channels).reshape(n_rows, cfg.in_channels)
    w = rng.take(cfg.out_channels * cfg.kernel_d * cfg.kernel_h * cfg.kernel_w * cfg.in_channels_per_group)
    b = rng.take(cfg.out_channels)
    return x, w, b


def test_lcg_small_kernel_grouped(cuda_device):
    cfg = F.SparseSubmConvConfig(4, 6, 3, 1, 1, groups=2)
    coords = np.array([[0, i, 0, 0] for i in range(16)], np.int32)
    x, w, b = lcg_case(42, cfg, 16)
    out, _ = conv_gpu(cfg, coords, x, w, b)
    exp = oracle.subm_conv_legacy(ocfg(cfg), w, b, coords.astype(np.uint32), x)
    assert np.abs(out - exp).max() <= 1e-4


@pytest.mark.parametrize("axis_order", [(0, 1, 2), (2, 1, 0), (1, 2, 0)])
@pytest.mark.parametrize("axis_sign", [(1, 1, 1), (-1, 1, 1), (1, -1, -1)])
def test_lcg_axis_permutations(cuda_device, axis_order, axis_sign):
    coords = np.array([[0, x, y, z] for x in range(6) for y in range(5) for z in range(4)
                       if (x + y + z) % 2 == 0], np.int32)
    cfg = F.SparseSubmConvConfig(6, 8, groups=2, axis_order=axis_order, axis_sign=axis_sign)
    x, w, b = lcg_case(991, cfg, coords.shape[0])
    out, _ = conv_gpu(cfg, coords, x, w, b)
    exp = oracle.subm_conv_legacy(ocfg(cfg), w, b, coords.astype(np.uint32), x)
    assert np.abs(out - exp).max() <= 1e-4


def test_config1_fp32_full(cuda_device):
    wl = synth.config1(0)
    cfg = F.SparseSubmConvConfig.subm3(64, 64)
    out, nbr = conv_gpu(cfg, wl.coords, wl.feats, wl.params["w"], wl.params["b"])
    exp = oracle.subm_conv_flex(ocfg(cfg), wl.params["w"], wl.params["b"], wl.feats, nbr.cpu().numpy(), threads=8)
    assert rel_l2(out, exp) <= 1e-4
    assert np.abs(out - exp).max() <= 1e-4
    assert_no_fault()


@pytest.mark.parametrize("cin,cout,scheduled", [(64, 128, True), (32, 64, False), (128, 64, True)])
def test_fp32_tiled_kernel_epilogues(cuda_device, cin, cout, scheduled):
    """The fp32 8x8-per-thread kernel (Cin % 16 == 0, Cout % 64 == 0): bias + residual,
    a scheduled row order, the LayerNorm/SiLU pass, and a row count that is not a
    multiple of its 64-row tile."""
    coords = shell(grid=30, r=10.0, seed=cin)[:-5]
    n = coords.shape[0]
    assert n % 64 != 0
    rng = np.random.default_rng(cin + cout)
    x = rng.standard_normal((n, cin)).astype(np.float32)
    w = (rng.standard_normal((cout, 3, 3, 3, cin)) * 0.05).astype(np.float32)
    b = rng.standard_normal(cout).astype(np.float32)
    res = rng.standard_normal((n, cout)).astype(np.float32)
    g = (1 + 0.1 * rng.standard_normal(cout)).astype(np.float32)
    be = (0.1 * rng.standard_normal(cout)).astype(np.float32)
    cfg = F.SparseSubmConvConfig.subm3(cin, cout)
    nbr = F.neighbor_rows_tensor_from_coords_tensor(cfg, to_dev(coords.astype(np.int32)))
    sched = F.neighbor_schedule(cfg, nbr) if scheduled else None
    out2 = torch.empty((n, cout), dtype=torch.float32, device="cuda:0")
    epi = F.Epilogue(residual=to_dev(res), layer_norm=True, ln_eps=1e-5, ln_gamma=to_dev(g), ln_beta=to_dev(be),
                     silu=True, out2=out2, schedule=sched)
    out, _ = conv_gpu(cfg, coords, x, w, b, torch.float32, epi, nbr=nbr)
    y = oracle.subm_conv_flex(ocfg(cfg), w, b, x, nbr.cpu().numpy(), threads=8) + res
    assert rel_l2(out, y) <= 1e-4
    assert np.abs(out - y).max() <= 1e-4 * max(1.0, float(np.abs(y).max()))
    exp2 = oracle.silu(oracle.layer_norm(y, g, be, 1e-5))
    assert rel_l2(out2.cpu().numpy(), exp2) <= 1e-4
    assert_no_fault()


def test_fp32_fallback_kernel_odd_channels(cuda_device):
    """Cin = 24 (not a multiple of 16) and Cout = 40: the generic CUDA-core kernel."""
    coords = shell(grid=24, r=8.0)
    rng = np.random.default_rng(11)
    x = rng.standard_normal((coords.shape[0], 24)).astype(np.float32)
    w = (rng.standard_normal((40, 3, 3, 3, 24)) * 0.05).astype(np.float32)
    b = rng.standard_normal(40).astype(np.float32)
    cfg = F.SparseSubmConvConfig.subm3(24, 40)
    out, nbr = conv_gpu(cfg, coords, x, w, b)
    exp = oracle.subm_conv_flex(ocfg(cfg), w, b, x, nbr.cpu().numpy(), threads=8)
    assert rel_l2(out, exp) <= 1e-4
    assert_no_fault()


def bf16_ref(cfg, x, w, b, nbr):
    return oracle.subm_conv_flex(ocfg(cfg), oracle.bf16_round(w), b, oracle.bf16_round(x), nbr, threads=8)


@pytest.mark.parametrize("cin,cout", [(64, 64), (96, 96), (128, 256), (192, 192), (256, 256), (384, 384),
                                      (512, 512), (768, 384), (64, 768), (256, 3072),
                                      (72, 128), (160, 96), (224, 64)])
def test_bf16_tensor_core_widths(cuda_device, cin, cout):
    """Widths on the tcgen05 kernel vs the oracle; Cin of 72, 96, 160, 224 end in a partial
    64-channel chunk whose stage runs only the MMAs of its real channels."""
    coords = shell()
    rng = np.random.default_rng(cin * 7 + cout)
    x = rng.standard_normal((coords.shape[0], cin)).astype(np.float32)
    w = (rng.standard_normal((cout, 3, 3, 3, cin)) * 0.05).astype(np.float32)
    b = rng.standard_normal(cout).astype(np.float32)
    cfg = F.SparseSubmConvConfig.subm3(cin, cout)
    assert F.uses_tensor_cores(cfg, BF16)
    out, nbr = conv_gpu(cfg, coords, x, w, b, BF16)
    exp = bf16_ref(cfg, x, w, b, nbr.cpu().numpy())
    assert rel_l2(out, exp) <= 1e-2, rel_l2(out, exp)
    assert rel_l2(out, exp) <= 4e-3
    assert_no_fault()


def test_bf16_row_tails_and_tap_skipping(cuda_device):
    # rows far apart (only the centre tap valid) plus a dense clump; N % 128 != 0
    rng = np.random.default_rng(5)
    sparse = np.stack([np.zeros(77), rng.choice(20000, 77, replace=False) * 3,
                       np.full(77, 5), np.full(77, 5)], 1).astype(np.int32)
    clump = np.array([[0, x, y, z] for x in range(7) for y in range(7) for z in range(5)], np.int32) + \
        np.array([0, 0, 100, 100], np.int32)
    coords = np.concatenate([sparse, clump])
    cfg = F.SparseSubmConvConfig.subm3(64, 128)
    x = rng.standard_normal((coords.shape[0], 64)).astype(np.float32)
    w = (rng.standard_normal((128, 3, 3, 3, 64)) * 0.05).astype(np.float32)
    b = np.zeros(128, np.float32)
    out, nbr = conv_gpu(cfg, coords, x, w, b, BF16)
    assert rel_l2(out, bf16_ref(cfg, x, w, b, nbr.cpu().numpy())) <= 4e-3
    assert_no_fault()


def _epi_case(c=256, seed=1):
    coords = shell(seed=seed)
    rng = np.random.default_rng(seed)
    n = coords.shape[0]
    x = rng.standard_normal((n, c)).astype(np.float32)
    w = (rng.standard_normal((c, 3, 3, 3, c)) * 0.02).astype(np.float32)
    b = (0.1 * rng.standard_normal(c)).astype(np.float32)
    res = rng.standard_normal((n, c)).astype(np.float32)
    g = (1 + 0.1 * rng.standard_normal(c)).astype(np.float32)
    be = (0.1 * rng.standard_normal(c)).astype(np.float32)
    return coords, x, w, b, res, g, be


@pytest.mark.parametrize("force_simt", [False, True])
def test_bf16_epilogue_ln_silu(cuda_device, force_simt, monkeypatch):
    if force_simt:
        monkeypatch.setenv("SC_FORCE_SIMT", "1")
    coords, x, w, b, res, g, be = _epi_case()
    cfg = F.SparseSubmConvConfig.subm3(256, 256)
    epi = F.Epilogue(layer_norm=True, ln_eps=1e-5, ln_gamma=to_dev(g), ln_beta=to_dev(be), silu=True)
    out, nbr = conv_gpu(cfg, coords, x, w, b, BF16, epi)
    y = bf16_ref(cfg, x, w, b, nbr.cpu().numpy())
    exp = oracle.silu(oracle.layer_norm(y, g, be, 1e-5))
    assert rel_l2(out, exp) <= 1e-2
    assert_no_fault()


@pytest.mark.parametrize("force_simt", [False, True])
def test_bf16_epilogue_residual_and_second_output(cuda_device, force_simt, monkeypatch):
    if force_simt:
        monkeypatch.setenv("SC_FORCE_SIMT", "1")
    coords, x, w, b, res, g, be = _epi_case(seed=2)
    cfg = F.SparseSubmConvConfig.subm3(256, 256)
    out2 = torch.empty((coords.shape[0], 256), dtype=BF16, device="cuda:0")
    epi = F.Epilogue(residual=to_dev(res, BF16), layer_norm=True, ln_eps=1e-5, ln_gamma=to_dev(g),
                     ln_beta=to_dev(be), silu=True, out2=out2)
    out, nbr = conv_gpu(cfg, coords, x, w, b, BF16, epi)
    y = bf16_ref(cfg, x, w, b, nbr.cpu().numpy()) + oracle.bf16_round(res)
    assert rel_l2(out, y) <= 1e-2
    exp2 = oracle.silu(oracle.layer_norm(y, g, be, 1e-5))
    assert rel_l2(out2.float().cpu().numpy(), exp2) <= 1e-2
    assert_no_fault()


def test_bf16_row_map_and_residual_offsets(cuda_device):
    # C2S conv1 shape: Cin=128 -> 8 blocks of 64, scattered to child rows with
    # per-block LayerNorm (no affine) + SiLU; then conv2 with the skip path.
    coords = shell(grid=20, r=6.0)
    n = coords.shape[0]
    rng = np.random.default_rng(9)
    cin, cc = 128, 64
    x = rng.standard_normal((n, cin)).astype(np.float32)
    w1 = (rng.standard_normal((8 * cc, 3, 3, 3, cin)) * 0.03).astype(np.float32)
    b1 = np.zeros(8 * cc, np.float32)
    mask = (rng.random((n, 8)) < 0.5).astype(np.uint8)
    child_row, child_coords, skip = F.subdivide(to_dev(coords), to_dev(mask), cin)
    oc, _ = oracle.channel2spatial(coords.astype(np.uint32), np.zeros((n, cin), np.float32), mask)
    np.testing.assert_array_equal(child_coords.cpu().numpy(), oc.astype(np.int32))
    nc = child_coords.shape[0]
    cfg1 = F.SparseSubmConvConfig.subm3(cin, 8 * cc)
    assert F.uses_tensor_cores(cfg1, BF16)
    epi = F.Epilogue(layer_norm=True, ln_width=cc, ln_eps=1e-6, silu=True, out_row_map=child_row,
                     out_row_map_cols=8)
    out, nbr = conv_gpu(cfg1, coords, x, w1, b1, BF16, epi, out_rows=nc)
    y1 = bf16_ref(cfg1, x, w1, b1, nbr.cpu().numpy())
    _, hup = oracle.channel2spatial(coords.astype(np.uint32), y1, mask)
    exp = oracle.silu(oracle.layer_norm(hup, None, None, 1e-6))
    assert rel_l2(out, exp) <= 1e-2
    # conv2 with the repeat-interleaved parent skip (rep = 64 / (128/8) = 4)
    w2 = (rng.standard_normal((cc, 3, 3, 3, cc)) * 0.03).astype(np.float32)
    cfg2 = F.SparseSubmConvConfig.subm3(cc, cc)
    h_up = to_dev(out, BF16)
    epi2 = F.Epilogue(residual=to_dev(x, BF16), residual_offset=skip, residual_repeat=4)
    out2, nbr2 = conv_gpu(cfg2, child_coords.cpu().numpy(), out, w2, np.zeros(cc, np.float32), BF16, epi2)
    _, xup = oracle.channel2spatial(coords.astype(np.uint32), oracle.bf16_round(x), mask)
    exp2 = bf16_ref(cfg2, out, w2, np.zeros(cc, np.float32), nbr2.cpu().numpy()) + np.repeat(xup, 4, axis=1)
    assert rel_l2(out2, exp2) <= 1e-2
    assert_no_fault()


def test_bf16_simt_fallback_grouped(cuda_device):
    coords = shell(grid=16, r=5.0)
    cfg = F.SparseSubmConvConfig.subm3(24, 40)
    cfg = F.SparseSubmConvConfig(24, 40, groups=2)
    assert not F.uses_tensor_cores(cfg, BF16)
    rng = np.random.default_rng(3)
    x = rng.standard_normal((coords.shape[0], 24)).astype(np.float32)
    w = rng.standard_normal((40, 3, 3, 3, 12)).astype(np.float32) * 0.1
    b = rng.standard_normal(40).astype(np.float32)
    out, nbr = conv_gpu(cfg, coords, x, w, b, BF16)
    assert rel_l2(out, bf16_ref(cfg, x, w, b, nbr.cpu().numpy())) <= 1e-2


def test_tensor_cores_agree_with_simt(cuda_device, monkeypatch):
    coords = shell()
    rng = np.random.default_rng(11)
    x = rng.standard_normal((coords.shape[0], 192)).astype(np.float32)
    w = (rng.standard_normal((192, 3, 3, 3, 192)) * 0.03).astype(np.float32)
    b = np.zeros(192, np.float32)
    cfg = F.SparseSubmConvConfig.subm3(192, 192)
    tc, nbr = conv_gpu(cfg, coords, x, w, b, BF16)
    monkeypatch.setenv("SC_FORCE_SIMT", "1")
    simt, _ = conv_gpu(cfg, coords, x, w, b, BF16, nbr=nbr)
    assert rel_l2(tc, simt) <= 5e-3


def test_bad_neighbor_index_reads_zero_and_raises_fault(cuda_device):
    cfg = F.SparseSubmConvConfig.subm3(64, 64)
    coords = shell(grid=12, r=3.0)
    n = coords.shape[0]
    nbr = F.neighbor_rows_tensor_from_coords_tensor(cfg, to_dev(coords))
    bad = nbr.clone()
    bad[0, 0] = n + 1000  # outside [-1, n_in): the kernels' bounds check turns it into an error
    x = to_dev(np.ones((n, 64), np.float32), BF16)
    w = to_dev(np.zeros((64, 3, 3, 3, 64), np.float32), BF16)
    F.sparse_subm_conv_forward(cfg, x, bad, w, None)
    torch.cuda.synchronize()
    assert _lib.device_fault() & 2
    assert _lib.device_fault() == 0  # reading clears the word


def test_full_size_config2_layer_sampled_rows(cuda_device):
    """One C=256 layer at BASELINE config 2 size; a Morton-contiguous and a
    random sample of rows checked against the oracle (size-independent)."""
    wl = synth.config2(0, blocks=1)
    cfg = F.SparseSubmConvConfig.subm3(256, 256)
    p = wl.params[0]
    out, nbr = conv_gpu(cfg, wl.coords, wl.feats, p["w1"], p["b1"], BF16)
    nb = nbr.cpu().numpy()
    rows = np.concatenate([np.arange(0, 2048), np.random.default_rng(0).choice(nb.shape[0], 2048, False)])
    exp = oracle.subm_conv_flex(ocfg(cfg), oracle.bf16_round(p["w1"]), p["b1"], oracle.bf16_round(wl.feats),
                                nb[rows], threads=8)
    assert rel_l2(out[rows], exp) <= 4e-3
    assert_no_fault()


def test_schedule_is_a_permutation_and_changes_nothing(cuda_device):
    wl = synth.config1(0)
    coords = wl.coords
    cfg = F.SparseSubmConvConfig.subm3(64, 64)
    nbr = F.neighbor_rows_tensor_from_coords_tensor(cfg, to_dev(coords))
    sched = F.neighbor_schedule(cfg, nbr)
    order = sched.order
    o = order.cpu().numpy()
    np.testing.assert_array_equal(sched.nbr_ordered.cpu().numpy(), nbr.cpu().numpy()[o])
    assert np.array_equal(np.sort(o), np.arange(coords.shape[0]))
    # keys are non-decreasing along the order (stable radix sort)
    rng = np.random.default_rng(4)
    x = rng.standard_normal((coords.shape[0], 64)).astype(np.float32)
    w = (rng.standard_normal((64, 3, 3, 3, 64)) * 0.05).astype(np.float32)
    b = rng.standard_normal(64).astype(np.float32)
    base, _ = conv_gpu(cfg, coords, x, w, b, BF16, nbr=nbr)
    ordered, _ = conv_gpu(cfg, coords, x, w, b, BF16, F.Epilogue(schedule=sched), nbr=nbr)
    assert rel_l2(ordered, base) <= 1e-6
    gathered, _ = conv_gpu(cfg, coords, x, w, b, BF16, F.Epilogue(row_order=order), nbr=nbr)
    assert rel_l2(gathered, base) <= 1e-6
    f32, _ = conv_gpu(cfg, coords, x, w, b, torch.float32, F.Epilogue(row_order=order), nbr=nbr)
    exp = oracle.subm_conv_flex(ocfg(cfg), w, b, x, nbr.cpu().numpy(), threads=8)
    assert rel_l2(f32, exp) <= 1e-4
    assert_no_fault()


@pytest.mark.parametrize("c", [96, 192, 320, 384])
def test_bf16_epilogue_writes_stay_inside_rows(cuda_device, c):
    """Outputs go to a view in the middle of a sentinel-filled buffer: the
    guard rows before and after must be untouched, and every element of the
    view must match the oracle (widths whose staging groups are not 128)."""
    coords = shell(grid=20, r=6.0)
    n = coords.shape[0]
    rng = np.random.default_rng(c)
    x = rng.standard_normal((n, c)).astype(np.float32)
    w = (rng.standard_normal((c, 3, 3, 3, c)) * 0.03).astype(np.float32)
    b = (0.1 * rng.standard_normal(c)).astype(np.float32)
    res = rng.standard_normal((n, c)).astype(np.float32)
    g = (1 + 0.1 * rng.standard_normal(c)).astype(np.float32)
    be = (0.1 * rng.standard_normal(c)).astype(np.float32)
    cfg = F.SparseSubmConvConfig.subm3(c, c)
    nbr = F.neighbor_rows_tensor_from_coords_tensor(cfg, to_dev(coords))
    big = torch.full((n + 16, c), 7.0, dtype=BF16, device="cuda:0")
    big2 = torch.full((n + 16, c), 7.0, dtype=BF16, device="cuda:0")
    out, out2 = big[8:8 + n], big2[8:8 + n]
    epi = F.Epilogue(residual=to_dev(res, BF16), layer_norm=True, ln_eps=1e-5, ln_gamma=to_dev(g),
                     ln_beta=to_dev(be), silu=True, out2=out2)
    F.sparse_subm_conv_forward(cfg, to_dev(x, BF16), nbr, to_dev(w, BF16), to_dev(b), epi, out=out)
    torch.cuda.synchronize()
    for t in (big, big2):
        guard = torch.cat([t[:8], t[8 + n:]]).float()
        assert torch.all(guard == 7.0), "write outside the output rows"
    y = bf16_ref(cfg, x, w, b, nbr.cpu().numpy()) + oracle.bf16_round(res)
    assert rel_l2(out.float().cpu().numpy(), y) <= 1e-2
    assert rel_l2(out2.float().cpu().numpy(), oracle.silu(oracle.layer_norm(y, g, be, 1e-5))) <= 1e-2
    plain = F.sparse_subm_conv_forward(cfg, to_dev(x, BF16), nbr, to_dev(w, BF16), to_dev(b))
    assert rel_l2(plain.float().cpu().numpy(), bf16_ref(cfg, x, w, b, nbr.cpu().numpy())) <= 4e-3
    assert_no_fault()


@pytest.mark.parametrize("cin,cout,mode", [(64, 64, "plain"), (96, 96, "ln"), (192, 192, "res_out2"),
                                           (256, 256, "res_out2"), (384, 384, "ln"), (512, 512, "plain"),
                                           (128, 512, "rowmap")])
def test_pair_and_single_cta_kernels_agree(cuda_device, monkeypatch, cin, cout, mode):
    """The 2-SM (CTA pair) kernel against the single-CTA kernel on the same
    inputs: identical arithmetic per row, so results agree to rounding."""
    coords = shell()
    n = coords.shape[0]
    rng = np.random.default_rng(cin + cout)
    x = to_dev(rng.standard_normal((n, cin)).astype(np.float32), BF16)
    w = to_dev((rng.standard_normal((cout, 3, 3, 3, cin)) * 0.03).astype(np.float32), BF16)
    b = to_dev((0.1 * rng.standard_normal(cout)).astype(np.float32))
    cfg = F.SparseSubmConvConfig.subm3(cin, cout)
    nbr = F.neighbor_rows_tensor_from_coords_tensor(cfg, to_dev(coords))

    def run():
        kw, extra = {}, {}
        if mode == "ln":
            epi = F.Epilogue(layer_norm=True, ln_eps=1e-5, silu=True)
        elif mode == "res_out2":
            res = to_dev(rng.standard_normal((n, cout)).astype(np.float32), BF16)
            extra["out2"] = torch.empty((n, cout), dtype=BF16, device="cuda:0")
            epi = F.Epilogue(residual=res, layer_norm=True, ln_eps=1e-5, silu=True, out2=extra["out2"])
        elif mode == "rowmap":
            mask = to_dev((np.random.default_rng(1).random((n, 8)) < 0.5).astype(np.uint8))
            child_row, child_coords, _ = F.subdivide(to_dev(coords), mask, cin)
            kw["out_rows"] = child_coords.shape[0]
            epi = F.Epilogue(layer_norm=True, ln_width=cout // 8, ln_eps=1e-6, silu=True, out_row_map=child_row,
                             out_row_map_cols=8)
        else:
            epi = F.Epilogue(schedule=F.neighbor_schedule(cfg, nbr))
        y = F.sparse_subm_conv_forward(cfg, x, nbr, w, b, epi, **kw)
        outs = [y.float().cpu()] + ([extra["out2"].float().cpu()] if "out2" in extra else [])
        return outs

    rng_state = rng.bit_generator.state
    monkeypatch.setenv("SC_TC_PAIR", "1")
    pair = run()
    rng.bit_generator.state = rng_state
    monkeypatch.setenv("SC_TC_PAIR", "0")
    single = run()
    for a, s in zip(pair, single):
        assert rel_l2(a.numpy(), s.numpy()) <= 1e-6
    assert_no_fault()


@pytest.mark.parametrize("channels,dtype", [(256, BF16), (512, BF16), (768, BF16), (1024, BF16), (96, BF16),
                                            (8, BF16), (16, BF16), (64, BF16), (128, BF16), (192, BF16), (2048, BF16),
                                            (100, BF16),
                                            (256, torch.float32)])
def test_layer_norm_act_rows(cuda_device, channels, dtype):
    """LayerNorm(+affine) -> SiLU, LayerNorm alone and SiLU alone over rows (the row
    kernel the decoder blocks run before their first conv), bf16 and fp32.  The bf16
    widths cover the lane-group sizes of the vector path (8 .. 128 values: 32 to 2
    rows per warp) and the scalar path (wider rows, and 100 values: not a multiple
    of 8); 1000 rows leave a partly filled last warp."""
    rng = np.random.default_rng(channels)
    n = 1000
    x = (rng.standard_normal((n, channels)) * 2 + 0.5).astype(np.float32)
    g = (1 + 0.1 * rng.standard_normal(channels)).astype(np.float32)
    be = (0.1 * rng.standard_normal(channels)).astype(np.float32)
    xd = to_dev(x, dtype)
    xr = xd.float().cpu().numpy()
    tol = 1e-2 if dtype == BF16 else 1e-5
    got = F.layer_norm_affine_silu_forward(xd, to_dev(g), to_dev(be), 1e-5).float().cpu().numpy()
    assert rel_l2(got, oracle.silu(oracle.layer_norm(xr, g, be, 1e-5))) <= tol
    got = F.layer_norm_affine_forward(xd, None, None, 1e-6).float().cpu().numpy()
    assert rel_l2(got, oracle.layer_norm(xr, np.ones(channels, np.float32), np.zeros(channels, np.float32),
                                         1e-6)) <= tol
    got = F.silu_forward(xd).float().cpu().numpy()
    assert rel_l2(got, oracle.silu(xr)) <= tol
    assert_no_fault()

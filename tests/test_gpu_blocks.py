"""Decoder blocks on the fused GPU path vs the oracle's block compositions
(SparseResBlock3d order: burn_trellis sparse_structure_decoder.rs:111-126;
C2S block order: sparse_decoder_runtime_impl.rs:1237-1345).  bf16 rel-L2
<= 1e-2; fp32 rel-L2 <= 1e-4."""
import numpy as np
import pytest
import torch

import oracle
import oracle.blocks as OB
from bevy_synth_b200 import blocks, synth
from bevy_synth_b200 import flex_gmm as F

from gpu_util import assert_no_fault, dev, rel_l2, to_dev

pytestmark = pytest.mark.gpu


def shell(grid=32, r=11.0):
    return synth.morton_sort(synth.unique_cells(0, synth.sphere_shell(grid, (grid / 2,) * 3, r, 1.0)))


@pytest.mark.parametrize("c,dtype,tol", [(64, torch.bfloat16, 1e-2), (256, torch.bfloat16, 1e-2),
                                         (64, torch.float32, 1e-4)])
def test_resblock_stack(cuda_device, c, dtype, tol):
    coords = shell()
    rng = np.random.default_rng(c)
    x = rng.standard_normal((coords.shape[0], c)).astype(np.float32)
    params = [synth.resblock_params(rng, c) for _ in range(3)]
    nbr = F.neighbor_rows_tensor_from_coords_tensor(F.SparseSubmConvConfig.subm3(c, c), to_dev(coords))
    stack = blocks.ResBlockStack([blocks.ResBlockParams.from_numpy(p, dev(), dtype) for p in params])
    got = stack.forward(to_dev(x, dtype), nbr).float().cpu().numpy()
    ref = OB.resblock_stack(x, nbr.cpu().numpy(), params, bf16=dtype == torch.bfloat16)
    assert rel_l2(got, ref) <= tol, rel_l2(got, ref)
    assert_no_fault()


@pytest.mark.parametrize("cin,cout", [(256, 128), (192, 96)])
def test_c2s_block(cuda_device, cin, cout):
    coords = shell(grid=24, r=8.0)
    n = coords.shape[0]
    rng = np.random.default_rng(cin)
    x = rng.standard_normal((n, cin)).astype(np.float32)
    p = synth.c2s_params(rng, cin, cout)
    mask = synth.child_mask(7, n)
    blk = blocks.C2SUpsampleBlock(blocks.C2SParams.from_numpy(p, dev()))
    cc, y, _ = blk.forward(to_dev(coords), to_dev(x, torch.bfloat16), to_dev(mask))
    rc, ry = OB.c2s_block(coords, x, mask, p, bf16=True)
    np.testing.assert_array_equal(cc.cpu().numpy(), rc.astype(np.int32))
    assert rel_l2(y.float().cpu().numpy(), ry) <= 1e-2
    assert_no_fault()


def test_mini_upsample_pyramid(cuda_device):
    """Config-3 structure at reduced width/size: 12^3 grid, 256->128->64->32."""
    rng = np.random.default_rng(0)
    occ = rng.random((12, 12, 12)) < 0.2
    coords = synth.morton_sort(synth.unique_cells(0, np.argwhere(occ)))
    chans = (256, 128, 64, 32)
    x = rng.standard_normal((coords.shape[0], chans[0])).astype(np.float32)
    levels = [{"c2s": synth.c2s_params(rng, a, b), "res": [synth.resblock_params(rng, b)],
               "mask_seed": 100 + i} for i, (a, b) in enumerate(zip(chans[:-1], chans[1:]))]
    pyr = blocks.UpsamplePyramid(levels, dev())
    c_t, x_t = to_dev(coords), to_dev(x, torch.bfloat16)
    c_o, x_o = coords, x
    for (c2s, res, seed), lv in zip(pyr.levels, levels):
        mask = synth.child_mask(seed, c_t.shape[0])
        c_t, x_t, nbr = c2s.forward(c_t, x_t, to_dev(mask))
        x_t = res.forward(x_t, nbr)
        c_o, x_o = OB.c2s_block(c_o, x_o, mask, lv["c2s"], bf16=True)
        x_o = OB.resblock_stack(x_o, OB.neighbor_map(c_o), lv["res"], bf16=True)
        np.testing.assert_array_equal(c_t.cpu().numpy(), c_o.astype(np.int32))
    assert rel_l2(x_t.float().cpu().numpy(), x_o) <= 1e-2
    assert_no_fault()


def test_full_size_config2_stack_tc_vs_fp32(cuda_device, monkeypatch):
    """BASELINE config 2 at full size: the bf16 tcgen05 stack against an
    independent fp32 CUDA-core run of the same stack."""
    wl = synth.config2(0)
    c = 256
    ct = to_dev(wl.coords)
    nbr = F.neighbor_rows_tensor_from_coords_tensor(F.SparseSubmConvConfig.subm3(c, c), ct)
    bf = blocks.ResBlockStack([blocks.ResBlockParams.from_numpy(p, dev(), torch.bfloat16) for p in wl.params])
    y_bf = bf.forward(to_dev(wl.feats, torch.bfloat16), nbr).float()
    f32 = blocks.ResBlockStack([blocks.ResBlockParams.from_numpy(p, dev(), torch.float32) for p in wl.params])
    y_32 = f32.forward(to_dev(wl.feats, torch.float32), nbr)
    r = float(torch.linalg.norm(y_bf - y_32) / torch.linalg.norm(y_32))
    assert r <= 1e-2, r
    assert_no_fault()


def test_resblock_stack_with_schedule_matches_plain(cuda_device):
    coords = shell()
    rng = np.random.default_rng(3)
    c = 128
    x = rng.standard_normal((coords.shape[0], c)).astype(np.float32)
    params = [synth.resblock_params(rng, c) for _ in range(2)]
    cfg = F.SparseSubmConvConfig.subm3(c, c)
    nbr = F.neighbor_rows_tensor_from_coords_tensor(cfg, to_dev(coords))
    stack = blocks.ResBlockStack([blocks.ResBlockParams.from_numpy(p, dev()) for p in params])
    xt = to_dev(x, torch.bfloat16)
    a = stack.forward(xt, nbr).float().clone()
    b = stack.forward(xt, nbr, schedule=F.neighbor_schedule(cfg, nbr)).float()
    assert rel_l2(b.cpu().numpy(), a.cpu().numpy()) <= 1e-6
    assert_no_fault()


@pytest.mark.parametrize("rows,cin,cout,dtype,tol", [(5000, 256, 1024, torch.bfloat16, 1e-2),
                                                     (3000, 1024, 256, torch.bfloat16, 1e-2),
                                                     (777, 96, 64, torch.bfloat16, 1e-2),
                                                     (1000, 64, 64, torch.float32, 1e-4)])
def test_linear_forward(cuda_device, rows, cin, cout, dtype, tol):
    """Linear layer (sparse_decoder_wgpu_ops.rs:1-60) as a 1x1x1 conv over the identity map."""
    rng = np.random.default_rng(rows)
    x = rng.standard_normal((rows, cin)).astype(np.float32)
    w = (0.05 * rng.standard_normal((cout, cin))).astype(np.float32)
    b = rng.standard_normal(cout).astype(np.float32)
    got = F.linear_forward(to_dev(x, dtype), to_dev(w, dtype), to_dev(b)).float().cpu().numpy()
    ref = OB.linear(x, w, b, bf16=dtype == torch.bfloat16)
    if dtype == torch.bfloat16:
        ref = oracle.bf16_round(ref)
    assert rel_l2(got, ref) <= tol, rel_l2(got, ref)
    assert_no_fault()


def test_linear_forward_errors(cuda_device):
    x = to_dev(np.zeros((4, 64), np.float32), torch.bfloat16)
    with pytest.raises(F.SparseConvError, match="invalid input len"):
        F.linear_forward(x, to_dev(np.zeros((32, 48), np.float32), torch.bfloat16))
    with pytest.raises(F.SparseConvError, match="bias len 16 does not match out_channels 32"):
        F.linear_forward(x, to_dev(np.zeros((32, 64), np.float32), torch.bfloat16), to_dev(np.zeros(16, np.float32)))


@pytest.mark.parametrize("c,hidden,nblocks", [(64, 256, 2), (256, 1024, 2)])
def test_convnext_stack(cuda_device, c, hidden, nblocks):
    """ConvNeXt decoder blocks (sparse_decoder_wgpu_ops.rs:1090-1161, MLP :355-489) vs the oracle."""
    coords = shell()
    rng = np.random.default_rng(c + hidden)
    x = rng.standard_normal((coords.shape[0], c)).astype(np.float32)
    params = [synth.convnext_params(rng, c, hidden) for _ in range(nblocks)]
    cfg = F.SparseSubmConvConfig.subm3(c, c)
    nbr = F.neighbor_rows_tensor_from_coords_tensor(cfg, to_dev(coords))
    stack = blocks.ConvNeXtStack([blocks.ConvNeXtParams.from_numpy(p, dev()) for p in params])
    for sched in (None, F.neighbor_schedule(cfg, nbr)):
        got = stack.forward(to_dev(x, torch.bfloat16), nbr, sched).float().cpu().numpy()
        ref = OB.convnext_stack(x, nbr.cpu().numpy(), params, bf16=True)
        assert rel_l2(got, ref) <= 1e-2, rel_l2(got, ref)
    assert_no_fault()

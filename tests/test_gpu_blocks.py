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


def test_c2s_conv2_emits_next_layer_norm(cuda_device):
    """With next_ln, the upsample's conv2 epilogue also writes SiLU(LN(y)) (the first
    ResBlock's input) as a second output: equal to the row kernel run on y."""
    coords = shell(grid=24, r=8.0)
    n = coords.shape[0]
    rng = np.random.default_rng(5)
    x = rng.standard_normal((n, 192)).astype(np.float32)
    p = synth.c2s_params(rng, 192, 96)
    mask = synth.child_mask(9, n)
    blk = blocks.C2SUpsampleBlock(blocks.C2SParams.from_numpy(p, dev()))
    g = torch.as_tensor((1 + 0.1 * rng.standard_normal(96)).astype(np.float32), device=dev())
    be = torch.as_tensor((0.1 * rng.standard_normal(96)).astype(np.float32), device=dev())
    keep = {}
    _, y, _ = blk.forward(to_dev(coords), to_dev(x, torch.bfloat16), to_dev(mask), keep=keep, next_ln=(g, be, 1e-5))
    ref = F.layer_norm_affine_silu_forward(y, g, be, 1e-5)
    assert rel_l2(keep["h_next"].float().cpu().numpy(), ref.float().cpu().numpy()) <= 1e-2
    assert_no_fault()


@pytest.mark.parametrize("n_keep", ["random", "none", "all"])
def test_subdivide_async_matches_sync(cuda_device, n_keep):
    """sc_subdivide_async leaves the child count on the device and writes the same child rows,
    coordinates and skip offsets as sc_subdivide (which reads the count back)."""
    coords = to_dev(shell(grid=24, r=8.0))
    n = coords.shape[0]
    mask = synth.child_mask(3, n)
    if n_keep != "random":
        mask[:] = 1 if n_keep == "all" else 0
    m = to_dev(mask)
    row_s, cc_s, sk_s = F.subdivide(coords, m, 64)
    row_a, cc_a, sk_a, count = F.subdivide_async(coords, m, 64)
    k = count.value()
    assert k == cc_s.shape[0] == int(mask.sum())
    assert cc_a.shape[0] == 8 * n
    assert torch.equal(row_a, row_s)
    assert torch.equal(cc_a[:k], cc_s)
    assert torch.equal(sk_a[:k], sk_s)
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


@pytest.mark.parametrize("rows,cin,cout,silu,residual", [(5000, 256, 1024, True, False), (3000, 1024, 256, False, True),
                                                       (777, 72, 128, True, True), (100, 64, 64, False, False),
                                                       (70000, 256, 768, True, False),
                                                       (500, 64, 96, True, False)])
def test_dense_linear_matches_conv_route(cuda_device, monkeypatch, rows, cin, cout, silu, residual):
    """The dense tensor-core linear (sc_linear_forward: TMA tiles, no map) against the same
    layer as a 1x1x1 conv over the identity map (SC_LINEAR_TC=0) and against the oracle:
    partial row tiles, a partial 64-channel chunk (72), split output tiles (768, 1024),
    SiLU and the residual add; 96 outputs (not a multiple of 64) take the conv route."""
    rng = np.random.default_rng(rows + cin)
    x = rng.standard_normal((rows, cin)).astype(np.float32)
    w = (0.05 * rng.standard_normal((cout, cin))).astype(np.float32)
    b = rng.standard_normal(cout).astype(np.float32)
    r = rng.standard_normal((rows, cout)).astype(np.float32)
    xd, wd, bd = to_dev(x, torch.bfloat16), to_dev(w, torch.bfloat16), to_dev(b)
    rd = to_dev(r, torch.bfloat16) if residual else None
    epi = F.Epilogue(silu=silu, residual=rd)
    dense = F.linear_forward(xd, wd, bd, epi)
    monkeypatch.setenv("SC_LINEAR_TC", "0")
    conv = F.linear_forward(xd, wd, bd, epi)
    monkeypatch.delenv("SC_LINEAR_TC")
    assert rel_l2(dense.float().cpu().numpy(), conv.float().cpu().numpy()) <= 1e-6
    ref = OB.linear(x, w, b, bf16=True)
    if residual:
        ref = ref + oracle.bf16_round(r)
    if silu:
        ref = oracle.silu(ref)
    assert rel_l2(dense.float().cpu().numpy(), oracle.bf16_round(ref)) <= 1e-2
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


@pytest.mark.parametrize("c,dtype,center,child", [(256, torch.bfloat16, False, None),
                                                  (96, torch.float32, True, None),
                                                  (768, torch.bfloat16, False, [0.1, float("nan"), -0.2, 0, 0, 0, 0, 0.3])])
def test_subdivision_head(cuda_device, c, dtype, center, child):
    """to_subdiv linear + centring + per-child threshold (sparse_decoder_runtime_impl.rs:852-890,
    sparse_decoder_wgpu_ops.rs:928-992, :1813-1822)."""
    rng = np.random.default_rng(c)
    n = 3000
    x = rng.standard_normal((n, c)).astype(np.float32)
    w = (0.1 * rng.standard_normal((8, c))).astype(np.float32)
    b = (0.1 * rng.standard_normal(8)).astype(np.float32)
    logits, mask = F.subdivision_head(to_dev(x, dtype), to_dev(w, dtype), to_dev(b), 0.05, child, center)
    rl, rm = OB.subdivision_head(x, w, b, 0.05, child, center, bf16=dtype == torch.bfloat16)
    got_l = logits.cpu().numpy()
    assert rel_l2(got_l, rl) <= 1e-5, rel_l2(got_l, rl)
    thr = np.array(F.subdivision_child_thresholds(0.05, child), np.float32)
    near = np.abs(rl - thr[None, :]) < 1e-4 * np.abs(rl).max()
    diff = mask.cpu().numpy() != rm
    assert not (diff & ~near).any()
    assert_no_fault()


def test_c2s_block_predicted_mask(cuda_device):
    """C2S upsample with the child mask predicted by to_subdiv (no guide)."""
    coords = shell(grid=24, r=8.0)
    n = coords.shape[0]
    cin, cout = 192, 96
    rng = np.random.default_rng(11)
    x = rng.standard_normal((n, cin)).astype(np.float32)
    p = synth.c2s_params(rng, cin, cout)
    w_sub = (0.1 * rng.standard_normal((8, cin))).astype(np.float32)
    b_sub = np.zeros(8, np.float32)
    xd = to_dev(x, torch.bfloat16)
    _, mask = F.subdivision_head(xd, to_dev(w_sub, torch.bfloat16), to_dev(b_sub))
    blk = blocks.C2SUpsampleBlock(blocks.C2SParams.from_numpy(p, dev()))
    cc, y, _ = blk.forward(to_dev(coords), xd, mask)
    m = mask.cpu().numpy()
    assert 0 < m.sum() < m.size
    rc, ry = OB.c2s_block(coords, x, m, p, bf16=True)
    np.testing.assert_array_equal(cc.cpu().numpy(), rc.astype(np.int32))
    assert rel_l2(y.float().cpu().numpy(), ry) <= 1e-2
    assert_no_fault()


@pytest.mark.parametrize("cin,cout,tb,ph,pw,dtype,tol", [(4, 40, 2, 2, 2, torch.float32, 1e-5),
                                                         (16, 64, 1, 2, 2, torch.bfloat16, 1e-2),
                                                         (8, 128, 2, 2, 2, torch.bfloat16, 1e-2)])
def test_sparse_patchify3d(cuda_device, cin, cout, tb, ph, pw, dtype, tol):
    """Sparse patch embedding (burn_flex_gmm lib.rs:133-240) vs the numpy oracle."""
    from oracle import patchify as OP
    cfg = F.SparsePatchify3dConfig(cin, cout, 8, 16, 12, tb, ph, pw)
    d = dict(cfg.__dict__)
    rng = np.random.default_rng(cin + cout)
    x = rng.standard_normal((2, cin, 8, 16, 12)).astype(np.float32)
    w = (0.1 * rng.standard_normal((cout, cin, tb, ph, pw))).astype(np.float32)
    b = rng.standard_normal(cout).astype(np.float32)
    gt, gh, gw = 8 // tb, 16 // ph, 12 // pw
    allc = np.array([[bb, t, y, xx] for bb in range(2) for t in range(gt) for y in range(gh) for xx in range(gw)],
                    np.int32)
    coords = allc[rng.random(len(allc)) < 0.3]
    got = F.sparse_patchify3d_forward(cfg, to_dev(x, dtype), to_dev(coords), to_dev(w, dtype), to_dev(b))
    xr, wr = (oracle.bf16_round(x), oracle.bf16_round(w)) if dtype == torch.bfloat16 else (x, w)
    ref = OP.sparse_patchify3d_forward(d, wr, b, coords, xr)
    if dtype == torch.bfloat16:
        ref = oracle.bf16_round(ref)
    assert rel_l2(got.float().cpu().numpy(), ref) <= tol, rel_l2(got.float().cpu().numpy(), ref)
    assert_no_fault()


def test_sparse_patchify3d_bad_coords(cuda_device):
    """A coordinate outside the grid: the gather's own check raises the fault word, the row is bias only."""
    from bevy_synth_b200 import _lib
    cfg = F.SparsePatchify3dConfig(2, 32, 2, 4, 4, 1, 2, 2)
    x = to_dev(np.ones((1, 2, 2, 4, 4), np.float32))
    w = to_dev(np.ones((32, 2, 1, 2, 2), np.float32))
    b = to_dev(np.arange(32, dtype=np.float32))
    coords = to_dev(np.array([[0, 0, 0, 0], [0, 5, 0, 0]], np.int32))
    out = F.sparse_patchify3d_forward(cfg, x, coords, w, b).cpu().numpy()
    torch.cuda.synchronize()
    assert _lib.device_fault() != 0
    np.testing.assert_allclose(out[0], np.arange(32) + 8.0)
    np.testing.assert_allclose(out[1], np.arange(32))
    with pytest.raises(F.SparseConvError, match="frames must be divisible by tubelet_size"):
        F.sparse_patchify3d_forward(F.SparsePatchify3dConfig(2, 32, 3, 4, 4, 2, 2, 2), x, coords,
                                    to_dev(np.ones((32, 2, 2, 2, 2), np.float32)), b)


def test_load_decoder_stage_from_safetensors(cuda_device, tmp_path):
    """Weight ingestion (sparse_decoder_loading.rs) -> ConvNeXt stage and C2S block, same results as
    building them from the arrays directly (f32 payloads rounded to bf16 by sc_cast; bf16 payloads copied)."""
    from bevy_synth_b200 import weights as Wt
    c, hidden, cout = 64, 256, 32
    rng = np.random.default_rng(5)
    blocks_np = [synth.convnext_params(rng, c, hidden) for _ in range(2)]
    c2s = synth.c2s_params(rng, c, cout)
    w_sub = (0.1 * rng.standard_normal((8, c))).astype(np.float32)
    t = {}
    for i, p in enumerate(blocks_np):
        pre = f"blocks.1.{i}"
        t.update({f"{pre}.conv.weight": p["w"], f"{pre}.conv.bias": p["b"], f"{pre}.norm.weight": p["norm_g"],
                  f"{pre}.norm.bias": p["norm_b"], f"{pre}.mlp.0.weight": p["w0"], f"{pre}.mlp.0.bias": p["b0"],
                  f"{pre}.mlp.2.weight": p["w2"], f"{pre}.mlp.2.bias": p["b2"]})
    pre = "blocks.1.2"
    t.update({f"{pre}.norm1.weight": c2s["ln1_g"], f"{pre}.norm1.bias": c2s["ln1_b"],
              f"{pre}.conv1.weight": c2s["w1"], f"{pre}.conv1.bias": c2s["b1"],
              f"{pre}.conv2.weight": c2s["w2"], f"{pre}.conv2.bias": c2s["b2"],
              f"{pre}.to_subdiv.weight": w_sub, f"{pre}.to_subdiv.bias": np.zeros(8, np.float32)})
    path = tmp_path / "decoder.safetensors"
    Wt.write_safetensors(path, t, bf16=tuple(k for k in t if k.endswith("mlp.0.weight")))
    st = Wt.read_safetensors(str(path))
    stack = Wt.load_convnext_stage(st, 1, 2, c, dev())
    direct = blocks.ConvNeXtStack([blocks.ConvNeXtParams.from_numpy(p, dev()) for p in blocks_np])
    coords = shell()
    x = to_dev(rng.standard_normal((coords.shape[0], c)).astype(np.float32), torch.bfloat16)
    nbr = F.neighbor_rows_tensor_from_coords_tensor(stack.cfg, to_dev(coords))
    a = stack.forward(x, nbr)
    b = direct.forward(x, nbr)
    assert torch.equal(a, b)
    blk = Wt.load_c2s_block(st, 1, 2, c, cout, dev())
    cc, y, _ = blk.forward(to_dev(coords), a)  # children from the loaded to_subdiv head
    assert cc.shape[0] > 0 and y.shape == (cc.shape[0], cout)
    assert_no_fault()


def test_c2s_grouped_schedule(cuda_device):
    """Parents grouped by kept-children mask (sc_neighbor_schedule_grouped): the order is a permutation
    sorted by group, and conv1's dry-stage skipping leaves the block's output bit-identical."""
    coords = shell(grid=28, r=10.0)
    n = coords.shape[0]
    cin, cout = 128, 64
    rng = np.random.default_rng(4)
    x = to_dev(rng.standard_normal((n, cin)).astype(np.float32), torch.bfloat16)
    p = synth.c2s_params(rng, cin, cout)
    mask = to_dev(synth.child_mask(3, n, 0.3))
    blk = blocks.C2SUpsampleBlock(blocks.C2SParams.from_numpy(p, dev()))
    nbr = F.neighbor_rows_tensor_from_coords_tensor(blk.cfg1, to_dev(coords))
    sched = F.neighbor_schedule(blk.cfg1, nbr, group_mask=mask)
    order = sched.order.cpu().numpy()
    assert np.array_equal(np.sort(order), np.arange(n))
    g = (mask.cpu().numpy().astype(np.int64) << np.arange(8)).sum(1)
    assert np.all(np.diff(g[order]) >= 0)
    np.testing.assert_array_equal(sched.nbr_ordered.cpu().numpy(), nbr.cpu().numpy()[order])
    blk.group_children = True
    c1, y1, _ = blk.forward(to_dev(coords), x, mask)
    blk.group_children = False
    c0, y0, _ = blk.forward(to_dev(coords), x, mask)
    assert torch.equal(c1, c0) and torch.equal(y1, y0)
    assert_no_fault()

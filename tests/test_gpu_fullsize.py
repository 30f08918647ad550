"""BASELINE configurations 2-5 at full size on the GPU against the CPU oracle,
in the pattern of the reference's device-vs-CPU checks
(burn_flex_gmm/src/wgpu/tests.rs:1360-1503): neighbor maps bit-exact, bf16
features within rel-L2 <= 1e-2 of the oracle run in fp32 on bf16-rounded
inputs and weights (rounded where the GPU stores bf16).

Where a whole configuration would take the CPU oracle minutes, each layer is
checked on sampled rows (Morton-contiguous blocks plus random rows) from the
GPU's own input to that layer, so errors cannot compound across layers and a
wrong layer is named."""
import os

import numpy as np
import pytest
import torch

import oracle
import oracle.blocks as OB
from bevy_synth_b200 import blocks, synth
from bevy_synth_b200 import flex_gmm as F
from bevy_synth_b200.workloads import Cfg5

from gpu_util import assert_no_fault, dev, ocfg, rel_l2, to_dev

pytestmark = pytest.mark.gpu
THREADS = os.cpu_count() or 8
TOL = 1e-2


def sample_rows(n: int, seed: int, blocks_of: int = 2048, n_blocks: int = 2, n_random: int = 2048) -> np.ndarray:
    """Morton-contiguous blocks (start, middle) plus random rows, sorted, unique."""
    rng = np.random.default_rng(seed)
    parts = [np.arange(0, min(blocks_of, n))]
    for b in range(1, n_blocks):
        a = (n * b) // n_blocks
        parts.append(np.arange(a, min(a + blocks_of, n)))
    parts.append(rng.integers(0, n, size=min(n_random, n)))
    return np.unique(np.concatenate(parts))


def conv_rows_ref(cfg: F.SparseSubmConvConfig, x_gpu: torch.Tensor, nbr_gpu: torch.Tensor, rows: np.ndarray,
                  w: np.ndarray, b: np.ndarray, silu: bool = False) -> np.ndarray:
    """Oracle flex conv (burn_flex_gmm lib.rs:242-375) of the sampled rows, on the
    GPU's own bf16 input: only the input rows the sampled rows read are copied."""
    r = torch.as_tensor(rows, device=nbr_gpu.device)
    nb = nbr_gpu.index_select(0, r).cpu().numpy()
    used = np.unique(nb[nb >= 0])
    x_sub = x_gpu.index_select(0, torch.as_tensor(used, device=x_gpu.device)).float().cpu().numpy()
    nb_sub = np.where(nb >= 0, np.searchsorted(used, np.maximum(nb, 0)), -1).astype(np.int32)
    y = oracle.subm_conv_flex(ocfg(cfg), oracle.bf16_round(w), b, x_sub, nb_sub, threads=THREADS)
    if silu:
        y = oracle.silu(y)
    return oracle.bf16_round(y)


def rows_of(t: torch.Tensor, rows: np.ndarray) -> np.ndarray:
    return t.index_select(0, torch.as_tensor(rows, device=t.device)).float().cpu().numpy()


def test_config5_full_grid(cuda_device):
    """Config 5: the 7.07M-row map bit-exact against the oracle's build_neighbor_rows; each of
    the 4 layers (64->64 on the CTA-pair kernel, 64->256, 256->256 x2) on sampled rows."""
    wl = Cfg5(dev())
    coords = wl.coords_np
    assert coords.shape[0] > 6_000_000
    ref_map = oracle.build_neighbor_rows(oracle.OracleConfig(64, 64), coords.astype(np.uint32))
    assert np.array_equal(wl.nbr.cpu().numpy(), ref_map)
    del ref_map
    x = wl.inputs(0)[0]
    rows = sample_rows(wl.n_local, 5, blocks_of=4096, n_random=4096)
    for i, (cfg, w, b) in enumerate(zip(wl.stack.cfgs, wl.stack.w, wl.stack.b)):
        y = F.sparse_subm_conv_forward(cfg, x, wl.nbr, w, b, F.Epilogue(schedule=wl.sched))
        ref = conv_rows_ref(cfg, x, wl.nbr, rows, wl.params["w"][i], wl.params["b"][i])
        r = rel_l2(rows_of(y, rows), ref)
        assert r <= TOL, (i, r)
        x = y
    # the stack's own forward gives the same last layer as the layer-by-layer run
    assert torch.equal(wl.step(0), x)
    assert_no_fault()


def test_config4_full_batch(cuda_device):
    """Config 4: 64 assets (795k rows), map bit-exact with no neighbor across assets; each of the
    8 SubM 512->512 + SiLU layers on sampled rows."""
    wl = synth.config4(0, feats=False)
    st = blocks.SubmStack(wl.params["w"], wl.params["b"], True, dev())
    ct = to_dev(wl.coords)
    nbr = F.neighbor_rows_tensor_from_coords_tensor(st.cfgs[0], ct)
    nb = nbr.cpu().numpy()
    assert np.array_equal(nb, oracle.build_neighbor_rows(oracle.OracleConfig(1, 1), wl.coords.astype(np.uint32)))
    valid = nb >= 0
    assert np.all(wl.coords[np.maximum(nb, 0), 0][valid] == np.broadcast_to(wl.coords[:, :1], nb.shape)[valid])
    sched = F.neighbor_schedule(st.cfgs[0], nbr)
    x = torch.cat([synth.device_normal(s, r, 512, dev(), torch.bfloat16)
                   for s, r in zip(wl.extra["feat_seeds"], wl.extra["rows"])])
    rows = sample_rows(x.shape[0], 4, blocks_of=1024, n_random=1024)
    for i, (cfg, w, b) in enumerate(zip(st.cfgs, st.w, st.b)):
        y = F.sparse_subm_conv_forward(cfg, x, nbr, w, b, F.Epilogue(silu=True, schedule=sched))
        ref = conv_rows_ref(cfg, x, nbr, rows, wl.params["w"][i], wl.params["b"][i], silu=True)
        r = rel_l2(rows_of(y, rows), ref)
        assert r <= TOL, (i, r)
        x = y
    assert_no_fault()


def test_config3_full_pyramid(cuda_device):
    """Config 3: the 3-level pyramid 768->384->192->96 (6.6k -> ~420k voxels).  Per level: child
    coordinates bit-exact (channel2spatial order), conv1's LN/SiLU child rows and the C2S
    output on sampled children, and the level's ResBlock stack in full, each from the GPU's own
    input to that step."""
    wl = synth.config3(0)
    pyr = blocks.UpsamplePyramid(wl.params, dev())
    coords = to_dev(wl.coords)
    x = to_dev(wl.feats, torch.bfloat16)
    for li, ((c2s, res, mseed), lv) in enumerate(zip(pyr.levels, wl.params)):
        mask_np = synth.child_mask(mseed, coords.shape[0])
        keep = {}
        cc, y, nb = c2s.forward(coords, x, to_dev(mask_np), keep=keep)
        p = lv["c2s"]
        cin, cout = c2s.cin, c2s.cout
        # child coordinates: the oracle's channel2spatial order, bit-exact
        co = coords.cpu().numpy()
        ref_cc, _ = oracle.channel2spatial(co, np.zeros((co.shape[0], 8), np.float32), mask_np)
        assert np.array_equal(cc.cpu().numpy(), ref_cc.astype(np.int32)), li
        # parents' LN + SiLU
        xs = x.float().cpu().numpy()
        h_ref = oracle.bf16_round(oracle.silu(oracle.layer_norm(xs, p["ln1_g"], p["ln1_b"], OB.C2S_LN_EPS)))
        assert rel_l2(keep["h"].float().cpu().numpy(), h_ref) <= TOL, li
        # conv1 + LN(no affine) + SiLU of sampled children, from the GPU's h
        child_row = keep["child_row"].cpu().numpy()
        par, blk = np.nonzero(child_row >= 0)
        n_child = cc.shape[0]
        # children are numbered parent-major, child-minor
        assert np.array_equal(child_row[par, blk], np.arange(n_child))
        s = sample_rows(n_child, 10 + li, blocks_of=1024, n_random=2048)
        sp, sb = par[s], blk[s]
        up = np.unique(sp)
        # conv1 in fp32 on the parents of the sampled children, then the child block's LN + SiLU
        y1 = oracle.subm_conv_flex(ocfg(c2s.cfg1), oracle.bf16_round(p["w1"]), p["b1"],
                                   *_rows_input(keep["h"], keep["nbr_parent"], up), threads=THREADS)
        blocks_ = y1[np.searchsorted(up, sp)].reshape(len(s), 8, cout)[np.arange(len(s)), sb]
        hup_ref = oracle.bf16_round(oracle.silu(oracle.layer_norm(blocks_, None, None, OB.C2S_LN_EPS)))
        assert rel_l2(rows_of(keep["h_up"], s), hup_ref) <= TOL, li
        # conv2 + repeat-interleaved parent skip, from the GPU's h_up
        y2 = oracle.subm_conv_flex(ocfg(c2s.cfg2), oracle.bf16_round(p["w2"]), p["b2"],
                                   *_rows_input(keep["h_up"], nb, s), threads=THREADS)
        w8 = cin // 8
        skip = np.repeat(np.stack([xs[pp, bb * w8:(bb + 1) * w8] for pp, bb in zip(sp, sb)]), cout // w8, axis=1)
        assert rel_l2(rows_of(y, s), oracle.bf16_round(y2 + skip)) <= TOL, li
        # the level's ResBlock stack in full, from the GPU's C2S output
        assert np.array_equal(nb.cpu().numpy(), OB.neighbor_map(cc.cpu().numpy().astype(np.uint32)))
        xr = res.forward(y, nb)
        ref = OB.resblock_stack(y.float().cpu().numpy(), nb.cpu().numpy(), lv["res"], bf16=True, threads=THREADS)
        assert rel_l2(xr.float().cpu().numpy(), ref) <= TOL, li
        coords, x = cc, xr
    assert coords.shape[0] > 300_000
    assert_no_fault()


def _rows_input(x_gpu, nbr_gpu, rows):
    """(x_sub, nbr_sub) for the oracle: the input rows the sampled rows read, ids remapped."""
    r = torch.as_tensor(rows, device=nbr_gpu.device)
    nb = nbr_gpu.index_select(0, r).cpu().numpy()
    used = np.unique(nb[nb >= 0])
    x_sub = x_gpu.index_select(0, torch.as_tensor(used, device=x_gpu.device)).float().cpu().numpy()
    nb_sub = np.where(nb >= 0, np.searchsorted(used, np.maximum(nb, 0)), -1).astype(np.int32)
    return x_sub, nb_sub


def test_config2_full_stack_vs_oracle(cuda_device):
    """Config 2: the whole 4-block SparseResBlock3d stack (8 fused convs) against the oracle's
    block composition (sparse_structure_decoder.rs:111-126) on all 102k rows."""
    wl = synth.config2(0)
    stack = blocks.ResBlockStack([blocks.ResBlockParams.from_numpy(p, dev()) for p in wl.params])
    nbr = F.neighbor_rows_tensor_from_coords_tensor(stack.cfg, to_dev(wl.coords))
    y = stack.forward(to_dev(wl.feats, torch.bfloat16), nbr, schedule=F.neighbor_schedule(stack.cfg, nbr))
    ref = OB.resblock_stack(wl.feats, nbr.cpu().numpy(), wl.params, bf16=True, threads=THREADS)
    r = rel_l2(y.float().cpu().numpy(), ref)
    assert r <= TOL, r
    assert_no_fault()

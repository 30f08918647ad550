"""Decoder blocks on the fused sparse-conv path.

* ``ResBlockStack`` -- chain of SparseResBlock3d
  (burn_trellis/src/runtime_model/sparse_structure_decoder.rs:111-126):
  ``x + conv2(SiLU(LN2(conv1(SiLU(LN1(x))))))``.  conv1's epilogue applies
  LN2 + SiLU; conv2's epilogue adds the residual and, for every block but the
  last, also emits the next block's SiLU(LN1(.)) as a second output, so each
  block costs exactly two conv launches.
* ``C2SUpsampleBlock`` -- the channel-to-space upsample of the TRELLIS.2
  decoder (host order: sparse_decoder_runtime_impl.rs:1237-1345):
  parents ``LN(g,b) -> SiLU -> SubM(Cin -> 8*Cout)``; conv1's epilogue writes
  each kept child's channel block straight to its child row with
  ``LN(no affine) -> SiLU`` applied (no [Np, 8*Cout] intermediate, no select);
  conv2 on the children adds the repeat-interleaved parent skip in its
  epilogue.
* ``UpsamplePyramid``: levels of [C2S + ResBlocks].
* ``ConvNeXtStack`` -- the production TRELLIS.2 decoder block
  (sparse_decoder.rs:602-609; device order sparse_decoder_wgpu_ops.rs:1090-1161,
  MLP :355-489): SubM conv whose epilogue applies bias + LayerNorm(g, b), then
  mlp_0 (+bias, SiLU fused) and mlp_2 (+bias, + the block input fused) as
  1x1x1 convs over the identity map -- three tcgen05 launches per block, no
  separate LayerNorm / SiLU / add passes.
"""
from __future__ import annotations

from dataclasses import dataclass

import numpy as np
import torch

from . import flex_gmm as F

RESBLOCK_LN_EPS = 1e-5  # sparse_structure_decoder.rs:22
C2S_LN_EPS = 1e-6       # sparse_decoder.rs:43 (LAYER_NORM32_EPS)
CONVNEXT_LN_EPS = 1e-6  # the same constant (sparse_decoder_wgpu_ops.rs:1137-1144)


def _dev(a, device, dtype=None):
    t = torch.as_tensor(np.ascontiguousarray(a), device=device)
    return t.to(dtype) if dtype is not None else t


@dataclass
class ResBlockParams:
    ln1_g: torch.Tensor
    ln1_b: torch.Tensor
    w1: torch.Tensor
    b1: torch.Tensor
    ln2_g: torch.Tensor
    ln2_b: torch.Tensor
    w2: torch.Tensor
    b2: torch.Tensor
    eps: float = RESBLOCK_LN_EPS

    @staticmethod
    def from_numpy(p: dict, device, dtype=torch.bfloat16) -> "ResBlockParams":
        f32 = torch.float32
        return ResBlockParams(_dev(p["ln1_g"], device, f32), _dev(p["ln1_b"], device, f32),
                              _dev(p["w1"], device, dtype), _dev(p["b1"], device, f32),
                              _dev(p["ln2_g"], device, f32), _dev(p["ln2_b"], device, f32),
                              _dev(p["w2"], device, dtype), _dev(p["b2"], device, f32),
                              float(p.get("eps", RESBLOCK_LN_EPS)))


class ResBlockStack:
    def __init__(self, blocks: list[ResBlockParams]):
        self.blocks = blocks
        c = blocks[0].w1.shape[0]
        self.cfg = F.SparseSubmConvConfig.subm3(c, c)
        self.channels = c

    def conv_count(self) -> int:
        return 2 * len(self.blocks)

    def forward(self, x: torch.Tensor, nbr: torch.Tensor, bufs: dict | None = None,
                schedule: "F.ConvSchedule | None" = None, h0: torch.Tensor | None = None) -> torch.Tensor:
        """x [N, C] (bf16 or f32) -> [N, C]; ``nbr`` is the [N, 27] map;
        ``schedule`` (optional) its conv schedule (F.neighbor_schedule); ``h0``
        (optional) SiLU(LN1(x)) of the first block, already computed by the
        producer of x (e.g. the upsample's conv2 epilogue), in a buffer the
        stack may overwrite."""
        n, c = x.shape
        if bufs is None:
            bufs = {}
        if h0 is not None:
            bufs["h"] = h0
        def buf(name):
            t = bufs.get(name)
            if t is None or t.shape != x.shape or t.dtype != x.dtype:
                t = torch.empty_like(x)
                bufs[name] = t
            return t
        b0 = self.blocks[0]
        h = h0 if h0 is not None else F.layer_norm_affine_silu_forward(x, b0.ln1_g, b0.ln1_b, b0.eps, out=buf("h"))
        cur = x
        ping = [buf("x0"), buf("x1")]
        for i, p in enumerate(self.blocks):
            h1 = F.sparse_subm_conv_forward(
                self.cfg, h, nbr, p.w1, p.b1,
                F.Epilogue(layer_norm=True, ln_eps=p.eps, ln_gamma=p.ln2_g, ln_beta=p.ln2_b, silu=True,
                           schedule=schedule),
                out=buf("h1"))
            nxt = ping[i % 2]
            if i + 1 < len(self.blocks):
                q = self.blocks[i + 1]
                e = F.Epilogue(residual=cur, layer_norm=True, ln_eps=q.eps, ln_gamma=q.ln1_g, ln_beta=q.ln1_b,
                               silu=True, out2=h, schedule=schedule)
            else:
                e = F.Epilogue(residual=cur, schedule=schedule)
            F.sparse_subm_conv_forward(self.cfg, h1, nbr, p.w2, p.b2, e, out=nxt)
            cur = nxt
        return cur


@dataclass
class C2SParams:
    ln1_g: torch.Tensor
    ln1_b: torch.Tensor
    w1: torch.Tensor   # [8*Cout, 3, 3, 3, Cin]
    b1: torch.Tensor
    w2: torch.Tensor   # [Cout, 3, 3, 3, Cout]
    b2: torch.Tensor
    w_sub: torch.Tensor | None = None  # to_subdiv [8, Cin] (used when no mask is given)
    b_sub: torch.Tensor | None = None

    @staticmethod
    def from_numpy(p: dict, device, dtype=torch.bfloat16) -> "C2SParams":
        f32 = torch.float32
        sub = (_dev(p["w_sub"], device, dtype), _dev(p["b_sub"], device, f32)) if "w_sub" in p else (None, None)
        return C2SParams(_dev(p["ln1_g"], device, f32), _dev(p["ln1_b"], device, f32), _dev(p["w1"], device, dtype),
                         _dev(p["b1"], device, f32), _dev(p["w2"], device, dtype), _dev(p["b2"], device, f32), *sub)


class C2SUpsampleBlock:
    def __init__(self, p: C2SParams):
        self.p = p
        self.cin = p.w1.shape[4]
        self.cout = p.w2.shape[0]
        self.cfg1 = F.SparseSubmConvConfig.subm3(self.cin, 8 * self.cout)
        self.cfg2 = F.SparseSubmConvConfig.subm3(self.cout, self.cout)
        self.group_children = True
        self.schedule_children = True

    def forward(self, coords: torch.Tensor, x: torch.Tensor, mask: torch.Tensor | None = None, nbr_parent=None,
                threshold: float = 0.0, keep: dict | None = None, next_ln=None):
        """Returns (child_coords, child_feats, child_nbr).  Without ``mask`` the
        children come from the to_subdiv head on x (logits > threshold).  With
        ``keep`` (a dict) the intermediates are left in it: ``h`` (parents after
        LN + SiLU), ``h_up`` (children after conv1's LN + SiLU epilogue),
        ``child_row`` ([Np, 8] child of each parent block), ``nbr_parent``,
        ``sched_child`` (the child map's conv schedule, for the convs that
        follow on the children; None when ``schedule_children`` is off) and,
        with ``next_ln`` = (gamma, beta, eps) of the block that follows,
        ``h_next`` = SiLU(LN(y)) emitted by conv2's epilogue as a second output."""
        p = self.p
        if mask is None:
            if p.w_sub is None:
                raise F.SparseConvError(F._lib.SC_ERR_INVALID,
                                        "decoder stage requires guide_subdivisions but none were provided")
            _, mask = F.subdivision_head(x, p.w_sub, p.b_sub, threshold, return_logits=False)
        # the child count stays on the device until conv1 is enqueued: conv1 writes each kept
        # child's row through child_row and is sized by the 8 * Np bound, so the host reads the
        # count only once the GPU has the parents' LayerNorm, map, schedule and conv1 queued
        child_row, coords_bound, skip_bound, count = F.subdivide_async(coords, mask, self.cin)
        h = F.layer_norm_affine_silu_forward(x, p.ln1_g, p.ln1_b, C2S_LN_EPS)
        if nbr_parent is None:
            nbr_parent = F.neighbor_rows_tensor_from_coords_tensor(self.cfg1, coords)
        # parents grouped by their kept-children mask, then by tap mask: a tile whose
        # parents keep none of a child block skips that block's MMAs (dry stage)
        sched1 = F.neighbor_schedule(self.cfg1, nbr_parent, group_mask=mask) if self.group_children else None
        h_up_bound = F.sparse_subm_conv_forward(
            self.cfg1, h, nbr_parent, p.w1, p.b1,
            F.Epilogue(layer_norm=True, ln_width=self.cout, ln_eps=C2S_LN_EPS, silu=True,
                       out_row_map=child_row, out_row_map_cols=8, schedule=sched1),
            out_rows=coords_bound.shape[0])
        n_child = count.value()
        child_coords, skip_off, h_up = coords_bound[:n_child], skip_bound[:n_child], h_up_bound[:n_child]
        nbr_child = F.neighbor_rows_tensor_from_coords_tensor(self.cfg2, child_coords)
        # the child grid is sparse (config 3: ~7 of 27 taps per row): grouping rows by tap mask
        # halves the executed MMA work of conv2 and of the ResBlock convs that follow
        sched2 = F.neighbor_schedule(self.cfg2, nbr_child) if self.schedule_children and n_child else None
        rep = self.cout // (self.cin // 8)
        h_next = None
        if next_ln is not None:
            g, be, eps = next_ln
            h_next = torch.empty((n_child, self.cout), dtype=x.dtype, device=x.device)
            e2 = F.Epilogue(residual=x, residual_offset=skip_off, residual_repeat=rep, schedule=sched2,
                            layer_norm=True, ln_eps=eps, ln_gamma=g, ln_beta=be, silu=True, out2=h_next)
        else:
            e2 = F.Epilogue(residual=x, residual_offset=skip_off, residual_repeat=rep, schedule=sched2)
        y = F.sparse_subm_conv_forward(self.cfg2, h_up, nbr_child, p.w2, p.b2, e2)
        if keep is not None:
            keep.update(h=h, h_up=h_up, child_row=child_row, nbr_parent=nbr_parent, sched_child=sched2,
                        h_next=h_next)
        return child_coords, y, nbr_child

    def flops(self, nbr_parent: torch.Tensor, nbr_child: torch.Tensor, mask: torch.Tensor) -> float:
        """Algorithmic FLOPs: conv1 counted on kept children only (the
        reference computes all 8 blocks, this path only kept ones)."""
        kept = mask.to(torch.int64)
        p_parent = (nbr_parent >= 0).sum(1).to(torch.int64)
        f1 = 2.0 * float((p_parent[:, None] * kept).sum()) * self.cin * self.cout
        f2 = 2.0 * float((nbr_child >= 0).sum()) * self.cout * self.cout
        return f1 + f2


class UpsamplePyramid:
    """[C2S upsample + ResBlocks] x levels."""

    def __init__(self, levels: list[dict], device, dtype=torch.bfloat16):
        self.levels = []
        for lv in levels:
            self.levels.append((C2SUpsampleBlock(C2SParams.from_numpy(lv["c2s"], device, dtype)),
                                ResBlockStack([ResBlockParams.from_numpy(r, device, dtype) for r in lv["res"]]),
                                lv["mask_seed"]))

    def forward(self, coords: torch.Tensor, x: torch.Tensor, masks: list[torch.Tensor]):
        stats = []
        nbr = None  # a level's child map is the next level's parent map (same 3x3x3 geometry)
        for (c2s, res, _), mask in zip(self.levels, masks):
            keep: dict = {}
            # (emitting the first ResBlock's SiLU(LN1(.)) from conv2's epilogue instead of the row
            # kernel measured no faster on config 3: conv2 with the LayerNorm epilogue took
            # 0.04-0.14 ms longer a level, about what the row kernel costs)
            coords, x, nbr = c2s.forward(coords, x, mask, nbr_parent=nbr, keep=keep)
            x = res.forward(x, nbr, schedule=keep["sched_child"])
            stats.append((coords.shape[0], nbr))
        return coords, x, stats


def layer_epilogue(cfg, silu: bool, schedule=None, tile_sources=None) -> F.Epilogue:
    """Bias [+ SiLU] epilogue of a plain SubM layer: a layer of 64 input and at
    most 128 output channels runs in map order on the map's tile-source plan
    when one is given, every other layer on the map's conv schedule."""
    if tile_sources is not None and cfg.in_channels == 64 and cfg.out_channels <= 128:
        return F.Epilogue(silu=silu, tile_sources=tile_sources)
    return F.Epilogue(silu=silu, schedule=schedule)


class SubmStack:
    """A chain of SubM3x3x3 layers with an optional SiLU after each (BASELINE
    config 4: 8 x (SubM 512->512 + SiLU); config 5: 64->64, 64->256,
    256->256, 256->256)."""

    def __init__(self, weights: list, biases: list, silu: bool, device, dtype=torch.bfloat16):
        self.w = [_dev(w, device, dtype) for w in weights]
        self.b = [_dev(b, device, torch.float32) for b in biases]
        self.cfgs = [F.SparseSubmConvConfig.subm3(w.shape[4], w.shape[0]) for w in weights]
        self.silu = silu

    def conv_count(self) -> int:
        return len(self.w)

    def forward(self, x: torch.Tensor, nbr: torch.Tensor, schedule=None, tile_sources=None) -> torch.Tensor:
        """``schedule``: the map's conv schedule (F.neighbor_schedule); ``tile_sources``: its
        tile-source plan (F.neighbor_tile_sources), taken by the layers with 64 input channels."""
        for cfg, w, b in zip(self.cfgs, self.w, self.b):
            x = F.sparse_subm_conv_forward(cfg, x, nbr, w, b, layer_epilogue(cfg, self.silu, schedule, tile_sources))
        return x

    def flops(self, nbr: torch.Tensor) -> float:
        p = float((nbr >= 0).sum())
        return sum(2.0 * p * c.in_channels * c.out_channels for c in self.cfgs)


@dataclass
class ConvNeXtParams:
    w: torch.Tensor       # [C, 3, 3, 3, C]
    b: torch.Tensor
    norm_g: torch.Tensor
    norm_b: torch.Tensor
    w0: torch.Tensor      # [hidden, C]
    b0: torch.Tensor
    w2: torch.Tensor      # [C, hidden]
    b2: torch.Tensor

    @staticmethod
    def from_numpy(p: dict, device, dtype=torch.bfloat16) -> "ConvNeXtParams":
        f32 = torch.float32
        return ConvNeXtParams(_dev(p["w"], device, dtype), _dev(p["b"], device, f32), _dev(p["norm_g"], device, f32),
                              _dev(p["norm_b"], device, f32), _dev(p["w0"], device, dtype),
                              _dev(p["b0"], device, f32), _dev(p["w2"], device, dtype), _dev(p["b2"], device, f32))


class ConvNeXtStack:
    """ConvNeXt decoder blocks of one stage (convnext_blocks_forward_wgpu_tensor,
    sparse_decoder_wgpu_ops.rs:1090-1161): the neighbor map is built once per
    stage and shared by the blocks."""

    def __init__(self, blocks: list[ConvNeXtParams]):
        self.blocks = blocks
        c = blocks[0].w.shape[0]
        self.channels = c
        self.hidden = blocks[0].w0.shape[0]
        self.cfg = F.SparseSubmConvConfig.subm3(c, c)

    def launches(self) -> int:
        return 3 * len(self.blocks)

    def forward(self, x: torch.Tensor, nbr: torch.Tensor, schedule=None, bufs: dict | None = None) -> torch.Tensor:
        n, c = x.shape
        if c != self.channels:
            raise F.SparseConvError(F._lib.SC_ERR_INVALID, f"decoder wgpu convnext tensor dims mismatch: got=[{n},{c}] "
                                        f"expected=[{n},{self.channels}]")
        bufs = {} if bufs is None else bufs

        def buf(name, cols):
            t = bufs.get(name)
            if t is None or t.shape != (n, cols) or t.dtype != x.dtype:
                t = torch.empty((n, cols), dtype=x.dtype, device=x.device)
                bufs[name] = t
            return t

        cur = x
        for i, p in enumerate(self.blocks):
            h = F.sparse_subm_conv_forward(
                self.cfg, cur, nbr, p.w, p.b,
                F.Epilogue(layer_norm=True, ln_eps=CONVNEXT_LN_EPS, ln_gamma=p.norm_g, ln_beta=p.norm_b,
                           schedule=schedule),
                out=buf("h", c))
            hid = F.linear_forward(h, p.w0, p.b0, F.Epilogue(silu=True), out=buf("hid", self.hidden))
            nxt = buf(f"x{i % 2}", c)
            cur = F.linear_forward(hid, p.w2, p.b2, F.Epilogue(residual=cur), out=nxt)
        return cur

    def flops(self, nbr: torch.Tensor) -> float:
        """Algorithmic FLOPs: 2*P*C^2 for the conv, 2*N*C*hidden per linear."""
        P = float((nbr >= 0).sum())
        n = nbr.shape[0]
        per = 2.0 * P * self.channels ** 2 + 2 * 2.0 * n * self.channels * self.hidden
        return per * len(self.blocks)

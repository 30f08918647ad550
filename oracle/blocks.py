"""Block-level compositions of the oracle -- TEST INFRASTRUCTURE.

Restates the block orders the BASELINE configs use, on top of the C
primitives in ``oracle/__init__.py``:

* SparseResBlock3d (burn_trellis/src/runtime_model/sparse_structure_decoder.rs:111-126):
  ``x + conv2(SiLU(LN2(conv1(SiLU(LN1(x))))))``, LayerNorm eps 1e-5 (:22).
* C2S upsample block, host order
  (burn_trellis/src/runtime_model/sparse_decoder_runtime_impl.rs:1237-1345):
  ``LN(g,b)->SiLU->SubM(Cin->8*Cout)`` on parents, channel2spatial, then
  ``LN(no affine)->SiLU->SubM(Cout->Cout)`` on children plus the skip
  (parent row as [8, Cin/8], row c, each channel repeated Cout/(Cin/8) times),
  LayerNorm eps 1e-6 (sparse_decoder.rs:43).
* ConvNeXt decoder block (sparse_decoder.rs:602-609; device order
  sparse_decoder_wgpu_ops.rs:1090-1161 with the MLP at :355-489; host order
  sparse_decoder_runtime_impl.rs:689-755): ``h = LN(g,b)(SubM(x))``,
  ``h = SiLU(mlp_0(h))``, ``out = mlp_2(h) + x``; LayerNorm eps 1e-6.

Precision.  ``bf16=True`` mirrors where the CUDA path stores bf16: inputs and
weights are rounded to bf16 (RNE, burn_flex_gmm/src/wgpu.rs:57-67); every
conv accumulates in fp32; the bias / residual / LayerNorm / SiLU epilogue runs
in fp32 on the fp32 accumulator and the result is rounded to bf16 where it is
stored.  In fp32 mode nothing is rounded.
"""
from __future__ import annotations

import numpy as np

from . import (DUP_LOWEST, OracleConfig, bf16_round, build_neighbor_rows, channel2spatial,
               layer_norm, silu, subm_conv_flex)

RESBLOCK_LN_EPS = 1e-5  # sparse_structure_decoder.rs:22
C2S_LN_EPS = 1e-6       # sparse_decoder.rs:43 (LAYER_NORM32_EPS)
CONVNEXT_LN_EPS = 1e-6  # the same LAYER_NORM32_EPS (sparse_decoder_wgpu_ops.rs:1137-1144)


def _q(x, bf16: bool):
    return bf16_round(x) if bf16 else np.asarray(x, np.float32)


def conv(x, nbr, w, b, bf16: bool, threads: int = 8):
    cout, kd, kh, kw, cin = w.shape
    cfg = OracleConfig(cin, cout, kd, kh, kw)
    return subm_conv_flex(cfg, _q(w, bf16), b, _q(x, bf16), nbr, threads=threads)


def linear(x, w, b, bf16: bool, threads: int = 8):
    """Linear layer, weight [out, in] (burn_trellis sparse_decoder.rs:623-631):
    ``linear_forward`` (sparse_decoder_wgpu_ops.rs:1-60) writes the bias into
    every output row, then accumulates input @ weight.T with sgemm (beta=1) --
    the flex conv's order, so it is the flex conv with one tap over the
    identity rows."""
    w = np.asarray(w, np.float32)
    cout, cin = w.shape
    cfg = OracleConfig(cin, cout, 1, 1, 1)
    n = np.asarray(x).shape[0]
    ident = np.arange(n, dtype=np.int32).reshape(n, 1)
    return subm_conv_flex(cfg, _q(w, bf16).reshape(cout, 1, 1, 1, cin), b, _q(x, bf16), ident, threads=threads)


def subdivision_head(x, w, b, threshold: float = 0.0, child_thresholds=None, center: bool = False,
                     bf16: bool = False, threads: int = 8):
    """to_subdiv logits [N, 8] = linear(x) (sparse_decoder_runtime_impl.rs:852-873), optionally
    minus the row mean (:875-877), and the child mask logits > threshold[c] with
    a finite per-child threshold overriding the shared one
    (sparse_decoder_wgpu_ops.rs:986-991, :1813-1822)."""
    logits = linear(x, w, b, bf16, threads).astype(np.float32)
    if center:
        logits = logits - logits.mean(axis=1, keepdims=True)
    ct = [float("nan")] * 8 if child_thresholds is None else list(child_thresholds)
    thr = np.array([c if np.isfinite(c) else threshold for c in ct], np.float32)
    return logits, (logits > thr[None, :]).astype(np.uint8)


def convnext_block(x, nbr, p, bf16: bool, threads: int = 8):
    """One ConvNeXt decoder block; returns the fp32 (unrounded) output."""
    x = _q(x, bf16)
    h = _q(layer_norm(conv(x, nbr, p["w"], p["b"], bf16, threads), p["norm_g"], p["norm_b"], CONVNEXT_LN_EPS),
           bf16)
    h = _q(silu(linear(h, p["w0"], p["b0"], bf16, threads)), bf16)
    return linear(h, p["w2"], p["b2"], bf16, threads) + x


def convnext_stack(x, nbr, blocks, bf16: bool, threads: int = 8):
    """Blocks in order, each output rounded where the CUDA path stores it."""
    y = np.asarray(x, np.float32)
    for p in blocks:
        y = _q(convnext_block(y, nbr, p, bf16, threads), bf16)
    return y


def neighbor_map(coords, kernel=(3, 3, 3)):
    cfg = OracleConfig(1, 1, *kernel)
    return build_neighbor_rows(cfg, coords, DUP_LOWEST)


def resblock(x, nbr, p, bf16: bool, threads: int = 8, pre=None):
    """One SparseResBlock3d.  ``pre`` (optional) is SiLU(LN1(x)) already
    computed by the previous block's fused epilogue (fp32, unrounded)."""
    eps = p.get("eps", RESBLOCK_LN_EPS)
    x = _q(x, bf16)
    h = pre if pre is not None else silu(layer_norm(x, p["ln1_g"], p["ln1_b"], eps))
    h = _q(h, bf16)
    y1 = conv(h, nbr, p["w1"], p["b1"], bf16, threads)
    h1 = _q(silu(layer_norm(y1, p["ln2_g"], p["ln2_b"], eps)), bf16)
    y2 = conv(h1, nbr, p["w2"], p["b2"], bf16, threads) + x
    return y2  # fp32 (unrounded) block output


def resblock_stack(x, nbr, blocks, bf16: bool, threads: int = 8):
    """Chain of SparseResBlock3d as the fused CUDA path runs it: each block's
    conv2 epilogue also emits the next block's SiLU(LN1(.)) from the fp32 sum."""
    pre = None
    y = np.asarray(x, np.float32)
    for i, p in enumerate(blocks):
        y = resblock(y, nbr, p, bf16, threads, pre)
        if i + 1 < len(blocks):
            q = blocks[i + 1]
            pre = silu(layer_norm(y, q["ln1_g"], q["ln1_b"], q.get("eps", RESBLOCK_LN_EPS)))
        y = _q(y, bf16)
    return y


def c2s_block(coords, x, mask, p, bf16: bool, threads: int = 8):
    """C2S upsample block.  Returns (child_coords, child_feats fp32-or-bf16)."""
    coords = np.asarray(coords, np.uint32)
    x = _q(x, bf16)
    cin = x.shape[1]
    w1, w2 = p["w1"], p["w2"]
    cout = w2.shape[0]
    h = _q(silu(layer_norm(x, p["ln1_g"], p["ln1_b"], C2S_LN_EPS)), bf16)
    nbr_p = neighbor_map(coords)
    y1 = conv(h, nbr_p, w1, p["b1"], bf16, threads)                 # [Np, 8*cout] fp32
    child_coords, h_up = channel2spatial(coords, y1, mask)
    h_up = _q(silu(layer_norm(h_up, None, None, C2S_LN_EPS)), bf16)
    _, x_up = channel2spatial(coords, x, mask)                       # [Nc, cin/8]
    skip = np.repeat(x_up, cout // (cin // 8), axis=1)
    nbr_c = neighbor_map(child_coords)
    y2 = conv(h_up, nbr_c, w2, p["b2"], bf16, threads) + skip
    return child_coords, _q(y2, bf16)

"""Oracle restatement of the ConvNeXt decoder block and of the linear layer,
checked against independent numpy arithmetic (CPU only)."""
import numpy as np

import oracle
import oracle.blocks as OB
from bevy_synth_b200 import synth


def _shell():
    return synth.morton_sort(synth.unique_cells(0, synth.sphere_shell(16, (8.0, 8.0, 8.0), 5.0, 1.0)))


def test_linear_matches_numpy():
    rng = np.random.default_rng(1)
    x = rng.standard_normal((57, 48)).astype(np.float32)
    w = rng.standard_normal((40, 48)).astype(np.float32)
    b = rng.standard_normal(40).astype(np.float32)
    got = OB.linear(x, w, b, bf16=False, threads=2)
    ref = x.astype(np.float64) @ w.T.astype(np.float64) + b
    np.testing.assert_allclose(got, ref, rtol=1e-5, atol=1e-4)


def test_convnext_block_matches_independent_composition():
    coords = _shell()
    n = coords.shape[0]
    c, hidden = 16, 64
    rng = np.random.default_rng(2)
    x = rng.standard_normal((n, c)).astype(np.float32)
    p = synth.convnext_params(rng, c, hidden)
    nbr = OB.neighbor_map(coords)
    got = OB.convnext_block(x, nbr, p, bf16=False, threads=2)
    # independent: the reference's legacy per-pair conv (lib.rs:428-510) + numpy LN / SiLU / matmuls
    cfg = oracle.OracleConfig(c, c, 3, 3, 3)
    h = oracle.subm_conv_legacy(cfg, p["w"], p["b"], coords.astype(np.uint32), x).astype(np.float64)
    mu = h.mean(1, keepdims=True)
    var = ((h - mu) ** 2).mean(1, keepdims=True)
    h = (h - mu) / np.sqrt(var + 1e-6) * p["norm_g"] + p["norm_b"]
    h = h @ p["w0"].T.astype(np.float64) + p["b0"]
    h = h / (1.0 + np.exp(-h))
    ref = h @ p["w2"].T.astype(np.float64) + p["b2"] + x
    np.testing.assert_allclose(got, ref, rtol=1e-4, atol=2e-4)

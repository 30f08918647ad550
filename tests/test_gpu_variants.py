"""Tuning variants of the tensor-core conv kernel give the default path's results.

The launcher reads some tuning switches (SC_TC_*) once per process, so each
variant runs in a child process on the same seeded inputs and writes its
outputs to a file; the parent compares them with the default variant's.  The
variants change scheduling and copy engines only (4 or 8 gather warps, TMA
row gathers, CTA pairs on or off, a persistent static schedule, 256-wide
column tiles), never the order of the fp32 accumulation, so the comparison bound is tight.
"""
import os
import subprocess
import sys

import numpy as np
import pytest

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))

_CHILD = r"""
import sys, numpy as np, torch
sys.path.insert(0, sys.argv[1])
from bevy_synth_b200 import flex_gmm as F
from bevy_synth_b200 import synth
dev = torch.device("cuda:0")
coords = torch.as_tensor(synth.config1(0).coords, device=dev)
out = {}
rng = np.random.default_rng(5)
for cin, cout, sched in ((64, 64, True), (128, 256, True), (64, 96, False), (128, 384, True)):
    cfg = F.SparseSubmConvConfig.subm3(cin, cout)
    nbr = F.neighbor_rows_tensor_from_coords_tensor(cfg, coords)
    n = coords.shape[0]
    x = torch.as_tensor(rng.standard_normal((n, cin)).astype(np.float32), device=dev).to(torch.bfloat16)
    w = torch.as_tensor((0.05 * rng.standard_normal((cout, 3, 3, 3, cin))).astype(np.float32), device=dev)
    b = torch.as_tensor(rng.standard_normal(cout).astype(np.float32), device=dev)
    epi = F.Epilogue(schedule=F.neighbor_schedule(cfg, nbr)) if sched else None
    y = F.sparse_subm_conv_forward(cfg, x, nbr, w.to(torch.bfloat16), b, epi)
    out[f"{cin}_{cout}"] = y.float().cpu().numpy()
np.savez(sys.argv[2], **out)
"""

VARIANTS = {
    "default": {},
    "four_gather_warps": {"SC_TC_PW": "4"},
    "tma_gather4": {"SC_TC_GATHER4": "1"},
    "half_tma_gather4": {"SC_TC_GATHER4": "2"},
    "cta_pair": {"SC_TC_PAIR": "1"},
    "no_cta_pair": {"SC_TC_PAIR": "0"},
    "cta_pair_eight_gather_warps": {"SC_TC_PAIR": "1", "SC_TC_PW": "8"},
    "static_schedule": {"SC_TC_STATIC": "1"},
    "narrow_column_tiles": {"SC_TC_WIDE": "0"},
}


def _run(tmp_path, name, env_extra):
    env = dict(os.environ)
    for k in ("SC_TC_PW", "SC_TC_GATHER4", "SC_TC_PAIR", "SC_TC_STATIC", "SC_TC_WIDE"):
        env.pop(k, None)
    env.update(env_extra)
    path = str(tmp_path / f"{name}.npz")
    subprocess.run([sys.executable, "-c", _CHILD, ROOT, path], env=env, check=True, timeout=300)
    return dict(np.load(path))


@pytest.mark.gpu
@pytest.mark.timeout(900)
def test_kernel_variants_match_default(tmp_path, cuda_device):
    ref = _run(tmp_path, "default", VARIANTS["default"])
    for name, env in VARIANTS.items():
        if name == "default":
            continue
        got = _run(tmp_path, name, env)
        for key, r in ref.items():
            g = got[key]
            err = float(np.linalg.norm(g - r) / max(np.linalg.norm(r), 1e-30))
            assert err <= 1e-6, f"variant {name} conv {key}: rel L2 {err:.3e} vs the default kernel"

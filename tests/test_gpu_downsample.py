"""Stride-2 sparse downsample conv (SparseConv3d, kernel 2, stride 2) against
its definition restated in oracle/downsample.py (the reference has no
downsample conv): output coordinates bit-exact, fp32 rel-L2 <= 1e-4 on the
CUDA-core kernel, bf16 rel-L2 <= 1e-2 on the tensor-core kernel."""
import numpy as np
import pytest
import torch

import oracle
from oracle import downsample as OD
from bevy_synth_b200 import synth
from bevy_synth_b200 import flex_gmm as F

from gpu_util import assert_no_fault, rel_l2, to_dev

pytestmark = pytest.mark.gpu


def grid(seed, n_batches=2):
    rng = np.random.default_rng(seed)
    parts = []
    for b in range(n_batches):
        occ = rng.random((14, 14, 14)) < 0.25
        parts.append(synth.morton_sort(synth.unique_cells(b, np.argwhere(occ))))
    return np.concatenate(parts)


@pytest.mark.parametrize("cin,cout,dtype,tol", [(16, 24, torch.float32, 1e-4), (64, 64, torch.bfloat16, 1e-2),
                                                (128, 256, torch.bfloat16, 1e-2)])
def test_stride2_downsample(cuda_device, cin, cout, dtype, tol):
    coords = grid(cin + cout)
    rng = np.random.default_rng(cout)
    x = rng.standard_normal((coords.shape[0], cin)).astype(np.float32)
    w = (0.1 * rng.standard_normal((cout, 2, 2, 2, cin))).astype(np.float32)
    b = rng.standard_normal(cout).astype(np.float32)
    oc, y = F.sparse_conv3d_stride2_forward(to_dev(x, dtype), to_dev(coords), to_dev(w, dtype), to_dev(b))
    roc = OD.downsample_coords(coords)
    np.testing.assert_array_equal(oc.cpu().numpy(), roc)
    if dtype == torch.bfloat16:
        x, w = oracle.bf16_round(x), oracle.bf16_round(w)
    _, ref = OD.conv3d_stride2(coords, x, w, b)
    if dtype == torch.bfloat16:
        ref = oracle.bf16_round(ref)
    assert rel_l2(y.float().cpu().numpy(), ref) <= tol
    if dtype == torch.bfloat16 and cin >= 64:
        assert F.uses_tensor_cores(F.SparseSubmConvConfig(cin, cout, 2, 2, 2), dtype)
    assert_no_fault()


def test_stride2_downsample_empty(cuda_device):
    oc, y = F.sparse_conv3d_stride2_forward(torch.zeros((0, 8), device="cuda"),
                                            torch.zeros((0, 4), dtype=torch.int32, device="cuda"),
                                            torch.zeros((8, 2, 2, 2, 8), device="cuda"))
    assert oc.shape == (0, 4) and y.shape == (0, 8)

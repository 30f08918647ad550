"""Sparse tensor / batch layout types (burn_trellis runtime_model/types/
sparse_tensor_device.rs:6-32, sparse_batch_layout_device.rs:4-26,
varlen_tensor_device.rs:6-28): per-batch offsets and lengths from batch-grouped
coordinates, per-batch slices, assembly from per-batch parts (CPU), and a SubM
conv of a multi-batch sparse tensor equal to the conv of each batch alone (GPU)."""
import numpy as np
import pytest
import torch

from bevy_synth_b200 import synth
from bevy_synth_b200 import flex_gmm as F
from bevy_synth_b200.sparse_tensor import SparseBatchLayout, SparseTensor, sparse_subm_conv3d


def test_layout_from_coords():
    c = torch.tensor([[3, 0, 0, 0], [3, 1, 0, 0], [5, 0, 0, 0], [5, 0, 1, 0], [5, 2, 2, 2], [9, 7, 7, 7]],
                     dtype=torch.int32)
    lay = SparseBatchLayout.from_coords(c)
    assert lay.batch_size() == 3 and lay.rows == 6
    assert lay.offsets.tolist() == [0, 2, 5] and lay.lengths.tolist() == [2, 3, 1]
    assert lay.batch_ids.tolist() == [3, 5, 9]
    parts = lay.split(torch.arange(6))
    assert [p.tolist() for p in parts] == [[0, 1], [2, 3, 4], [5]]


def test_layout_empty_and_errors():
    lay = SparseBatchLayout.from_coords(torch.zeros((0, 4), dtype=torch.int32))
    assert lay.batch_size() == 0 and lay.rows == 0
    with pytest.raises(F.SparseConvError, match="grouped by ascending batch"):
        SparseBatchLayout.from_coords(torch.tensor([[1, 0, 0, 0], [0, 0, 0, 0]], dtype=torch.int32))
    with pytest.raises(F.SparseConvError, match="shape \\[N, 4\\]"):
        SparseBatchLayout.from_coords(torch.zeros((3, 3), dtype=torch.int32))


def test_from_batches_and_batch_slices():
    a = torch.tensor([[1, 2, 3], [4, 5, 6]], dtype=torch.int32)
    b = torch.tensor([[0, 0, 0]], dtype=torch.int32)
    fa, fb = torch.ones((2, 4)), torch.zeros((1, 4))
    st = SparseTensor.from_batches([(a, fa), (b, fb)], 64, batch_ids=[8, 9])
    assert st.rows() == 3 and st.values.channels == 4 and st.sparse_resolution == 64
    assert st.coords[:, 0].tolist() == [8, 8, 9]
    assert st.layout.batch_ids.tolist() == [8, 9]
    one = st.batch(1)
    assert one.rows() == 1 and one.coords.tolist() == [[9, 0, 0, 0]]
    with pytest.raises(F.SparseConvError, match="rows"):
        st.with_values(torch.zeros((2, 4)))


@pytest.mark.gpu
def test_batched_conv_equals_per_batch_conv(cuda_device):
    """Config-4 structure (assets in coord[0]): one conv over the batch equals each asset's
    conv alone, bit for bit; the grid's map is built once and reused."""
    wl = synth.config4(1, assets=3, layers=1, channels=128)
    dev = torch.device("cuda:0")
    st = SparseTensor.new(torch.as_tensor(wl.coords, device=dev),
                          torch.as_tensor(wl.feats, device=dev).to(torch.bfloat16), 64)
    assert st.layout.batch_size() == 3
    cfg = F.SparseSubmConvConfig.subm3(128, 128)
    w = torch.as_tensor(wl.params["w"][0], device=dev).to(torch.bfloat16)
    b = torch.as_tensor(np.zeros(128, np.float32), device=dev)
    y = sparse_subm_conv3d(st, cfg, w, b, F.Epilogue(silu=True))
    y2 = sparse_subm_conv3d(y, cfg, w, b)
    assert len(st._maps) == 1 and y2._maps is st._maps
    for i in range(3):
        yi = sparse_subm_conv3d(st.batch(i), cfg, w, b, F.Epilogue(silu=True))
        assert torch.equal(yi.feats, y.feats[st.layout.rows_of(i)])

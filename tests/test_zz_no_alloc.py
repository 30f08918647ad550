"""The no-allocation neighbor map (sc_neighbor_map_noalloc) through the C ABI.

It exists for callers that cannot allocate device memory -- they hold only
the buffers they pass in, or must not call cudaMalloc on their execution path
-- and keeps its hash table in a fixed static device array.  Its output must
equal the allocating entry point's exactly (neighbor maps are bit-exact), on
two calls in a row, so the shared table is shown to be cleared between calls.
This file is collected last on purpose."""
import ctypes

import numpy as np
import pytest
import torch

from bevy_synth_b200 import _lib, synth
from bevy_synth_b200 import flex_gmm as F

pytestmark = pytest.mark.gpu

MAX_ROWS = 262_144


def noalloc_map(cfg, coords_t):
    out = torch.empty((coords_t.shape[0], F.kernel_rows(cfg)), dtype=torch.int32, device=coords_t.device)
    c = cfg.c()
    rc = _lib.lib().sc_neighbor_map_noalloc(ctypes.byref(c), ctypes.c_void_p(coords_t.data_ptr()),
                                            coords_t.shape[0], ctypes.c_void_p(out.data_ptr()),
                                            ctypes.c_void_p(torch.cuda.current_stream().cuda_stream))
    _lib.check(rc)
    return out


def test_noalloc_map_matches_allocating_map_twice(cuda_device):
    cfg = F.SparseSubmConvConfig.subm3(4, 4)
    first = torch.as_tensor(synth.config2(0, blocks=1, channels=8).coords, device=cuda_device)
    # a different, smaller set second: stale entries of the first call must not leak
    second = torch.as_tensor(synth.config1(0).coords, device=cuda_device)
    for coords in (first, second):
        got = noalloc_map(cfg, coords)
        exp = F.neighbor_rows_tensor_from_coords_tensor(cfg, coords)
        torch.cuda.synchronize()
        assert torch.equal(got, exp)
    assert _lib.device_fault() == 0


def test_noalloc_map_rejects_more_rows_than_the_static_table(cuda_device):
    cfg = F.SparseSubmConvConfig.subm3(4, 4)
    c = cfg.c()
    rc = _lib.lib().sc_neighbor_map_noalloc(ctypes.byref(c), None, MAX_ROWS + 1, None, None)
    assert rc == _lib.SC_ERR_CAPACITY
    assert "static table limit" in _lib.last_error()

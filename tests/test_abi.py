"""CPU checks of the C ABI: the library loads, exports every symbol that
include/sparseconv.h declares, and its host-only entry points validate
arguments the way the reference does (no GPU needed)."""
import ctypes
import os
import re

import numpy as np
import pytest

import oracle
from bevy_synth_b200 import _lib
from bevy_synth_b200 import flex_gmm as F

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))


def declared_symbols():
    src = open(os.path.join(ROOT, "include", "sparseconv.h")).read()
    src = re.sub(r"/\*.*?\*/", "", src, flags=re.S)
    return sorted(set(re.findall(r"\b(sc_[a-z0-9_]+)\s*\(", src)))


def test_library_exports_every_declared_symbol():
    L = _lib.lib()
    names = declared_symbols()
    assert len(names) >= 16
    for n in names:
        assert hasattr(L, n), f"missing export {n}"
    assert set(names) == set(_lib.EXPORTED)


def test_version():
    assert _lib.lib().sc_version() >= 1


@pytest.mark.parametrize("kernel", [(3, 3, 3), (3, 1, 1), (3, 3, 1), (9, 9, 9), (5, 3, 1)])
@pytest.mark.parametrize("axis_order,axis_sign", [((0, 1, 2), (1, 1, 1)), ((2, 1, 0), (-1, 1, 1)),
                                                  ((1, 2, 0), (1, -1, -1))])
def test_kernel_offsets_match_oracle(kernel, axis_order, axis_sign):
    cfg = F.SparseSubmConvConfig(4, 4, *kernel, axis_order=axis_order, axis_sign=axis_sign)
    ocfg = oracle.OracleConfig(4, 4, *kernel, axis_order=axis_order, axis_sign=axis_sign)
    assert F.kernel_rows(cfg) == ocfg.kernel_rows
    np.testing.assert_array_equal(F.kernel_offsets(cfg).numpy(), oracle.kernel_offsets(ocfg))


@pytest.mark.parametrize("bad,msg", [
    (dict(in_channels=0), "channel dimensions must be non-zero"),
    (dict(kernel_d=0), "kernel dimensions must be non-zero"),
    (dict(groups=0, in_channels_per_group=4, out_channels_per_group=4), "groups must be non-zero"),
    (dict(in_channels_per_group=3), "in_channels/group mismatch"),
    (dict(out_channels_per_group=3), "out_channels/group mismatch"),
    (dict(axis_order=(0, 0, 1)), "axis_order must be a permutation"),
])
def test_config_validation_messages(bad, msg):
    base = dict(in_channels=4, out_channels=4)
    base.update(bad)
    cfg = F.SparseSubmConvConfig(**base)
    with pytest.raises(_lib.SparseConvError, match=msg) as ei:
        F.kernel_rows(cfg)
    assert ei.value.code == _lib.SC_ERR_INVALID


def test_conv_rejects_more_queries_than_inputs_without_gpu():
    # reference: sparse_conv.rs:439-444 ("neighbor row count exceeds input rows")
    cfg = F.SparseSubmConvConfig(4, 4).c()
    rc = _lib.lib().sc_subm_conv_forward(ctypes.byref(cfg), _lib.DTYPE_F32, None, 1, None, 2, None, None,
                                         None, None, None)
    assert rc == _lib.SC_ERR_INVALID
    assert "exceeds input rows" in _lib.last_error()


def test_empty_conv_is_a_no_op_without_gpu():
    cfg = F.SparseSubmConvConfig(4, 4).c()
    assert _lib.lib().sc_subm_conv_forward(ctypes.byref(cfg), _lib.DTYPE_F32, None, 0, None, 0, None, None,
                                           None, None, None) == 0


def test_neighbor_workspace_too_small_is_capacity_error():
    cfg = F.SparseSubmConvConfig(4, 4).c()
    rc = _lib.lib().sc_neighbor_map(ctypes.byref(cfg), None, 100, None, 0, None, None)
    assert rc == _lib.SC_ERR_CAPACITY
    assert "workspace too small" in _lib.last_error()


def test_workspace_size_grows_with_rows():
    b = [ctypes.c_size_t(0) for _ in range(3)]
    for n, v in zip((0, 10_000, 1_000_000), b):
        assert _lib.lib().sc_neighbor_workspace_bytes(n, ctypes.byref(v)) == 0
    assert b[0].value < b[1].value < b[2].value
    assert b[2].value >= 2 * 1_000_000 * 16

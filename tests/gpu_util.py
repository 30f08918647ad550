"""Helpers shared by the GPU parity tests."""
import numpy as np
import torch

import oracle
from bevy_synth_b200 import _lib
from bevy_synth_b200 import flex_gmm as F


def dev():
    return torch.device("cuda:0")


def to_dev(a, dtype=None):
    t = torch.as_tensor(np.ascontiguousarray(a), device=dev())
    return t.to(dtype) if dtype is not None else t


def gpu_map(cfg: F.SparseSubmConvConfig, coords, query=None) -> np.ndarray:
    c = to_dev(np.asarray(coords, np.int32))
    if query is None:
        out = F.neighbor_rows_tensor_from_coords_tensor(cfg, c)
    else:
        out = F.neighbor_rows_query_tensor(cfg, c, to_dev(np.asarray(query, np.int32)))
    return out.cpu().numpy()


def ocfg(cfg: F.SparseSubmConvConfig) -> oracle.OracleConfig:
    return oracle.OracleConfig(cfg.in_channels, cfg.out_channels, cfg.kernel_d, cfg.kernel_h, cfg.kernel_w,
                               groups=cfg.groups, axis_order=cfg.axis_order, axis_sign=cfg.axis_sign)


def rel_l2(a, b) -> float:
    a = np.asarray(a, np.float64)
    b = np.asarray(b, np.float64)
    return float(np.linalg.norm(a - b) / max(np.linalg.norm(b), 1e-30))


def assert_no_fault():
    torch.cuda.synchronize()
    f = _lib.device_fault()
    assert f == 0, f"device fault word = {f:#x}"

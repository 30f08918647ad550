"""CPU oracle for the sparse submanifold convolution path -- TEST INFRASTRUCTURE.

This package restates, on the CPU, the reference's (mosure/bevy_synth)
sparse-conv path: ``burn_flex_gmm``'s flex gather+SGEMM conv, its legacy loop,
the neighbor-map builder, the weight packer, and the decoder-block math of
``burn_trellis`` (LayerNorm, SiLU, channel-to-space, repeat-interleave, the
SparseResBlock3d and C2S upsample block orders).

Only ``tests/``, ``__graft_entry__.smoke()`` and ``bench.py``'s CPU-baseline
leg may import it, and only as the checker / the timed CPU baseline.  The
product library never routes through it.

Parity status: the reference is Rust and cannot be compiled here (no cargo),
so no reference-produced output exists.  The restatement is pinned to the
reference's own known-answer tests and LCG-driven property tests; see
``tests/test_oracle.py``.
"""
from __future__ import annotations

import ctypes
import os
import subprocess
from dataclasses import dataclass, field

import numpy as np

_HERE = os.path.dirname(os.path.abspath(__file__))
_LIB_PATH = os.path.join(_HERE, "liboracle.so")
_lib = None

DUP_LAST = 0    # CPU HashMap::insert semantics (burn_flex_gmm/src/lib.rs:83-86)
DUP_LOWEST = 1  # device builders (burn_flex_gmm/src/wgpu/neighbor_kernels.rs:249-256)


class _Cfg(ctypes.Structure):
    _fields_ = [
        ("in_channels", ctypes.c_int64), ("out_channels", ctypes.c_int64),
        ("kernel_d", ctypes.c_int64), ("kernel_h", ctypes.c_int64), ("kernel_w", ctypes.c_int64),
        ("in_channels_per_group", ctypes.c_int64), ("out_channels_per_group", ctypes.c_int64),
        ("groups", ctypes.c_int64),
        ("axis_order", ctypes.c_int32 * 3), ("axis_sign", ctypes.c_int32 * 3),
    ]


def build() -> str:
    """Compile liboracle.so with the committed Makefile."""
    subprocess.run(["make", "-s", "-C", _HERE], check=True)
    return _LIB_PATH


def lib():
    global _lib
    if _lib is None:
        if not os.path.exists(_LIB_PATH):
            build()
        _lib = ctypes.CDLL(_LIB_PATH)
        _lib.oc_last_error.restype = ctypes.c_char_p
    return _lib


def _check(rc: int) -> None:
    if rc != 0:
        raise ValueError(lib().oc_last_error().decode())


def _p(a: np.ndarray):
    return a.ctypes.data_as(ctypes.c_void_p) if a is not None else None


@dataclass(frozen=True)
class OracleConfig:
    """Mirror of ``SparseSubmConvConfig`` (burn_flex_gmm/src/lib.rs:5-17)."""

    in_channels: int
    out_channels: int
    kernel_d: int = 3
    kernel_h: int = 3
    kernel_w: int = 3
    in_channels_per_group: int | None = None
    out_channels_per_group: int | None = None
    groups: int = 1
    axis_order: tuple = (0, 1, 2)
    axis_sign: tuple = (1, 1, 1)

    def c(self) -> _Cfg:
        cig = self.in_channels_per_group or self.in_channels // self.groups
        cog = self.out_channels_per_group or self.out_channels // self.groups
        return _Cfg(self.in_channels, self.out_channels, self.kernel_d, self.kernel_h,
                    self.kernel_w, cig, cog, self.groups,
                    (ctypes.c_int32 * 3)(*self.axis_order), (ctypes.c_int32 * 3)(*self.axis_sign))

    @property
    def kernel_rows(self) -> int:
        return self.kernel_d * self.kernel_h * self.kernel_w


def kernel_offsets(cfg: OracleConfig) -> np.ndarray:
    out = np.zeros((cfg.kernel_rows, 3), np.int32)
    c = cfg.c()
    _check(lib().oc_kernel_offsets(ctypes.byref(c), _p(out)))
    return out


def build_neighbor_rows(cfg: OracleConfig, coords, dup_rule: int = DUP_LOWEST,
                        query=None) -> np.ndarray:
    """lib.rs:69-109.  ``query`` (optional) queries other coordinates against
    the table built from ``coords``."""
    coords = np.ascontiguousarray(coords, dtype=np.uint32).reshape(-1, 4)
    q = coords if query is None else np.ascontiguousarray(query, dtype=np.uint32).reshape(-1, 4)
    out = np.empty((q.shape[0], cfg.kernel_rows), np.int32)
    c = cfg.c()
    _check(lib().oc_build_neighbor_rows_query(ctypes.byref(c), _p(coords), ctypes.c_int64(coords.shape[0]),
                                              _p(q), ctypes.c_int64(q.shape[0]), dup_rule, _p(out)))
    return out


def pack_flex_weight(cfg: OracleConfig, weight) -> np.ndarray:
    w = np.ascontiguousarray(weight, dtype=np.float32).reshape(-1)
    cig = cfg.in_channels // cfg.groups
    out = np.empty(cfg.groups * cfg.kernel_rows * cig * (cfg.out_channels // cfg.groups), np.float32)
    c = cfg.c()
    _check(lib().oc_pack_flex_weight(ctypes.byref(c), _p(w), _p(out)))
    return out


def subm_conv_flex(cfg: OracleConfig, weight, bias, inp, neighbor_rows, packed=None,
                   threads: int = 1) -> np.ndarray:
    """lib.rs:242-375 (sparse_subm_conv_forward_flex_precomputed)."""
    w = np.ascontiguousarray(weight, dtype=np.float32).reshape(-1)
    b = np.ascontiguousarray(bias, dtype=np.float32).reshape(-1)
    x = np.ascontiguousarray(inp, dtype=np.float32).reshape(-1, cfg.in_channels)
    nbr = np.ascontiguousarray(neighbor_rows, dtype=np.int32).reshape(-1, cfg.kernel_rows)
    out = np.empty((nbr.shape[0], cfg.out_channels), np.float32)
    pk = None if packed is None else np.ascontiguousarray(packed, dtype=np.float32)
    c = cfg.c()
    _check(lib().oc_subm_conv_flex_precomputed(
        ctypes.byref(c), _p(w), _p(b), _p(x), ctypes.c_int64(x.shape[0]), _p(nbr),
        ctypes.c_int64(nbr.shape[0]), _p(pk), ctypes.c_int(threads), _p(out)))
    return out


def subm_conv_forward_flex(cfg: OracleConfig, weight, bias, coords, inp) -> np.ndarray:
    """lib.rs:111-131: build the map with the CPU (last-wins) rule, then conv."""
    nbr = build_neighbor_rows(cfg, coords, DUP_LAST)
    return subm_conv_flex(cfg, weight, bias, inp, nbr)


def subm_conv_legacy(cfg: OracleConfig, weight, bias, coords, inp) -> np.ndarray:
    """lib.rs:428-510."""
    w = np.ascontiguousarray(weight, dtype=np.float32).reshape(-1)
    b = np.ascontiguousarray(bias, dtype=np.float32).reshape(-1)
    co = np.ascontiguousarray(coords, dtype=np.uint32).reshape(-1, 4)
    x = np.ascontiguousarray(inp, dtype=np.float32).reshape(-1)
    out = np.empty((co.shape[0], cfg.out_channels), np.float32)
    c = cfg.c()
    _check(lib().oc_subm_conv_legacy(ctypes.byref(c), _p(w), _p(b), _p(co),
                                     ctypes.c_int64(co.shape[0]), _p(x), _p(out)))
    return out


def layer_norm(x, gamma=None, beta=None, eps: float = 1e-5) -> np.ndarray:
    """sparse_decoder_wgpu_ops.rs:1642-1711 (returns a new array)."""
    y = np.array(x, dtype=np.float32, copy=True, order="C")
    rows, ch = y.shape
    g = None if gamma is None else np.ascontiguousarray(gamma, dtype=np.float32)
    b = None if beta is None else np.ascontiguousarray(beta, dtype=np.float32)
    _check(lib().oc_layer_norm_inplace(_p(y), ctypes.c_int64(rows), ctypes.c_int64(ch), _p(g), _p(b),
                                       ctypes.c_float(eps)))
    return y


def silu(x) -> np.ndarray:
    """sparse_decoder_wgpu_ops.rs:1713-1720."""
    y = np.array(x, dtype=np.float32, copy=True, order="C")
    lib().oc_silu_inplace(_p(y), ctypes.c_int64(y.size))
    return y


def bf16_round(x) -> np.ndarray:
    """burn_flex_gmm/src/wgpu.rs:57-67 (RNE to bf16, kept in f32)."""
    y = np.array(x, dtype=np.float32, copy=True, order="C")
    lib().oc_bf16_round_inplace(_p(y), ctypes.c_int64(y.size))
    return y


def channel2spatial(coords, feats, mask):
    """sparse_decoder_wgpu_ops.rs:1999-2054 -> (child_coords, child_feats)."""
    co = np.ascontiguousarray(coords, dtype=np.uint32).reshape(-1, 4)
    f = np.ascontiguousarray(feats, dtype=np.float32)
    m = np.ascontiguousarray(mask, dtype=np.uint8).reshape(-1, 8)
    rows, cin = f.shape
    n_out = int(m.sum())
    oc = np.empty((n_out, 4), np.uint32)
    of = np.empty((n_out, cin // 8), np.float32)
    n = ctypes.c_int64(0)
    _check(lib().oc_channel2spatial(_p(co), ctypes.c_int64(rows), _p(f), ctypes.c_int64(cin), _p(m),
                                    _p(oc), _p(of), ctypes.byref(n)))
    assert n.value == n_out
    return oc, of


def repeat_interleave_channels(feats, repeat: int) -> np.ndarray:
    """sparse_decoder_wgpu_ops.rs:2056-2076."""
    return np.repeat(np.asarray(feats, np.float32), repeat, axis=1)


@dataclass
class Lcg:
    """The reference test generator (burn_flex_gmm/src/lib.rs:764-778;
    identical copy at burn_trellis/.../sparse_decoder_tests.rs:171-187)."""

    seed: int
    state: int = field(init=False)

    def __post_init__(self):
        self.state = (self.seed | 1) & 0xFFFFFFFFFFFFFFFF

    def next_f32(self) -> float:
        self.state = (self.state * 6364136223846793005 + 1) & 0xFFFFFFFFFFFFFFFF
        bits = ((self.state >> 40) & 0xFFFFFFFF) | 1
        # (bits as f32 / u32::MAX as f32) * 2.0 - 1.0, evaluated in f32
        v = np.float32(np.float32(bits) / np.float32(4294967295.0))
        return float(np.float32(v * np.float32(2.0)) - np.float32(1.0))

    def take(self, n: int) -> np.ndarray:
        return np.array([self.next_f32() for _ in range(n)], dtype=np.float32)

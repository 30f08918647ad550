"""Host-side mirror of the reference's sparse-conv operator API
(mosure/bevy_synth, crate ``burn_flex_gmm``), backed by libsparseconv.so.

Names, argument meaning and error behaviour follow the reference so that a
caller of ``burn_flex_gmm`` finds the same operations:

=============================================  ===============================================
this module                                    reference (crates/burn_flex_gmm/...)
=============================================  ===============================================
``SparseSubmConvConfig``                       ``SparseSubmConvConfig`` (src/lib.rs:5-17)
``kernel_rows`` / ``kernel_offsets``           ``kernel_rows`` / ``kernel_layout`` (lib.rs:59-67, 727-752)
``neighbor_rows_tensor_from_coords_tensor``    same name (src/wgpu/neighbor.rs:977-1006)
``neighbor_rows_query_tensor``                 chunked query (burn_trellis sparse_decoder_tests.rs:238-292)
``sparse_subm_conv_forward_cubecl``            same name (src/wgpu/sparse_conv.rs:293-308)
``sparse_subm_conv_forward``                   the above + the fused epilogue (``Epilogue``)
``layer_norm_affine_forward``                  ``layer_norm_affine_forward_wgpu`` (src/wgpu/ops.rs:1464-1550)
``layer_norm_affine_silu_forward``             ``layer_norm_affine_silu_forward_wgpu`` (ops.rs:1552-1639)
``bf16_round_to_f32``                          ``bf16_round_to_f32_wgpu`` (src/wgpu.rs:69-102)
=============================================  ===============================================

Tensors are torch CUDA tensors (PyTorch is only the device-memory and stream
plumbing); every computation runs in libsparseconv.  Errors are raised as
``SparseConvError`` with the reference's messages where it has one.
"""
from __future__ import annotations

import ctypes
import functools
from dataclasses import dataclass, field

import torch

from . import _lib
from ._lib import DTYPE_BF16, DTYPE_F32, ScConvConfig, ScEpilogue, ScPatchify3dConfig, SparseConvError, check, lib

INVALID_NEIGHBOR_ROW = -1


@dataclass(frozen=True)
class SparseSubmConvConfig:
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

    def __post_init__(self):
        object.__setattr__(self, "axis_order", tuple(self.axis_order))
        object.__setattr__(self, "axis_sign", tuple(self.axis_sign))
        if self.in_channels_per_group is None:
            object.__setattr__(self, "in_channels_per_group", self.in_channels // max(self.groups, 1))
        if self.out_channels_per_group is None:
            object.__setattr__(self, "out_channels_per_group", self.out_channels // max(self.groups, 1))

    def c(self) -> ScConvConfig:
        """The C struct (built once per distinct config; callers pass it by reference only)."""
        return _config_struct(self)

    @staticmethod
    def subm3(in_channels: int, out_channels: int) -> "SparseSubmConvConfig":
        """The decoder's 3x3x3, groups=1, identity-axis layer
        (burn_trellis sparse_decoder_wgpu_ops.rs:1634-1640)."""
        return SparseSubmConvConfig(in_channels, out_channels)


@functools.lru_cache(maxsize=512)
def _config_struct(config: SparseSubmConvConfig) -> ScConvConfig:
    return ScConvConfig(config.in_channels, config.out_channels, config.kernel_d, config.kernel_h, config.kernel_w,
                        config.in_channels_per_group, config.out_channels_per_group, config.groups,
                        (ctypes.c_int32 * 3)(*config.axis_order), (ctypes.c_int32 * 3)(*config.axis_sign))


@functools.lru_cache(maxsize=512)
def _kernel_rows_cached(config: SparseSubmConvConfig) -> int:
    v = ctypes.c_int64(0)
    check(lib().sc_kernel_rows(ctypes.byref(config.c()), ctypes.byref(v)))
    return v.value


def kernel_rows(config: SparseSubmConvConfig) -> int:
    return _kernel_rows_cached(config)


def kernel_offsets(config: SparseSubmConvConfig) -> torch.Tensor:
    K = kernel_rows(config)
    out = torch.zeros((K, 3), dtype=torch.int32)
    c = config.c()
    check(lib().sc_kernel_offsets(ctypes.byref(c), ctypes.c_void_p(out.data_ptr())))
    return out


def _stream(t: torch.Tensor):
    return ctypes.c_void_p(torch.cuda.current_stream(t.device).cuda_stream)


def _ptr(t):
    return ctypes.c_void_p(t.data_ptr()) if t is not None else None


def _require_cuda(name: str, t: torch.Tensor):
    if not isinstance(t, torch.Tensor) or not t.is_cuda:
        raise SparseConvError(_lib.SC_ERR_INVALID, f"sparse conv {name} must be a CUDA tensor")
    if not t.is_contiguous():
        raise SparseConvError(_lib.SC_ERR_INVALID, f"sparse conv {name} must be contiguous")


def _coords_tensor(coords_t: torch.Tensor) -> torch.Tensor:
    _require_cuda("coords", coords_t)
    if coords_t.dim() != 2 or coords_t.shape[1] != 4:
        raise SparseConvError(_lib.SC_ERR_INVALID,
                              f"sparse conv coords must have shape [N, 4], got {list(coords_t.shape)}")
    if coords_t.dtype != torch.int32:
        raise SparseConvError(_lib.SC_ERR_INVALID,
                              f"sparse conv coords dtype must be I32, got {coords_t.dtype}")
    return coords_t


class NeighborWorkspace:
    """Caller-owned device workspace for the coordinate hash table."""

    def __init__(self, device, n_in: int):
        b = ctypes.c_size_t(0)
        check(lib().sc_neighbor_workspace_bytes(n_in, ctypes.byref(b)))
        self.bytes = b.value
        self.buf = torch.empty(self.bytes, dtype=torch.uint8, device=device)

    def status(self, device) -> int:
        probe = ctypes.c_int32(0)
        check(lib().sc_neighbor_status(_ptr(self.buf), ctypes.byref(probe),
                                       ctypes.c_void_p(torch.cuda.current_stream(device).cuda_stream)))
        return probe.value


def neighbor_rows_query_tensor(config: SparseSubmConvConfig, in_coords_t: torch.Tensor,
                               query_coords_t: torch.Tensor, check_status: bool = True,
                               workspace: NeighborWorkspace | None = None) -> torch.Tensor:
    """[n_query, K] int32 rows of ``in_coords_t`` at query+offset (-1 absent)."""
    _coords_tensor(in_coords_t)
    _coords_tensor(query_coords_t)
    K = kernel_rows(config)
    n_in, n_q = in_coords_t.shape[0], query_coords_t.shape[0]
    dev = in_coords_t.device
    out = torch.empty((n_q, K), dtype=torch.int32, device=dev)
    ws = workspace or NeighborWorkspace(dev, n_in)
    c = config.c()
    check(lib().sc_neighbor_map_query(ctypes.byref(c), _ptr(in_coords_t), n_in, _ptr(query_coords_t), n_q,
                                      _ptr(ws.buf), ws.bytes, _ptr(out), _stream(in_coords_t)))
    if check_status:
        ws.status(dev)  # one host readback, as the reference's overflow check (neighbor.rs:859-879)
    return out


def neighbor_rows_tensor_from_coords_tensor(config: SparseSubmConvConfig, coords_t: torch.Tensor,
                                            check_status: bool = True,
                                            workspace: NeighborWorkspace | None = None) -> torch.Tensor:
    """Device neighbor map [N, K] int32; duplicates resolve to the lowest row."""
    return neighbor_rows_query_tensor(config, coords_t, coords_t, check_status, workspace)


@dataclass
class ConvSchedule:
    """Row order of a neighbor map (rows grouped by equal valid-tap masks so
    tensor-core tiles skip more taps) and the map permuted into that order.
    Computed once per map; changes scheduling only, never results."""

    order: torch.Tensor          # [N] int32 permutation: tile position -> output row
    nbr_ordered: torch.Tensor    # [N, K] int32 = nbr[order]


def neighbor_schedule(config: SparseSubmConvConfig, neighbor_rows: torch.Tensor,
                      group_mask: torch.Tensor | None = None) -> ConvSchedule:
    """Conv schedule of a map (sc_neighbor_schedule).  With ``group_mask``
    ([N, 8] uint8 0/1, e.g. a C2S conv1's kept-children mask) rows are grouped
    by that mask first (sc_neighbor_schedule_grouped)."""
    _require_cuda("neighbor_rows", neighbor_rows)
    if group_mask is not None:
        return _neighbor_schedule_grouped(config, neighbor_rows, group_mask)
    n = neighbor_rows.shape[0]
    b = ctypes.c_size_t(0)
    check(lib().sc_neighbor_schedule_scratch_bytes(n, ctypes.byref(b)))
    scratch = torch.empty(max(b.value, 1), dtype=torch.uint8, device=neighbor_rows.device)
    order = torch.empty(n, dtype=torch.int32, device=neighbor_rows.device)
    ordered = torch.empty_like(neighbor_rows)
    c = config.c()
    check(lib().sc_neighbor_schedule(ctypes.byref(c), _ptr(neighbor_rows), n, _ptr(scratch), b.value, _ptr(order),
                                     _ptr(ordered), _stream(neighbor_rows)))
    return ConvSchedule(order, ordered)


def _neighbor_schedule_grouped(config, neighbor_rows, group_mask) -> ConvSchedule:
    n = neighbor_rows.shape[0]
    if group_mask.shape != (n, 8) or group_mask.dtype != torch.uint8:
        raise SparseConvError(_lib.SC_ERR_INVALID, "schedule group mask must be [rows, 8] uint8")
    b = ctypes.c_size_t(0)
    check(lib().sc_neighbor_schedule_grouped_scratch_bytes(n, ctypes.byref(b)))
    scratch = torch.empty(max(b.value, 1), dtype=torch.uint8, device=neighbor_rows.device)
    order = torch.empty(n, dtype=torch.int32, device=neighbor_rows.device)
    ordered = torch.empty_like(neighbor_rows)
    c = config.c()
    check(lib().sc_neighbor_schedule_grouped(ctypes.byref(c), _ptr(neighbor_rows), n, _ptr(group_mask.contiguous()),
                                             _ptr(scratch), b.value, _ptr(order), _ptr(ordered),
                                             _stream(neighbor_rows)))
    return ConvSchedule(order, ordered)


@dataclass
class TileSources:
    """Tile-source plan of a neighbor map (sc_neighbor_tile_sources): per
    128-row tile, its distinct source rows and each (row, tap)'s index into
    them.  Lets 64-channel bf16 convs stage each tile's source rows once."""

    buf: torch.Tensor      # the plan (uint8 device buffer)
    max_sources: int       # the largest per-tile distinct-row count


def neighbor_tile_sources(config: SparseSubmConvConfig, neighbor_rows: torch.Tensor,
                          n_in: int | None = None) -> "TileSources | None":
    """The tile-source plan of a map, or None when some tile reads more
    distinct rows than the kernel stages (the convs then run without it).
    ``n_in`` is the number of input rows the map addresses (default: its rows)."""
    _require_cuda("neighbor_rows", neighbor_rows)
    n = neighbor_rows.shape[0]
    K = kernel_rows(config)
    b = ctypes.c_size_t(0)
    check(lib().sc_neighbor_tile_sources_bytes(n, K, ctypes.byref(b)))
    buf = torch.empty(max(b.value, 16), dtype=torch.uint8, device=neighbor_rows.device)
    mx = ctypes.c_int32(0)
    c = config.c()
    rc = lib().sc_neighbor_tile_sources(ctypes.byref(c), _ptr(neighbor_rows), n, n if n_in is None else n_in,
                                        _ptr(buf), b.value, ctypes.byref(mx), _stream(neighbor_rows))
    if rc == _lib.SC_ERR_CAPACITY:
        return None
    check(rc)
    return TileSources(buf, int(mx.value))


@dataclass
class Epilogue:
    """Fused conv epilogue (see sc_epilogue in include/sparseconv.h).

    y = conv + bias (+ residual); ``out`` receives y when ``out2`` is given,
    otherwise post(y) = [LayerNorm(gamma, beta)] -> [SiLU]."""

    residual: torch.Tensor | None = None
    residual_offset: torch.Tensor | None = None
    residual_repeat: int = 1
    layer_norm: bool = False
    ln_width: int = 0
    ln_eps: float = 1e-5
    ln_gamma: torch.Tensor | None = None
    ln_beta: torch.Tensor | None = None
    silu: bool = False
    out2: torch.Tensor | None = None
    out_row_map: torch.Tensor | None = None
    out_row_map_cols: int = 0
    row_order: torch.Tensor | None = None
    nbr_ordered: torch.Tensor | None = None
    schedule: ConvSchedule | None = None
    tile_sources: TileSources | None = None
    _keep: list = field(default_factory=list, repr=False)

    def c(self) -> ScEpilogue:
        order, ordered = self.row_order, self.nbr_ordered
        if self.schedule is not None:
            order, ordered = self.schedule.order, self.schedule.nbr_ordered
        ts = self.tile_sources
        return ScEpilogue(_ptr(self.residual), _ptr(self.residual_offset), int(self.residual_repeat),
                          int(self.layer_norm), int(self.ln_width), float(self.ln_eps), _ptr(self.ln_gamma),
                          _ptr(self.ln_beta), int(self.silu), _ptr(self.out2), _ptr(self.out_row_map),
                          int(self.out_row_map_cols), _ptr(order), _ptr(ordered),
                          _ptr(ts.buf) if ts is not None else None, int(ts.max_sources) if ts is not None else 0)


_DT = {torch.float32: DTYPE_F32, torch.bfloat16: DTYPE_BF16}


def _validate_conv(config, input, neighbor_rows, weight, bias):
    """Mirror of validate_tensor_shapes (src/wgpu/sparse_conv.rs:369-473),
    extended to bf16 (input and weight share the dtype; bias is f32)."""
    for name, t in (("input", input), ("neighbor_rows", neighbor_rows), ("weight", weight)):
        _require_cuda(name, t)
    if input.dtype not in _DT:
        raise SparseConvError(_lib.SC_ERR_INVALID,
                              f"sparse conv input dtype must be F32 or BF16 for kernel path, got {input.dtype}")
    if weight.dtype != input.dtype:
        raise SparseConvError(_lib.SC_ERR_INVALID,
                              f"sparse conv weight dtype must match input ({input.dtype}), got {weight.dtype}")
    if bias is not None:
        _require_cuda("bias", bias)
        if bias.dtype != torch.float32:
            raise SparseConvError(_lib.SC_ERR_INVALID,
                                  f"sparse conv bias dtype must be F32 for kernel path, got {bias.dtype}")
    if neighbor_rows.dtype != torch.int32:
        raise SparseConvError(_lib.SC_ERR_INVALID,
                              f"sparse conv neighbor_rows dtype must be I32 for kernel path, got {neighbor_rows.dtype}")
    if input.dim() != 2:
        raise SparseConvError(_lib.SC_ERR_INVALID, f"sparse conv input rank mismatch: got {input.dim()} expected 2")
    if neighbor_rows.dim() != 2:
        raise SparseConvError(_lib.SC_ERR_INVALID,
                              f"sparse conv neighbor_rows rank mismatch: got {neighbor_rows.dim()} expected 2")
    if weight.dim() != 5:
        raise SparseConvError(_lib.SC_ERR_INVALID, f"sparse conv weight rank mismatch: got {weight.dim()} expected 5")
    if input.shape[1] != config.in_channels:
        raise SparseConvError(_lib.SC_ERR_INVALID,
                              f"sparse conv input channel mismatch: got {input.shape[1]} expected {config.in_channels}")
    if neighbor_rows.shape[0] > input.shape[0]:
        raise SparseConvError(_lib.SC_ERR_INVALID,
                              f"sparse conv neighbor row count exceeds input rows: got {neighbor_rows.shape[0]} "
                              f"input rows {input.shape[0]}")
    K = kernel_rows(config)
    if neighbor_rows.shape[1] != K:
        raise SparseConvError(_lib.SC_ERR_INVALID,
                              f"sparse conv neighbor kernel rows mismatch: got {neighbor_rows.shape[1]} expected {K}")
    exp = [config.out_channels, config.kernel_d, config.kernel_h, config.kernel_w, config.in_channels_per_group]
    if list(weight.shape) != exp:
        raise SparseConvError(_lib.SC_ERR_INVALID,
                              f"sparse conv weight shape mismatch: got {list(weight.shape)} expected {exp}")
    if bias is not None and (bias.dim() != 1 or bias.shape[0] != config.out_channels):
        raise SparseConvError(_lib.SC_ERR_INVALID,
                              f"sparse conv bias len mismatch: got {bias.shape[0]} expected {config.out_channels}")


def sparse_subm_conv_forward(config: SparseSubmConvConfig, input: torch.Tensor, neighbor_rows: torch.Tensor,
                             weight: torch.Tensor, bias: torch.Tensor | None = None,
                             epilogue: Epilogue | None = None, out: torch.Tensor | None = None,
                             out_rows: int | None = None) -> torch.Tensor:
    """Sparse submanifold conv with an optional fused epilogue.  Returns a new
    contiguous [N_query, Cout] tensor (or ``out``) in the input's dtype."""
    _validate_conv(config, input, neighbor_rows, weight, bias)
    n_q = neighbor_rows.shape[0]
    e = epilogue or Epilogue()
    if out is None:
        if e.out_row_map is not None:
            width = config.out_channels // e.out_row_map_cols
            rows = out_rows if out_rows is not None else n_q * e.out_row_map_cols
            out = torch.empty((rows, width), dtype=input.dtype, device=input.device)
        else:
            out = torch.empty((n_q, config.out_channels), dtype=input.dtype, device=input.device)
    c = config.c()
    ec = e.c()
    obs = _CONV_OBSERVER
    if obs is not None:
        obs.before(config, n_q)
    check(lib().sc_subm_conv_forward(ctypes.byref(c), _DT[input.dtype], _ptr(input), input.shape[0],
                                     _ptr(neighbor_rows), n_q, _ptr(weight), _ptr(bias), ctypes.byref(ec),
                                     _ptr(out), _stream(input)))
    if obs is not None:
        obs.after(config, n_q)
    return out


_CONV_OBSERVER = None


def set_conv_observer(observer) -> None:
    """Installs ``observer`` (or removes it, with None): its ``before(config,
    n_rows)`` and ``after(config, n_rows)`` are called around every conv launch,
    on the launching host thread, so that it can record CUDA events on the
    current stream (per-launch device timing).  Changes no result."""
    global _CONV_OBSERVER
    _CONV_OBSERVER = observer


def sparse_subm_conv_forward_cubecl(config: SparseSubmConvConfig, input: torch.Tensor,
                                    neighbor_rows: torch.Tensor, weight: torch.Tensor,
                                    bias: torch.Tensor) -> torch.Tensor:
    """The reference's device entry point (src/wgpu/sparse_conv.rs:293-308):
    plain conv + bias, new output tensor."""
    return sparse_subm_conv_forward(config, input, neighbor_rows, weight, bias)


_IDENTITY_ROWS: dict = {}


def identity_rows(n: int, device) -> torch.Tensor:
    """[n, 1] int32 map with row r -> r: a dense per-row layer as a 1x1x1
    sparse conv.  Cached per device (grown on demand, sliced)."""
    key = torch.device(device)
    t = _IDENTITY_ROWS.get(key)
    if t is None or t.shape[0] < n:
        t = torch.arange(max(n, 1024), dtype=torch.int32, device=key).view(-1, 1)
        _IDENTITY_ROWS[key] = t
    return t[:n]


def linear_forward(input: torch.Tensor, weight: torch.Tensor, bias: torch.Tensor | None = None,
                   epilogue: Epilogue | None = None, out: torch.Tensor | None = None) -> torch.Tensor:
    """Linear layer ``out = input @ weight.T + bias`` with the conv's fused
    epilogue (SiLU, residual, LayerNorm), run as a 1x1x1 sparse conv over the
    identity map, so it takes the same tcgen05 gather-GEMM as the convs.
    ``weight`` is [out, in] row-major as PyTorch stores linear layers (the
    reference's LinearLayer, burn_trellis src/runtime_model/sparse_decoder.rs:623-631;
    math of ``linear_forward``, sparse_decoder_wgpu_ops.rs:1-60: bias first,
    then the GEMM accumulates)."""
    _require_cuda("input", input)
    if input.dim() != 2 or weight.dim() != 2:
        raise SparseConvError(_lib.SC_ERR_INVALID, "linear input and weight must be 2-D")
    rows, cin = input.shape
    cout = weight.shape[0]
    if weight.shape[1] != cin:
        raise SparseConvError(_lib.SC_ERR_INVALID,
                              f"linear: invalid input len {rows * cin}, expected {rows * weight.shape[1]} "
                              f"(rows={rows} in_channels={weight.shape[1]})")
    if bias is not None and bias.shape[0] != cout:
        raise SparseConvError(_lib.SC_ERR_INVALID,
                              f"linear: bias len {bias.shape[0]} does not match out_channels {cout}")
    e = epilogue or Epilogue()
    if (input.dtype == torch.bfloat16 and weight.dtype == torch.bfloat16 and not e.layer_norm and e.out2 is None
            and e.out_row_map is None and e.residual_offset is None and e.schedule is None
            and e.tile_sources is None and (e.residual is None or (e.residual.shape == (rows, cout)
                                                                   and e.residual.dtype == torch.bfloat16))):
        # the dense tensor-core linear (sc_linear_forward); it declines shapes it does not take
        y = out if out is not None else torch.empty((rows, cout), dtype=input.dtype, device=input.device)
        res = e.residual.contiguous() if e.residual is not None else None
        obs = _CONV_OBSERVER
        lcfg = SparseSubmConvConfig(cin, cout, 1, 1, 1)
        if obs is not None:
            obs.before(lcfg, rows)
        rc = lib().sc_linear_forward(_DT[input.dtype], _ptr(input.contiguous()), rows, cin,
                                     _ptr(weight.contiguous()), cout, _ptr(bias), _ptr(res), int(e.silu), _ptr(y),
                                     _stream(input))
        if rc == _lib.SC_OK:
            if obs is not None:
                obs.after(lcfg, rows)
            return y
        if rc != _lib.SC_ERR_UNSUPPORTED:
            check(rc)
    cfg = SparseSubmConvConfig(cin, cout, 1, 1, 1)
    return sparse_subm_conv_forward(cfg, input, identity_rows(rows, input.device),
                                    weight.reshape(cout, 1, 1, 1, cin), bias, epilogue, out=out)


def uses_tensor_cores(config: SparseSubmConvConfig, dtype: torch.dtype) -> bool:
    f = ctypes.c_int32(0)
    c = config.c()
    check(lib().sc_conv_uses_tensor_cores(ctypes.byref(c), _DT[dtype], ctypes.byref(f)))
    return bool(f.value)


def _layer_norm_act(x, gamma, beta, eps, ln, silu, out=None):
    _require_cuda("input", x)
    if x.dim() != 2:
        raise SparseConvError(_lib.SC_ERR_INVALID, "layer norm input must be [rows, channels]")
    y = out if out is not None else torch.empty_like(x)
    check(lib().sc_layer_norm_act(_DT[x.dtype], _ptr(x), x.shape[0], x.shape[1], _ptr(gamma), _ptr(beta),
                                  ctypes.c_float(eps), int(ln), int(silu), _ptr(y), _stream(x)))
    return y


def layer_norm_affine_forward(x, gamma=None, beta=None, eps: float = 1e-5, out=None):
    return _layer_norm_act(x, gamma, beta, eps, True, False, out)


def layer_norm_affine_silu_forward(x, gamma=None, beta=None, eps: float = 1e-5, out=None):
    return _layer_norm_act(x, gamma, beta, eps, True, True, out)


def silu_forward(x, out=None):
    return _layer_norm_act(x, None, None, 0.0, False, True, out)


def bf16_round_to_f32(x: torch.Tensor) -> torch.Tensor:
    _require_cuda("input", x)
    if x.dtype != torch.float32:
        raise SparseConvError(_lib.SC_ERR_INVALID, "bf16_round_to_f32 expects an F32 tensor")
    y = torch.empty_like(x)
    check(lib().sc_bf16_round(_ptr(x), x.numel(), _ptr(y), _stream(x)))
    return y


def gather_rows(src: torch.Tensor, idx: torch.Tensor, out: torch.Tensor | None = None) -> torch.Tensor:
    """out[i] = src[idx[i]] (rows of a contiguous 2-D CUDA tensor)."""
    _require_cuda("src", src)
    _require_cuda("idx", idx)
    if idx.dtype != torch.int32:
        raise SparseConvError(_lib.SC_ERR_INVALID, "gather index dtype must be I32")
    if out is None:
        out = torch.empty((idx.shape[0],) + tuple(src.shape[1:]), dtype=src.dtype, device=src.device)
    row_bytes = src[0].numel() * src.element_size() if src.shape[0] else out[0].numel() * out.element_size()
    check(lib().sc_gather_rows(_ptr(src), src.shape[0], row_bytes, _ptr(idx), idx.shape[0], _ptr(out), _stream(src)))
    return out


def cast(x: torch.Tensor, dtype: torch.dtype) -> torch.Tensor:
    _require_cuda("input", x)
    y = torch.empty(x.shape, dtype=dtype, device=x.device)
    check(lib().sc_cast(_DT[x.dtype], _DT[dtype], _ptr(x), x.numel(), _ptr(y), _stream(x)))
    return y


def subdivision_child_thresholds(threshold: float = 0.0, child_thresholds=None) -> list:
    """Per-child thresholds: a finite child threshold overrides the shared one
    (decoder_subdivision_child_thresholds, sparse_decoder_wgpu_ops.rs:1813-1822)."""
    import math
    ct = list(child_thresholds) if child_thresholds is not None else [float("nan")] * 8
    return [c if math.isfinite(c) else threshold for c in ct]


def subdivision_head(feats: torch.Tensor, weight: torch.Tensor, bias: torch.Tensor | None = None,
                     threshold: float = 0.0, child_thresholds=None, center: bool = False,
                     return_logits: bool = True):
    """to_subdiv logits [N, 8] (linear C -> 8, fp32 accumulate; optional
    centring on the row mean, sparse_decoder_runtime_impl.rs:852-880) and the
    child mask [N, 8] uint8 = logits > per-child threshold
    (subdivision_active_indices_wgpu_async, sparse_decoder_wgpu_ops.rs:928-992).
    ``weight`` is [8, C] in feats' dtype, ``bias`` fp32."""
    _require_cuda("feats", feats)
    if feats.dim() != 2 or weight.shape != (8, feats.shape[1]) or weight.dtype != feats.dtype:
        raise SparseConvError(_lib.SC_ERR_INVALID,
                              f"decoder subdivision logits tensor must have 8 columns (weight {tuple(weight.shape)})")
    n = feats.shape[0]
    logits = torch.empty((n, 8), dtype=torch.float32, device=feats.device) if return_logits else None
    mask = torch.empty((n, 8), dtype=torch.uint8, device=feats.device)
    thr = (ctypes.c_float * 8)(*subdivision_child_thresholds(threshold, child_thresholds))
    check(lib().sc_subdiv_head(_DT[feats.dtype], _ptr(feats), n, feats.shape[1], _ptr(weight.contiguous()),
                               _ptr(bias), ctypes.c_float(threshold), thr, int(center),
                               _ptr(logits) if logits is not None else None, _ptr(mask), _stream(feats)))
    return logits, mask


def subdivide(parent_coords: torch.Tensor, mask: torch.Tensor, parent_channels: int):
    """Channel-to-space child expansion.  Returns (child_row [Np, 8] int32,
    child_coords [Nc, 4] int32, skip_offset [Nc] int64)."""
    _coords_tensor(parent_coords)
    _require_cuda("mask", mask)
    n = parent_coords.shape[0]
    dev = parent_coords.device
    b = ctypes.c_size_t(0)
    check(lib().sc_subdivide_scratch_bytes(n, ctypes.byref(b)))
    scratch = torch.empty(max(b.value, 1), dtype=torch.uint8, device=dev)
    child_row = torch.empty((n, 8), dtype=torch.int32, device=dev)
    coords = torch.empty((max(8 * n, 1), 4), dtype=torch.int32, device=dev)
    skip = torch.empty(max(8 * n, 1), dtype=torch.int64, device=dev)
    nc = ctypes.c_int64(0)
    check(lib().sc_subdivide(_ptr(parent_coords), _ptr(mask), n, parent_channels, _ptr(scratch), _ptr(child_row),
                             _ptr(coords), _ptr(skip), ctypes.byref(nc), _stream(parent_coords)))
    k = nc.value
    return child_row, coords[:k].contiguous(), skip[:k].contiguous()


class DeviceCount:
    """A row count left on the device by an asynchronous call: copied to pinned
    host memory behind the producing kernels; ``value()`` waits for that copy
    only (an event), not for the stream."""

    def __init__(self, d_count: torch.Tensor):
        self.host = torch.empty(1, dtype=d_count.dtype, pin_memory=True)
        self.host.copy_(d_count, non_blocking=True)
        self.event = torch.cuda.Event()
        self.event.record(torch.cuda.current_stream(d_count.device))
        self._value = None

    def value(self) -> int:
        if self._value is None:
            self.event.synchronize()
            self._value = int(self.host[0])
        return self._value


def subdivide_async(parent_coords: torch.Tensor, mask: torch.Tensor, parent_channels: int):
    """sc_subdivide_async: like ``subdivide`` with the child count left on the
    device.  Returns (child_row [Np, 8], child_coords [8 Np, 4], skip_offset
    [8 Np], count: DeviceCount); rows >= count.value() of the last two are
    unused."""
    _coords_tensor(parent_coords)
    _require_cuda("mask", mask)
    n = parent_coords.shape[0]
    dev = parent_coords.device
    b = ctypes.c_size_t(0)
    check(lib().sc_subdivide_scratch_bytes(n, ctypes.byref(b)))
    scratch = torch.empty(max(b.value, 1), dtype=torch.uint8, device=dev)
    child_row = torch.empty((n, 8), dtype=torch.int32, device=dev)
    coords = torch.empty((max(8 * n, 1), 4), dtype=torch.int32, device=dev)
    skip = torch.empty(max(8 * n, 1), dtype=torch.int64, device=dev)
    d_count = torch.empty(4, dtype=torch.int32, device=dev)
    check(lib().sc_subdivide_async(_ptr(parent_coords), _ptr(mask), n, parent_channels, _ptr(scratch),
                                   _ptr(child_row), _ptr(coords), _ptr(skip), _ptr(d_count), _stream(parent_coords)))
    return child_row, coords, skip, DeviceCount(d_count[:1])


@dataclass(frozen=True)
class SparsePatchify3dConfig:
    """Mirror of burn_flex_gmm's SparsePatchify3dConfig (src/lib.rs:26-35)."""
    in_channels: int
    out_channels: int
    frames: int
    height: int
    width: int
    tubelet_size: int
    patch_h: int
    patch_w: int

    def c(self) -> ScPatchify3dConfig:
        return ScPatchify3dConfig(self.in_channels, self.out_channels, self.frames, self.height, self.width,
                                  self.tubelet_size, self.patch_h, self.patch_w)

    def inner_len(self) -> int:
        return self.in_channels * self.tubelet_size * self.patch_h * self.patch_w


def sparse_patchify3d_forward(config: SparsePatchify3dConfig, input: torch.Tensor, coords: torch.Tensor,
                              weight: torch.Tensor, bias: torch.Tensor) -> torch.Tensor:
    """Patch embedding at the listed patches (sparse_patchify3d_forward_flex,
    burn_flex_gmm src/lib.rs:133-240).  ``input`` [B, Cin, T, H, W] (or any
    contiguous tensor of B * Cin*T*H*W elements), ``coords`` [rows, 4] int32
    (batch, tubelet, patch_row, patch_col), ``weight`` [Cout, Cin, tubelet,
    patch_h, patch_w] in the input's dtype, ``bias`` [Cout] fp32.  Returns
    [rows, Cout].  A coordinate outside the grid raises the device fault word
    (the reference's CPU path returns an error) and yields the bias row."""
    for name, t in (("input", input), ("coords", coords), ("weight", weight), ("bias", bias)):
        _require_cuda(name, t)
    if input.dtype not in _DT or weight.dtype != input.dtype:
        raise SparseConvError(_lib.SC_ERR_INVALID, "sparse patchify input and weight must share an F32 or BF16 dtype")
    if bias.shape[0] != config.out_channels:
        raise SparseConvError(_lib.SC_ERR_INVALID, f"sparse patchify bias len mismatch: got {bias.shape[0]} "
                                                   f"expected {config.out_channels}")
    if weight.numel() != config.out_channels * config.inner_len():
        raise SparseConvError(_lib.SC_ERR_INVALID, f"sparse patchify weight len mismatch: got {weight.numel()} "
                                                   f"expected {config.out_channels * config.inner_len()}")
    if coords.dtype != torch.int32 or coords.dim() != 2 or coords.shape[1] != 4:
        raise SparseConvError(_lib.SC_ERR_INVALID, "sparse patchify coords must be [rows, 4] int32")
    rows = coords.shape[0]
    out = torch.empty((rows, config.out_channels), dtype=input.dtype, device=input.device)
    c = config.c()
    nbytes = ctypes.c_size_t(0)
    check(lib().sc_patchify3d_scratch_bytes(ctypes.byref(c), rows, _DT[input.dtype], ctypes.byref(nbytes)))
    scratch = torch.empty(max(int(nbytes.value), 1), dtype=torch.uint8, device=input.device)
    check(lib().sc_patchify3d_forward(ctypes.byref(c), _DT[input.dtype], _ptr(input.contiguous()), input.numel(),
                                      _ptr(coords.contiguous()), rows, _ptr(weight.contiguous()), _ptr(bias),
                                      _ptr(scratch), int(nbytes.value), _ptr(out), _stream(input)))
    return out


def downsample_coords(coords: torch.Tensor) -> torch.Tensor:
    """Output grid of a stride-2 sparse conv: the distinct cells
    ``(batch, x >> 1, y >> 1, z >> 1)`` of ``coords``, sorted by (batch, Morton
    code) like every grid of this path."""
    from .sharding import morton_key

    _coords_tensor(coords)
    if coords.shape[0] == 0:
        return coords.clone()
    half = torch.cat([coords[:, :1], coords[:, 1:] >> 1], 1)
    key = morton_key(half[:, 0], half[:, 1:])
    ukey, inv = torch.unique(key, sorted=True, return_inverse=True)
    out = torch.empty((ukey.numel(), 4), dtype=torch.int32, device=coords.device)
    out[inv] = half
    return out


def sparse_conv3d_stride2_forward(input: torch.Tensor, coords: torch.Tensor, weight: torch.Tensor,
                                  bias: torch.Tensor | None = None, epilogue: Epilogue | None = None,
                                  out_coords: torch.Tensor | None = None):
    """Stride-2 sparse downsample convolution (SparseConv3d, kernel 2, stride 2,
    no padding): the output grid is ``downsample_coords(coords)`` and
    ``out[o] = bias + sum_{(a,b,c) in {0,1}^3} in[row of 2*o + (a,b,c)] @ W[:, a, b, c, :]^T``
    (absent input cells contribute nothing).  ``weight`` is [Cout, 2, 2, 2, Cin].
    The reference has no downsample conv; this is the operation's definition.
    The 2x2x2 map is a neighbor query of 2*o + 1 (the offsets of a 2-wide kernel
    are -1 and 0) and the conv runs on the same gather-GEMM kernels as SubM.
    Returns (out_coords [M, 4], out [M, Cout])."""
    _coords_tensor(coords)
    if weight.dim() != 5 or tuple(weight.shape[1:4]) != (2, 2, 2):
        raise SparseConvError(_lib.SC_ERR_INVALID,
                              f"stride-2 sparse conv weight must be [Cout, 2, 2, 2, Cin], got {list(weight.shape)}")
    cout, cin = int(weight.shape[0]), int(weight.shape[4])
    cfg = SparseSubmConvConfig(cin, cout, 2, 2, 2)
    oc = downsample_coords(coords) if out_coords is None else out_coords
    query = torch.cat([oc[:, :1], oc[:, 1:] * 2 + 1], 1).contiguous()
    nbr = neighbor_rows_query_tensor(cfg, coords, query)
    e = epilogue or Epilogue()
    if e.schedule is None and e.row_order is None and oc.shape[0]:
        e.schedule = neighbor_schedule(cfg, nbr)
    out = sparse_subm_conv_forward(cfg, input, nbr, weight, bias, e)
    return oc, out

"""Decoder weight ingestion: safetensors (f32 / f16 / bf16) -> device tensors in
the layouts the kernels read.

The reference loads every tensor to f32 on the host and packs conv weights for
its CPU GEMM (burn_trellis src/runtime_model/sparse_decoder_loading.rs:1-306).
Here the conv kernel reads the reference layout [Cout, KD, KH, KW, Cin/g]
directly through a TMA tensor map, so ingestion is: parse, validate with the
reference's rules and messages, copy to the device once and store as bf16
(bf16 payloads are copied bit-for-bit; f32 payloads are rounded on the device
by ``sc_cast``; f16 payloads are widened to f32 on the host first).  Biases and
LayerNorm vectors stay f32, as the epilogues read them.

The safetensors container is parsed here (8-byte little-endian header length,
a JSON header of ``{name: {dtype, shape, data_offsets}}``, then the payload),
so no third-party package is needed.
"""
from __future__ import annotations

import json
import struct
from dataclasses import dataclass

import numpy as np
import torch

from . import flex_gmm as F

_DTYPES = {"F32": (np.float32, 4), "F16": (np.float16, 2), "BF16": (np.uint16, 2)}


class WeightError(ValueError):
    """A tensor is missing, has the wrong rank/shape, or an unsupported dtype."""


@dataclass
class TensorView:
    dtype: str       # "F32" | "F16" | "BF16"
    shape: tuple
    data: np.ndarray  # raw payload: float32, float16, or uint16 bit patterns for BF16


def read_safetensors(path_or_bytes) -> dict:
    """name -> TensorView (the payload is a view of the file's bytes)."""
    buf = path_or_bytes if isinstance(path_or_bytes, (bytes, bytearray)) else open(path_or_bytes, "rb").read()
    if len(buf) < 8:
        raise WeightError("safetensors: truncated header")
    (hlen,) = struct.unpack("<Q", buf[:8])
    header = json.loads(bytes(buf[8:8 + hlen]).decode("utf-8"))
    base = 8 + hlen
    out = {}
    for name, meta in header.items():
        if name == "__metadata__":
            continue
        dt = meta["dtype"]
        shape = tuple(int(v) for v in meta["shape"])
        b0, b1 = (int(v) for v in meta["data_offsets"])
        if dt not in _DTYPES:
            out[name] = TensorView(dt, shape, np.frombuffer(buf, np.uint8, b1 - b0, base + b0))
            continue
        npdt, size = _DTYPES[dt]
        if (b1 - b0) % size != 0:
            raise WeightError(f"invalid {dt.lower()} tensor payload byte length {b1 - b0}; must be divisible by {size}")
        out[name] = TensorView(dt, shape, np.frombuffer(buf, npdt, (b1 - b0) // size, base + b0))
    return out


def read_weights(path: str) -> dict:
    """name -> TensorView of a decoder weight file: safetensors, or a ``.bpk``
    blob burnpack (or its ``.parts.json`` split) whose payload is the
    safetensors file, as the reference's loader accepts
    (sparse_decoder_loading.rs:315-348)."""
    if str(path).lower().endswith(".bpk"):
        from .burnpack import read_blob

        return read_safetensors(read_blob(str(path)))
    return read_safetensors(path)


def write_safetensors(path, tensors: dict, bf16: tuple = ()) -> None:
    """Writes float32 / float16 arrays; names in ``bf16`` are stored as BF16
    (round-to-nearest-even of the float32 values)."""
    header, blobs, off = {}, [], 0
    for name, arr in tensors.items():
        a = np.ascontiguousarray(arr)
        if name in bf16:
            u = a.astype(np.float32).view(np.uint32)
            blob = (((u + 0x7FFF + ((u >> 16) & 1)) >> 16).astype(np.uint16)).tobytes()
            dt = "BF16"
        elif a.dtype == np.float16:
            blob, dt = a.tobytes(), "F16"
        else:
            blob, dt = a.astype(np.float32).tobytes(), "F32"
        header[name] = {"dtype": dt, "shape": list(a.shape), "data_offsets": [off, off + len(blob)]}
        blobs.append(blob)
        off += len(blob)
    h = json.dumps(header).encode("utf-8")
    h += b" " * ((8 - len(h) % 8) % 8)
    with open(path, "wb") as f:
        f.write(struct.pack("<Q", len(h)))
        f.write(h)
        for b in blobs:
            f.write(b)


def _tensor(st: dict, key: str) -> TensorView:
    """load_tensor_f32 (sparse_decoder_loading.rs:236-263): presence, dtype, element count."""
    if key not in st:
        raise WeightError(f"missing tensor '{key}' in safetensors")
    v = st[key]
    if v.dtype not in _DTYPES:
        raise WeightError(f"tensor '{key}' has unsupported dtype {v.dtype}; expected f32/f16/bf16")
    expected = int(np.prod(v.shape, dtype=np.int64)) if v.shape else 1
    if v.data.size != expected:
        raise WeightError(f"tensor '{key}' element count mismatch: expected {expected}, got {v.data.size}")
    return v


def _to_device(v: TensorView, device, dtype) -> torch.Tensor:
    """Host payload -> device tensor of ``dtype`` (bf16 or f32)."""
    if v.dtype == "BF16":
        t = torch.from_numpy(v.data.view(np.int16).reshape(v.shape).copy()).to(device).view(torch.bfloat16)
        return t if dtype == torch.bfloat16 else F.cast(t, torch.float32)
    host = v.data.astype(np.float32) if v.dtype == "F16" else np.array(v.data, np.float32)
    t = torch.from_numpy(host.reshape(v.shape)).to(device)
    return t if dtype == torch.float32 else F.cast(t, dtype)


def load_vector(st: dict, key: str, expected_len: int, device) -> torch.Tensor:
    """load_vector (sparse_decoder_loading.rs:215-234)."""
    v = _tensor(st, key)
    if len(v.shape) != 1:
        raise WeightError(f"tensor '{key}' expected rank=1, got rank={len(v.shape)}")
    if expected_len > 0 and v.shape[0] != expected_len:
        raise WeightError(f"tensor '{key}' expected len={expected_len}, got len={v.shape[0]}")
    return _to_device(v, device, torch.float32)


def _bias(st: dict, key: str, out_channels: int) -> TensorView:
    v = _tensor(st, key)
    if len(v.shape) != 1 or v.shape[0] != out_channels:
        raise WeightError(f"tensor '{key}' expected shape=[{out_channels}], got {list(v.shape)}")
    return v


def load_linear(st: dict, weight_key: str, bias_key: str, expected_in: int, expected_out: int, device,
                dtype=torch.bfloat16):
    """load_linear / load_linear_dynamic (sparse_decoder_loading.rs:1-91):
    weight [out, in] (PyTorch layout, as linear_forward consumes it), bias [out]."""
    v = _tensor(st, weight_key)
    if len(v.shape) != 2:
        raise WeightError(f"tensor '{weight_key}' expected rank=2, got rank={len(v.shape)}")
    out_c, in_c = v.shape
    if expected_in > 0 and in_c != expected_in:
        raise WeightError(f"tensor '{weight_key}' expected in_channels={expected_in}, got {in_c}")
    if expected_out > 0 and out_c != expected_out:
        raise WeightError(f"tensor '{weight_key}' expected out_channels={expected_out}, got {out_c}")
    bv = _bias(st, bias_key, out_c)  # every check before any copy
    return _to_device(v, device, dtype), _to_device(bv, device, torch.float32)


def load_sparse_conv(st: dict, weight_key: str, bias_key: str, expected_in: int, expected_out: int, device,
                     dtype=torch.bfloat16):
    """load_sparse_conv (sparse_decoder_loading.rs:93-200): weight
    [Cout, KD, KH, KW, Cin/g] kept in that layout (the TMA tensor map reads it
    as-is: no packing), groups = expected_in / (Cin/g).  Returns
    (SparseSubmConvConfig, weight, bias)."""
    v = _tensor(st, weight_key)
    if len(v.shape) != 5:
        raise WeightError(f"tensor '{weight_key}' expected rank=5, got rank={len(v.shape)}")
    out_c, kd, kh, kw, in_pg = v.shape
    if kd == 0 or kh == 0 or kw == 0:
        raise WeightError(f"tensor '{weight_key}' has invalid kernel dims ({kd},{kh},{kw})")
    if in_pg == 0:
        raise WeightError(f"tensor '{weight_key}' has invalid in_channels_per_group=0")
    if expected_out > 0 and out_c != expected_out:
        raise WeightError(f"tensor '{weight_key}' expected out_channels={expected_out}, got {out_c}")
    in_c = expected_in if expected_in > 0 else in_pg
    if in_c < in_pg or in_c % in_pg != 0:
        raise WeightError(f"tensor '{weight_key}' expected_in={in_c} is incompatible with in_per_group={in_pg}")
    groups = in_c // in_pg
    if groups == 0 or out_c % groups != 0:
        raise WeightError(f"tensor '{weight_key}' has incompatible grouped channels (groups={groups}, "
                          f"out_channels={out_c})")
    bv = _bias(st, bias_key, out_c)
    cfg = F.SparseSubmConvConfig(in_c, out_c, kd, kh, kw, in_pg, out_c // groups, groups)
    return cfg, _to_device(v, device, dtype), _to_device(bv, device, torch.float32)


def load_convnext_stage(st: dict, stage_idx: int, num_blocks: int, channels: int, device,
                        dtype=torch.bfloat16):
    """The ConvNeXt blocks of decoder stage ``stage_idx`` (keys
    ``blocks.{stage}.{block}.conv / norm / mlp.0 / mlp.2``,
    sparse_decoder_runtime_impl.rs:97-135) as a ConvNeXtStack."""
    from .blocks import ConvNeXtParams, ConvNeXtStack

    out = []
    for b in range(num_blocks):
        pre = f"blocks.{stage_idx}.{b}"
        _, w, bias = load_sparse_conv(st, f"{pre}.conv.weight", f"{pre}.conv.bias", channels, channels, device, dtype)
        ng = load_vector(st, f"{pre}.norm.weight", channels, device)
        nb = load_vector(st, f"{pre}.norm.bias", channels, device)
        w0, b0 = load_linear(st, f"{pre}.mlp.0.weight", f"{pre}.mlp.0.bias", channels, 0, device, dtype)
        w2, b2 = load_linear(st, f"{pre}.mlp.2.weight", f"{pre}.mlp.2.bias", w0.shape[0], channels, device, dtype)
        out.append(ConvNeXtParams(w, bias, ng, nb, w0, b0, w2, b2))
    return ConvNeXtStack(out)


def load_c2s_block(st: dict, stage_idx: int, up_idx: int, in_channels: int, out_channels: int, device,
                   with_subdiv: bool = True, dtype=torch.bfloat16):
    """The C2S upsample block (keys ``blocks.{stage}.{up}.norm1 / conv1 / conv2 /
    to_subdiv``, sparse_decoder_runtime_impl.rs:140-185)."""
    from .blocks import C2SParams, C2SUpsampleBlock

    pre = f"blocks.{stage_idx}.{up_idx}"
    g = load_vector(st, f"{pre}.norm1.weight", in_channels, device)
    b = load_vector(st, f"{pre}.norm1.bias", in_channels, device)
    _, w1, b1 = load_sparse_conv(st, f"{pre}.conv1.weight", f"{pre}.conv1.bias", in_channels, 8 * out_channels,
                                 device, dtype)
    _, w2, b2 = load_sparse_conv(st, f"{pre}.conv2.weight", f"{pre}.conv2.bias", out_channels, out_channels,
                                 device, dtype)
    sub = load_linear(st, f"{pre}.to_subdiv.weight", f"{pre}.to_subdiv.bias", in_channels, 8, device, dtype) \
        if with_subdiv else (None, None)
    return C2SUpsampleBlock(C2SParams(g, b, w1, b1, w2, b2, *sub))

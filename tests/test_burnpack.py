"""Burnpack (.bpk) decoder-weight containers (burn_trellis src/blob_burnpack.rs,
src/runtime_model/weight_parts.rs, loader sparse_decoder_loading.rs:315-396):
single-tensor and chunked blobs, split parts with a manifest, the reference's
error messages, and weights loaded from a .bpk equal to the same safetensors."""
import json
import struct

import numpy as np
import pytest

from bevy_synth_b200 import burnpack as B
from bevy_synth_b200 import weights as W


def _safetensors_bytes(tmp_path):
    rng = np.random.default_rng(0)
    t = {"blocks.0.conv.weight": rng.standard_normal((8, 3, 3, 3, 4)).astype(np.float32),
         "blocks.0.conv.bias": rng.standard_normal(8).astype(np.float32),
         "blocks.0.mlp.0.weight": rng.standard_normal((16, 8)).astype(np.float32)}
    p = tmp_path / "m.safetensors"
    W.write_safetensors(p, t, bf16=("blocks.0.mlp.0.weight",))
    return p.read_bytes(), t


@pytest.mark.parametrize("chunk", [1 << 20, 333])
def test_blob_roundtrip_and_weights(tmp_path, chunk):
    raw, t = _safetensors_bytes(tmp_path)
    path = str(tmp_path / "model.bpk")
    sizes = B.write_blob(path, raw, chunk)
    assert (len(sizes) == 1) == (chunk >= len(raw))
    assert B.read_blob(path) == raw
    a, b = W.read_weights(path), W.read_safetensors(raw)
    assert set(a) == set(b)
    for k in a:
        assert a[k].dtype == b[k].dtype and a[k].shape == b[k].shape
        assert np.array_equal(a[k].data.view(np.uint8), b[k].data.view(np.uint8))


def test_parts_manifest(tmp_path):
    raw, _ = _safetensors_bytes(tmp_path)
    half = len(raw) // 2
    parts = []
    for i, piece in enumerate((raw[:half], raw[half:])):
        name = f"model.bpk.part-{i:05d}.bpk"
        B.write_blob(str(tmp_path / name), piece)
        parts.append({"path": name, "bytes": len(piece)})
    (tmp_path / "model.bpk.parts.json").write_text(json.dumps({"source_file": "model.bpk", "parts": parts}))
    assert B.read_blob(str(tmp_path / "model.bpk")) == raw
    (tmp_path / "other.bpk.parts.json").write_text(json.dumps({"source_file": "model.bpk", "parts": parts}))
    with pytest.raises(B.BurnpackError, match="does not match requested"):
        B.read_blob(str(tmp_path / "other.bpk"))


def test_wide_integer_blob_keeps_low_bytes(tmp_path):
    """Blob tensors stored as wider integers keep the low byte of each element."""
    payload = np.arange(10, dtype=np.int64)
    meta = B._cbor_encode({"tensors": {"bytes": {"dtype": "I64", "shape": [10], "data_offsets": [0, 80]}}})
    start = (10 + len(meta) + 255) // 256 * 256
    data = struct.pack("<IHI", B.MAGIC, 1, len(meta)) + meta + b"\0" * (start - 10 - len(meta)) + payload.tobytes()
    assert B.blob_bytes(data) == bytes(range(10))


def test_errors(tmp_path):
    with pytest.raises(B.BurnpackError, match="invalid burnpack magic"):
        B.blob_bytes(b"\0" * 64)
    with pytest.raises(B.BurnpackError, match="too short"):
        B.blob_bytes(b"BU")
    meta = B._cbor_encode({"tensors": {"weights": {"dtype": "U8", "shape": [4], "data_offsets": [0, 4]}}})
    data = struct.pack("<IHI", B.MAGIC, 1, len(meta)) + meta + b"\0" * 300
    with pytest.raises(B.BurnpackError, match="not a blob payload"):
        B.blob_bytes(data)
    meta = B._cbor_encode({"tensors": {"bytes": {"dtype": "F32", "shape": [1], "data_offsets": [0, 4]}}})
    data = struct.pack("<IHI", B.MAGIC, 1, len(meta)) + meta + b"\0" * 300
    with pytest.raises(B.BurnpackError, match="unsupported dtype"):
        B.blob_bytes(data)


def test_cbor_decoder_against_reference_encoding():
    cbor2 = pytest.importorskip("cbor2")
    obj = {"tensors": {"blob_chunks.0": {"dtype": "U8", "shape": [70000], "data_offsets": [0, 70000]},
                       "blob_chunks.1": {"dtype": {"Bool": "Native"}, "shape": [3], "data_offsets": [70144, 70147]}},
           "metadata": {"x": [1, -2, 3.5, True, None]}}
    enc = cbor2.dumps(obj)
    assert B._cbor_decode(enc)[0] == obj
    assert cbor2.loads(B._cbor_encode(obj["tensors"])) == obj["tensors"]

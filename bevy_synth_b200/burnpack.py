"""Burnpack (``.bpk``) weight containers, the format the reference ships its
decoder weights in (burn_trellis src/runtime_model/sparse_decoder_loading.rs:
315-396 -> src/blob_burnpack.rs, with split files via
src/runtime_model/weight_parts.rs).

A decoder ``.bpk`` is a *blob* burnpack: its tensors hold the bytes of the
original safetensors file, either as one tensor ``bytes`` or as chunks
``blob_chunks.<i>``.  The container is:

* a 10-byte header -- magic ``0x4255524E`` (little-endian u32), 2 bytes, and
  the metadata length (little-endian u32) at bytes 6..10;
* CBOR metadata ``{"tensors": {name: {"dtype", "shape", "data_offsets"}}}``;
* the data section, starting at the header + metadata length rounded up to
  256 bytes; ``data_offsets`` are relative to it.  Files written by older
  writers put the payload at the end of the file instead; the start is
  inferred the way the reference does (``blob_payload_start``).

Byte tensors are copied; wider integer tensors keep the low byte of each
element (the reference's ``append_blob_segment_bytes``).  A ``<name>.parts.json``
manifest ``{"source_file", "parts": [{"path", "bytes"}]}`` splits one blob over
several part files, each itself a blob burnpack; their payloads concatenate.

The CBOR subset the metadata uses (maps, arrays, strings, integers, simple
values) is decoded here, so no third-party package is needed.
"""
from __future__ import annotations

import json
import os
import struct

MAGIC = 0x4255524E
HEADER_SIZE = 10
TENSOR_ALIGNMENT = 256
BLOB_CHUNK_PREFIX = "blob_chunks."
_INT_SIZES = {"U8": 1, "I8": 1, "U16": 2, "I16": 2, "U32": 4, "I32": 4, "U64": 8, "I64": 8}


class BurnpackError(ValueError):
    """The file is not a readable blob burnpack."""


# ------------------------------------------------------------------ CBOR
def _cbor_decode(buf: bytes, pos: int = 0):
    """One CBOR item at ``pos`` -> (value, next position)."""
    if pos >= len(buf):
        raise BurnpackError("burnpack metadata: truncated CBOR")
    ib = buf[pos]
    major, info = ib >> 5, ib & 31
    pos += 1

    def arg(info, pos):
        if info < 24:
            return info, pos
        n = {24: 1, 25: 2, 26: 4, 27: 8}.get(info)
        if n is None:
            return None, pos  # indefinite length
        if pos + n > len(buf):
            raise BurnpackError("burnpack metadata: truncated CBOR")
        return int.from_bytes(buf[pos:pos + n], "big"), pos + n

    if major in (0, 1):
        v, pos = arg(info, pos)
        return (v if major == 0 else -1 - v), pos
    if major in (2, 3):
        n, pos = arg(info, pos)
        if n is None:  # indefinite: definite-length chunks until 0xff
            parts = []
            while buf[pos] != 0xFF:
                p, pos = _cbor_decode(buf, pos)
                parts.append(p)
            pos += 1
            return (b"".join(parts) if major == 2 else "".join(parts)), pos
        raw = bytes(buf[pos:pos + n])
        return (raw if major == 2 else raw.decode("utf-8")), pos + n
    if major == 4:
        n, pos = arg(info, pos)
        out = []
        while (n is None and buf[pos] != 0xFF) or (n is not None and len(out) < n):
            v, pos = _cbor_decode(buf, pos)
            out.append(v)
        return out, pos + (1 if n is None else 0)
    if major == 5:
        n, pos = arg(info, pos)
        out = {}
        while (n is None and buf[pos] != 0xFF) or (n is not None and len(out) < n):
            k, pos = _cbor_decode(buf, pos)
            v, pos = _cbor_decode(buf, pos)
            out[k if not isinstance(k, list) else tuple(k)] = v
        return out, pos + (1 if n is None else 0)
    if major == 6:
        _, pos = arg(info, pos)
        return _cbor_decode(buf, pos)
    # major 7: simple values and floats
    if info == 20:
        return False, pos
    if info == 21:
        return True, pos
    if info in (22, 23):
        return None, pos
    if info == 25:
        return struct.unpack(">e", buf[pos:pos + 2])[0], pos + 2
    if info == 26:
        return struct.unpack(">f", buf[pos:pos + 4])[0], pos + 4
    if info == 27:
        return struct.unpack(">d", buf[pos:pos + 8])[0], pos + 8
    raise BurnpackError(f"burnpack metadata: unsupported CBOR item {ib:#x}")


def _cbor_encode(v) -> bytes:
    def head(major, n):
        if n < 24:
            return bytes([(major << 5) | n])
        for info, size in ((24, 1), (25, 2), (26, 4), (27, 8)):
            if n < (1 << (8 * size)):
                return bytes([(major << 5) | info]) + n.to_bytes(size, "big")
        raise BurnpackError("CBOR integer too large")

    if isinstance(v, bool):
        return bytes([0xF5 if v else 0xF4])
    if isinstance(v, int):
        return head(0, v) if v >= 0 else head(1, -1 - v)
    if isinstance(v, str):
        b = v.encode("utf-8")
        return head(3, len(b)) + b
    if isinstance(v, (bytes, bytearray)):
        return head(2, len(v)) + bytes(v)
    if isinstance(v, (list, tuple)):
        return head(4, len(v)) + b"".join(_cbor_encode(x) for x in v)
    if isinstance(v, dict):
        return head(5, len(v)) + b"".join(_cbor_encode(k) + _cbor_encode(x) for k, x in v.items())
    raise BurnpackError(f"cannot CBOR-encode {type(v).__name__}")


# ------------------------------------------------------------------ reading
def _dtype_name(d) -> str:
    """serde's encoding of burn's DType: a unit variant is its name, a variant
    with data is a one-entry map {name: data}."""
    if isinstance(d, str):
        return d
    if isinstance(d, dict) and len(d) == 1:
        return str(next(iter(d)))
    raise BurnpackError(f"burnpack metadata: unreadable dtype {d!r}")


def _payload_start(data_section_start: int, file_len: int, max_end: int) -> int:
    """Where the tensor data begins (blob_burnpack.rs blob_payload_start): the
    aligned data section, or -- for files whose payload was written flush to
    the end -- file_len - max_end when that differs by more than the alignment."""
    inferred = max(file_len - max_end, 0)
    if inferred >= data_section_start:
        return data_section_start if inferred - data_section_start <= TENSOR_ALIGNMENT else inferred
    return inferred if data_section_start - inferred <= TENSOR_ALIGNMENT else data_section_start


def blob_bytes(data: bytes, name: str = "<memory>") -> bytes:
    """The blob payload of one burnpack file's bytes."""
    if len(data) < HEADER_SIZE:
        raise BurnpackError(f"burnpack byte stream is too short ({len(data)} bytes)")
    (magic,) = struct.unpack("<I", data[:4])
    if magic != MAGIC:
        raise BurnpackError(f"invalid burnpack magic in '{name}': expected {MAGIC:#x}, found {magic:#x}")
    (meta_len,) = struct.unpack("<I", data[6:10])
    if HEADER_SIZE + meta_len > len(data):
        raise BurnpackError(f"burnpack metadata out of bounds: header={HEADER_SIZE} metadata={meta_len} "
                            f"total={len(data)}")
    meta, _ = _cbor_decode(data[HEADER_SIZE:HEADER_SIZE + meta_len])
    tensors = meta.get("tensors", {}) if isinstance(meta, dict) else {}
    if not tensors:
        raise BurnpackError(f"burnpack '{name}' contains no tensors")
    data_start = (HEADER_SIZE + meta_len + TENSOR_ALIGNMENT - 1) // TENSOR_ALIGNMENT * TENSOR_ALIGNMENT
    if "bytes" in tensors:
        segs = [(0, tensors["bytes"])]
    else:
        segs = []
        for tname, desc in tensors.items():
            if tname.startswith(BLOB_CHUNK_PREFIX):
                head = tname[len(BLOB_CHUNK_PREFIX):].split(".")[0]
                segs.append((int(head) if head.isdigit() else 1 << 62, desc))
        if not segs:
            raise BurnpackError(f"burnpack '{name}' is not a blob payload (expected legacy 'bytes' tensor or "
                                f"'{BLOB_CHUNK_PREFIX}' tensor prefix)")
        segs.sort(key=lambda s: (s[0], int(s[1]["data_offsets"][0])))
    max_end = max(int(d["data_offsets"][1]) for _, d in segs)
    base = _payload_start(data_start, len(data), max_end)
    out = bytearray()
    for ordinal, d in segs:
        start, end = (int(v) for v in d["data_offsets"])
        if end < start:
            raise BurnpackError(f"invalid burnpack tensor offsets in '{name}': {start}..{end}")
        if end == start:
            continue
        if base + end > len(data):
            raise BurnpackError(f"burnpack '{name}' payload slice out of bounds: {base + start}..{base + end} "
                                f"(total={len(data)})")
        raw = data[base + start:base + end]
        dt = _dtype_name(d["dtype"])
        size = 1 if dt.startswith("Bool") else _INT_SIZES.get(dt)
        if size is None:
            raise BurnpackError(f"blob tensor '{ordinal}' uses unsupported dtype {dt}; expected byte or "
                                f"integer storage")
        count = 1
        for dim in d["shape"]:
            count *= int(dim)
        if count * size != len(raw):
            raise BurnpackError(f"blob tensor '{ordinal}' byte length mismatch for dtype {dt}: shape "
                                f"{list(d['shape'])} implies {count * size} bytes, offsets contain {len(raw)} bytes")
        out += raw if size == 1 else raw[::size]   # low byte of each little-endian element
    return bytes(out)


def parts_manifest_path(path: str) -> str:
    return os.path.join(os.path.dirname(path), os.path.basename(path) + ".parts.json")


def read_blob(path: str) -> bytes:
    """The blob of ``path``, or of its ``.parts.json`` split when the file
    itself is absent (weight_parts.rs load_blob_bytes_from_burnpack_or_parts)."""
    if os.path.exists(path):
        with open(path, "rb") as f:
            return blob_bytes(f.read(), path)
    manifest = parts_manifest_path(path)
    if not os.path.exists(manifest):
        raise BurnpackError(f"burnpack '{path}' not found (and no '{manifest}')")
    with open(manifest, "rb") as f:
        m = json.loads(f.read())
    parts = m.get("parts") or []
    if not parts:
        raise BurnpackError(f"burnpack parts manifest '{manifest}' contains no parts")
    src = str(m.get("source_file", "")).strip()
    if src and os.path.basename(path) != src:
        raise BurnpackError(f"burnpack parts manifest '{manifest}' source_file '{src}' does not match "
                            f"requested '{path}'")
    merged = bytearray()
    for i, part in enumerate(parts):
        p = part["path"] if os.path.isabs(part["path"]) else os.path.join(os.path.dirname(manifest), part["path"])
        with open(p, "rb") as f:
            raw = f.read()
        try:
            payload = blob_bytes(raw, p)
        except BurnpackError as e:
            raise BurnpackError(f"failed to decode burnpack part {i + 1}/{len(parts)} '{p}' for '{path}': {e}")
        want = int(part.get("bytes", 0))
        if want > 0 and not (len(raw) == want or 0 <= len(raw) - want <= TENSOR_ALIGNMENT or len(payload) == want):
            raise BurnpackError(f"burnpack part '{p}' size mismatch: manifest={want} file={len(raw)} "
                                f"payload={len(payload)}")
        merged += payload
    return bytes(merged)


# ------------------------------------------------------------------ writing (tests, tooling)
def write_blob(path: str, blob: bytes, chunk_bytes: int = 32 << 20) -> list:
    """Writes ``blob`` as a blob burnpack: one ``bytes`` tensor when it fits one
    chunk, else ``blob_chunks.<i>`` tensors of ``chunk_bytes`` each (u8, each
    256-byte aligned in the data section).  Returns the chunk sizes."""
    chunk_bytes = max(int(chunk_bytes), 1)
    chunks = [blob[i:i + chunk_bytes] for i in range(0, len(blob), chunk_bytes)] or [b""]
    names = ["bytes"] if len(chunks) == 1 else [f"{BLOB_CHUNK_PREFIX}{i}" for i in range(len(chunks))]
    tensors, off, payload = {}, 0, bytearray()
    for nm, c in zip(names, chunks):
        pad = (-off) % TENSOR_ALIGNMENT
        payload += b"\0" * pad
        off += pad
        tensors[nm] = {"dtype": "U8", "shape": [len(c)], "data_offsets": [off, off + len(c)]}
        payload += c
        off += len(c)
    meta = _cbor_encode({"tensors": tensors})
    head = struct.pack("<IHI", MAGIC, 1, len(meta))
    start = (HEADER_SIZE + len(meta) + TENSOR_ALIGNMENT - 1) // TENSOR_ALIGNMENT * TENSOR_ALIGNMENT
    with open(path, "wb") as f:
        f.write(head + meta + b"\0" * (start - HEADER_SIZE - len(meta)) + payload)
    return [len(c) for c in chunks]

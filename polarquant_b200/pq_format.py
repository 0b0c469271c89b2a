"""The corpus and parameter files of the reference: `.pq` and `.params`
(remex/pq_format.py), and the host side of the `.npz` and Arrow IPC files of
CompressedVectors / PackedVectors (remex/core.py:64-116, :326-439).

`.pq` (remex/pq_format.py:3-17, :87-131), little-endian:

    bytes 0-3   b"PQ\\x00\\x01" (magic, reserved byte, version 1)
    bytes 4-7   d, u32
    bytes 8-15  n, u64
    byte 16     bits, u8
    bytes 17-31 zero
    then        the packed code stream of all n*d codes (packed_nbytes(n, d, bits) bytes)
    then        n f32 norms

`.params` (remex/pq_format.py:41-66): b"PR\\x00\\x01", d u32 at byte 4, bits u8 at
byte 8, zero to byte 16, then R (d x d f32, row-major), the 2^bits - 1
boundaries and the 2^bits centroids (f32).

These are host-side file formats (the Mojo CLI's inputs), kept byte-identical
so files move between the two implementations.  A corpus resident on the GPU
is written from its device rows when every row is a whole number of bytes
(the stream is then the rows back to back); otherwise, and on loading, the
host packers of `polarquant_b200.packing` do the work.
"""

from __future__ import annotations

import struct
from pathlib import Path

import numpy as np

from .packing import pack, packed_nbytes, unpack

PQ_HEADER_BYTES = 32
PQ_VERSION = 1
PQ_MAGIC = b"PQ\x00\x01"

PARAMS_HEADER_BYTES = 16
PARAMS_VERSION = 1
PARAMS_MAGIC = b"PR\x00\x01"


def save_params(path, quantizer) -> None:
    """Writes (R, boundaries, centroids) of a Quantizer (remex/pq_format.py:41-66)."""
    d, bits = int(quantizer.d), int(quantizer.bits)
    R = np.ascontiguousarray(quantizer.R, dtype=np.float32)
    bnd = np.ascontiguousarray(quantizer.boundaries, dtype=np.float32)
    cent = np.ascontiguousarray(quantizer.centroids, dtype=np.float32)
    if R.shape != (d, d):
        raise ValueError(f"R shape {R.shape} != (d, d) = ({d}, {d})")
    if bnd.size != (1 << bits) - 1:
        raise ValueError("boundaries size mismatch")
    if cent.size != (1 << bits):
        raise ValueError("centroids size mismatch")
    head = bytearray(PARAMS_HEADER_BYTES)
    head[0:4] = PARAMS_MAGIC
    head[4:8] = struct.pack("<I", d)
    head[8] = bits & 0xFF
    with open(path, "wb") as f:
        f.write(bytes(head))
        f.write(R.astype("<f4", copy=False).tobytes())
        f.write(bnd.astype("<f4", copy=False).tobytes())
        f.write(cent.astype("<f4", copy=False).tobytes())


def _code_stream(compressed) -> np.ndarray:
    """The packed stream of all n*d codes of a CompressedVectors."""
    n, d, bits = int(compressed.n), int(compressed.d), int(compressed.bits)
    rows = getattr(compressed, "_rows", None)
    if rows is not None and (d * bits) % 8 == 0:
        return rows.rows_host().reshape(-1)  # rows of d*bits/8 bytes, back to back
    return pack(np.asarray(compressed.indices).reshape(-1), bits)


def save_pq(path, compressed) -> None:
    """Writes a CompressedVectors as a .pq file (remex/pq_format.py:69-91)."""
    n, d, bits = int(compressed.n), int(compressed.d), int(compressed.bits)
    stream = np.ascontiguousarray(_code_stream(compressed), dtype=np.uint8)
    want = packed_nbytes(n, d, bits)
    if stream.nbytes != want:
        raise ValueError(f"packed indices size mismatch: got {stream.nbytes}, expected {want}")
    head = bytearray(PQ_HEADER_BYTES)
    head[0:4] = PQ_MAGIC
    head[4:8] = struct.pack("<I", d)
    head[8:16] = struct.pack("<Q", n)
    head[16] = bits & 0xFF
    norms = np.ascontiguousarray(compressed.norms, dtype=np.float32)
    with open(path, "wb") as f:
        f.write(bytes(head))
        f.write(stream.tobytes())
        f.write(norms.astype("<f4", copy=False).tobytes())


def load_pq(path):
    """Reads a .pq file into a CompressedVectors (remex/pq_format.py:94-131).

    Same checks and messages as the reference: size, magic, version,
    5-7-bit widths, truncation.  The codes are unpacked on the host; the
    corpus moves to the GPU on its first search."""
    from .core import CompressedVectors

    raw = Path(path).read_bytes()
    if len(raw) < PQ_HEADER_BYTES:
        raise ValueError(".pq file too small")
    if raw[0:2] != b"PQ":
        raise ValueError("bad .pq magic")
    if raw[3] != PQ_VERSION:
        raise ValueError(f"unsupported .pq version: {raw[3]}")
    (d,) = struct.unpack("<I", raw[4:8])
    (n,) = struct.unpack("<Q", raw[8:16])
    bits = raw[16]
    if bits in (5, 6, 7):
        raise ValueError(f"bits={bits} is not supported. Use 1-4 or 8 bits.")
    nbytes = packed_nbytes(n, d, bits)
    if len(raw) < PQ_HEADER_BYTES + nbytes + 4 * n:
        raise ValueError("truncated .pq data")
    stream = np.frombuffer(raw, dtype=np.uint8, count=nbytes, offset=PQ_HEADER_BYTES)
    norms = np.frombuffer(raw, dtype="<f4", count=n, offset=PQ_HEADER_BYTES + nbytes)
    codes = unpack(stream, bits, n * d).reshape(n, d)
    return CompressedVectors(codes.copy(), norms.astype(np.float32), d, bits)


# ---------------------------------------------------------------------------
# .npz (remex/core.py:64-91, :326-347) and Arrow IPC / Feather v2
# (remex/core.py:349-439): the host side of CompressedVectors / PackedVectors
# .save, .load, .save_arrow and .load_arrow.  The classes hand these the host
# copies of their rows and norms and build device rows from what they return.
# ---------------------------------------------------------------------------

def write_npz(path, packed_flat, norms, d: int, bits: int, n: int) -> None:
    """Keys packed_indices (flat uint8), norms, d, bits, n (int32), compressed."""
    np.savez_compressed(path, packed_indices=np.ascontiguousarray(packed_flat, np.uint8).ravel(),
                        norms=norms, d=np.int32(d), bits=np.int32(bits), n=np.int32(n))


def read_npz(path) -> dict:
    """The arrays of a .npz corpus file: d, bits, n, norms, and either
    packed_indices (flat uint8) or, in files of the older layout, indices
    (n x d uint8 codes)."""
    data = np.load(path)
    out = {"d": int(data["d"]), "bits": int(data["bits"]), "n": int(data["n"]),
           "norms": data["norms"]}
    if "packed_indices" in data:
        out["packed_indices"] = data["packed_indices"]
    else:
        out["indices"] = data["indices"]
    return out


def _pyarrow(feather_only: bool = False):
    try:
        import pyarrow.feather as feather
        if feather_only:
            return None, feather
        import pyarrow as pa
    except ImportError:
        raise ImportError("pyarrow is required for Arrow IPC format: pip install pyarrow")
    return pa, feather


def write_arrow(path, packed_rows, norms, d: int, bits: int, seed=None,
                **extra_metadata) -> None:
    """One record batch with columns norms (float32) and packed_indices
    (FixedSizeBinary of one packed row); d, bits, n, the optional seed and any
    extra key-value pairs as schema metadata (values as decimal strings)."""
    pa, feather = _pyarrow()
    rows = np.ascontiguousarray(packed_rows, np.uint8)
    n = int(rows.shape[0])
    rb = packed_nbytes(1, d, bits)
    if rows.size != n * rb:
        raise ValueError(f"packed rows size mismatch: got {rows.size}, expected {n * rb}")
    meta = {b"d": str(d).encode(), b"bits": str(bits).encode(), b"n": str(n).encode()}
    if seed is not None:
        meta[b"seed"] = str(seed).encode()
    for k, v in extra_metadata.items():
        meta[k.encode() if isinstance(k, str) else k] = str(v).encode()
    schema = pa.schema([pa.field("norms", pa.float32()),
                        pa.field("packed_indices", pa.binary(rb))], metadata=meta)
    col = pa.FixedSizeBinaryArray.from_buffers(pa.binary(rb), n,
                                               [None, pa.py_buffer(rows.tobytes())])
    table = pa.table({"norms": pa.array(np.asarray(norms, np.float32), type=pa.float32()),
                      "packed_indices": col}, schema=schema)
    feather.write_feather(table, path)


def read_arrow(path, memory_map: bool = False):
    """(packed rows (n x row_bytes uint8), norms (float32), n, d, bits) of a
    file written by write_arrow or by the reference's save_arrow."""
    _, feather = _pyarrow(feather_only=True)
    table = feather.read_table(path, memory_map=memory_map)
    meta = table.schema.metadata
    d, bits, n = int(meta[b"d"]), int(meta[b"bits"]), int(meta[b"n"])
    rb = packed_nbytes(1, d, bits)
    norms = table.column("norms").to_numpy().astype(np.float32)
    col = table.column("packed_indices").combine_chunks()
    if n == 0:
        return np.zeros((0, rb), np.uint8), norms, n, d, bits
    flat = np.frombuffer(col.buffers()[1], dtype=np.uint8)[col.offset * rb:(col.offset + n) * rb]
    return flat.reshape(n, rb).copy(), norms, n, d, bits

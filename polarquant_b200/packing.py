"""Host-side bit packing with the reference's byte layout.

Every supported width of remex/packing.py:18-127 is the same thing: an
MSB-first bitstream of ``bits``-bit codes (4-bit: high nibble first; 2-bit:
``v0<<6|v1<<4|v2<<2|v3``; 3-bit: 8 codes in 3 bytes; 1-bit: ``np.packbits``),
zero-padded to a whole group of codes (2 for 4-bit, 4 for 2-bit, 8 for 3- and
1-bit).  This module implements the layout once, generically, through
``np.unpackbits``/``np.packbits``.  The CUDA kernels read and write the same
stream.  These helpers serve the host side of the API (``.npz`` files,
``from_rows``); the hot path packs on the device.
"""

from __future__ import annotations

import numpy as np

SUPPORTED_BITS = (1, 2, 3, 4, 8)
_GROUP = {1: 8, 2: 4, 3: 8, 4: 2, 8: 1}


def _check(bits: int) -> None:
    if bits in (5, 6, 7):
        raise ValueError(
            f"Bit width {bits} is not supported. Use 1-4 or 8 bits. "
            f"5-7 bit widths offer negligible benefit over 4-bit or 8-bit.")
    if bits not in SUPPORTED_BITS:
        raise ValueError(f"Bit width {bits} is not supported. Use 1-4 or 8 bits.")


def packed_nbytes(n_values: int, d: int, bits: int) -> int:
    """Packed size of n_values vectors of dimension d (remex/packing.py:130-150)."""
    _check(bits)
    total = int(n_values) * int(d)
    g = _GROUP[bits]
    return (total + g - 1) // g * g * bits // 8


def pack(indices: np.ndarray, bits: int) -> np.ndarray:
    """Packs uint8 codes (any shape, flattened) into the MSB-first stream."""
    _check(bits)
    flat = np.asarray(indices).ravel().astype(np.uint8)
    if bits == 8:
        return flat.copy()
    g = _GROUP[bits]
    pad = (-len(flat)) % g
    if pad:
        flat = np.concatenate([flat, np.zeros(pad, np.uint8)])
    # (n, 8) bit matrix of each code, keep the low `bits` columns (MSB first).
    bitmat = np.unpackbits(flat[:, None], axis=1)[:, 8 - bits:]
    return np.packbits(bitmat.ravel())


def unpack(packed: np.ndarray, bits: int, n_values: int) -> np.ndarray:
    """Inverse of pack: the first n_values codes of the stream."""
    _check(bits)
    p = np.asarray(packed, dtype=np.uint8).ravel()
    if bits == 8:
        return p[:n_values].copy()
    n_avail = (len(p) * 8) // bits
    n = min(int(n_values), n_avail)
    stream = np.unpackbits(p)[: n * bits].reshape(n, bits)
    if bits < 8:
        stream = np.concatenate([np.zeros((n, 8 - bits), np.uint8), stream], axis=1)
    return np.packbits(stream, axis=1).ravel()


def pack_rows(indices: np.ndarray, bits: int) -> np.ndarray:
    """(n, d) codes -> (n, packed_nbytes(1, d, bits)) rows (PackedVectors layout)."""
    idx = np.asarray(indices, dtype=np.uint8)
    n, d = idx.shape
    rb = packed_nbytes(1, d, bits)
    if n == 0:
        return np.zeros((0, rb), np.uint8)
    g = _GROUP[bits]
    dp = (d + g - 1) // g * g
    if dp != d:
        idx = np.concatenate([idx, np.zeros((n, dp - d), np.uint8)], axis=1)
    return pack(idx, bits).reshape(n, rb)


def unpack_rows(rows: np.ndarray, bits: int, d: int) -> np.ndarray:
    """(n, row_bytes) packed rows -> (n, d) codes."""
    r = np.asarray(rows, dtype=np.uint8)
    n = r.shape[0]
    if n == 0:
        return np.zeros((0, d), np.uint8)
    rb = r.shape[1]
    per_row = (rb * 8) // bits
    return unpack(r.ravel(), bits, n * per_row).reshape(n, per_row)[:, :d].copy()

"""B200 drop-in for remex.core: Quantizer, CompressedVectors, PackedVectors.

Same constructors, method names, argument meanings, return types and errors
as remex/core.py.  The corpus lives on the GPU as packed rows (the reference's
row-padded byte layout with a 16-byte-aligned device stride) plus f32 norms;
encode, rotation, ADC scans, top-k and rerank run as kernels of the
polarquant_b200 CUDA library (include/polarquant_b200.h).  Host arrays
(``indices``, ``norms``, ``_packed``) are produced on demand.

Differences from the reference, by design:
  * ``search()`` is served by the ADC scan; the scores equal the cached f32
    path's (remex/core.py:534-580 vs :582-636, equal to rtol 1e-5 by the
    reference's own tests), so no n x d f32 ``_x_hat_rot`` cache is built and
    ``_x_hat_rot`` stays ``None``.
  * ``resident_bytes`` counts device bytes plus any host copies made.
  * Extra batch entry points (``search_adc_many``, ``search_twostage_many``)
    run many queries per launch.
"""

from __future__ import annotations

from typing import Iterable, Optional, Tuple

import numpy as np
import torch

from . import _lib
from .device import (alloc_rows, check_device_errors, ptr, require_cuda, row_stride,
                     rows_to_device, rows_to_host, stream_ptr, to_device_f32, topk_to_numpy,
                     workspace)
from .packing import pack, packed_nbytes, pack_rows, unpack, unpack_rows
from .pq_format import read_arrow, read_npz, write_arrow, write_npz
from .params import haar_rotation, lloyd_max_codebook, nested_codebooks

TOPK_MAX = _lib.PQ_TOPK_MAX
BATCH_MIN = 64       # queries per call from which the tensor-core path is used
BATCH_MIN_LARGE = 8  # ... on corpora of at least LARGE_ROWS rows
LARGE_ROWS = 1 << 20
SCAN_BYTES_MAX = 512 << 20  # scan traffic below which a batch stays on the scan

# Cost model of the two paths on corpora of LARGE_ROWS+ rows, from B200
# measurements at d=1536 (100M rows; 40M at 8 bits).  One batched call
# costs BATCH_FIXED_S + BATCH_QUERY_S per query + BATCH_S_PER_ROW_DIM[bits]
# per row and dimension for every 256 queries (int8 tensor cores at 2, 4 and
# 8 bits, fp16 at 1 and 3); the streaming scan moves row_bytes + 4 bytes per
# row and query at SCAN_BYTES_PER_S[bits] (byte tables; 8-bit rows over
# 1 KB take the per-coordinate scan).
BATCH_FIXED_S = 0.9e-3
BATCH_QUERY_S = 0.1e-3
BATCH_S_PER_ROW_DIM = {1: 6.2e-13, 2: 5.7e-13, 3: 6.2e-13, 4: 4.7e-13, 8: 8.3e-13}
SCAN_BYTES_PER_S = {1: 3.1e12, 2: 4.2e12, 3: 3.0e12, 4: 4.5e12, 8: 4.2e12}
SCAN_BYTES_PER_S_WIDE8 = 3.4e12


def use_tensor_cores(n: int, nq: int, k: int, row_bytes: Optional[int] = None,
                     bits: Optional[int] = None, d: Optional[int] = None) -> bool:
    """Whether a batch of nq queries runs the tensor-core ADC (pq_adc_batch).

    The batched kernels process 256 queries per tile whatever the batch size;
    at d=1536 4-bit one pass of them over the corpus costs about as much as
    4-5 single-query streaming scans, so on large corpora (where their fixed
    start-up cost is negligible) batches of 8 or more queries are faster on
    the tensor cores (pq_twostage's coarse stage keeps this fixed rule).
    With `row_bytes`, batches whose scans read at most SCAN_BYTES_MAX in all
    stay on the streaming scan: the batched call costs ~0.7 ms whatever the
    size (200 queries over 10k rows of 192 bytes: scan 0.37 ms, batched
    0.71 ms; over 100k rows: 2.3 ms against 0.77).  With `bits` and `d` as
    well, batches of fewer than BATCH_MIN queries on LARGE_ROWS+ rows take
    the path the cost model above rates faster: the crossover is about 3
    queries at 8 bits, 5 at 4, 10 at 2 and 16 at 1 bit."""
    if k > BATCH_MAX_K:
        return False
    if row_bytes is not None and n * nq * (row_bytes + 4) <= SCAN_BYTES_MAX:
        return False
    if nq >= BATCH_MIN:
        return True
    if n < LARGE_ROWS:
        return False
    if row_bytes is None or bits not in BATCH_S_PER_ROW_DIM or d is None:
        return nq >= BATCH_MIN_LARGE
    tiles = (nq + 255) // 256
    t_batch = (BATCH_FIXED_S + BATCH_QUERY_S * nq +
               BATCH_S_PER_ROW_DIM[bits] * float(n) * d * tiles)
    rate = (SCAN_BYTES_PER_S_WIDE8 if bits == 8 and row_bytes > 1024
            else SCAN_BYTES_PER_S[bits])
    t_scan = nq * float(n) * (row_bytes + 4) / rate
    return t_batch < t_scan


BATCH_MAX_K = 256    # largest k of the tensor-core path


# ---------------------------------------------------------------------------
# Device corpus storage shared by both containers
# ---------------------------------------------------------------------------

class _DeviceRows:
    """Packed rows (stride ldb) + f32 norms on one CUDA device."""

    __slots__ = ("buf", "norms", "n", "d", "bits", "ldb", "device", "_signs")

    def __init__(self, buf, norms, n, d, bits, ldb, device):
        self.buf, self.norms, self.n, self.d = buf, norms, int(n), int(d)
        self.bits, self.ldb, self.device = int(bits), int(ldb), device
        self._signs = None

    def sign_tier(self) -> "_DeviceRows":
        """The 1-bit Matryoshka level (the MSB of every code) as packed rows,
        made once by pq_repack and kept: the popcount scorer's input."""
        if self.bits == 1:
            return self
        if self._signs is None:
            self._signs = self.at_precision(1)
        return self._signs

    @classmethod
    def from_codes(cls, indices: np.ndarray, norms: np.ndarray, d: int, bits: int):
        dev = require_cuda()
        idx = np.ascontiguousarray(indices, dtype=np.uint8).reshape(-1, d)
        n = idx.shape[0]
        ldb = row_stride(d, bits)
        buf = alloc_rows(n, ldb, dev)
        nrm = to_device_f32(np.asarray(norms, np.float32).reshape(n), dev)
        if n:
            codes = torch.from_numpy(idx).to(dev)
            _lib.call("pq_pack_codes", ptr(codes), n, d, bits, ptr(buf), ldb, stream_ptr(dev))
        return cls(buf, nrm, n, d, bits, ldb, dev)

    @classmethod
    def from_rows(cls, rows: np.ndarray, norms: np.ndarray, d: int, bits: int):
        dev = require_cuda()
        ldb = row_stride(d, bits)
        rows = np.asarray(rows, dtype=np.uint8)
        n = rows.shape[0]
        buf = rows_to_device(rows, ldb, dev)
        nrm = to_device_f32(np.asarray(norms, np.float32).reshape(n), dev)
        return cls(buf, nrm, n, d, bits, ldb, dev)

    @property
    def row_bytes(self) -> int:
        return packed_nbytes(1, self.d, self.bits)

    def codes(self, shift: int = 0) -> torch.Tensor:
        out = torch.empty((self.n, self.d), dtype=torch.uint8, device=self.device)
        if self.n:
            _lib.call("pq_unpack_rows", ptr(self.buf), self.ldb, self.n, self.d, self.bits, shift,
                      ptr(out), stream_ptr(self.device))
        return out

    def codes_at(self, idx: np.ndarray, shift: int = 0) -> torch.Tensor:
        ii = torch.from_numpy(np.ascontiguousarray(idx, dtype=np.int64)).to(self.device)
        m = ii.numel()
        if m and (int(ii.min()) < 0 or int(ii.max()) >= self.n):
            raise IndexError("row index out of range")
        out = torch.empty((m, self.d), dtype=torch.uint8, device=self.device)
        if m:
            _lib.call("pq_unpack_at", ptr(self.buf), self.ldb, ptr(ii), m, self.d, self.bits,
                      shift, ptr(out), stream_ptr(self.device))
        return out

    def rows_host(self) -> np.ndarray:
        return rows_to_host(self.buf, self.n, self.ldb, self.row_bytes)

    def subset(self, idx) -> "_DeviceRows":
        ii = np.asarray(idx, dtype=np.int64).reshape(-1)
        if ii.size and (ii.min() < -self.n or ii.max() >= self.n):
            raise IndexError("row index out of range")
        ii = np.where(ii < 0, ii + self.n, ii)
        t = torch.from_numpy(ii).to(self.device)
        m = len(ii)
        buf = alloc_rows(m, self.ldb, self.device)
        if m:
            buf[: m * self.ldb].view(m, self.ldb).copy_(
                self.buf[: self.n * self.ldb].view(self.n, self.ldb).index_select(0, t))
        return _DeviceRows(buf, self.norms.index_select(0, t).contiguous(), m, self.d,
                           self.bits, self.ldb, self.device)

    def at_precision(self, target_bits: int) -> "_DeviceRows":
        ldb = row_stride(self.d, target_bits)
        buf = alloc_rows(self.n, ldb, self.device)
        if self.n:
            _lib.call("pq_repack", ptr(self.buf), self.ldb, self.n, self.d, self.bits,
                      target_bits, ptr(buf), ldb, stream_ptr(self.device))
        return _DeviceRows(buf, self.norms.clone(), self.n, self.d, target_bits, ldb,
                           self.device)

    @property
    def device_bytes(self) -> int:
        return self.buf.numel() + self.norms.numel() * 4


def _validate_bits(bits: int) -> None:
    if bits < 1 or bits > 8:
        raise ValueError(f"bits must be 1-4 or 8, got {bits}")
    if bits in (5, 6, 7):
        raise ValueError(
            f"bits={bits} is not supported. Use 1-4 or 8 bits. "
            f"5-7 bit widths offer negligible benefit over 4-bit or 8-bit.")


class CompressedVectors:
    """Encoded corpus (remex/core.py:10-117), resident on the GPU.

    ``indices`` (n, d) uint8 and ``norms`` (n,) f32 are host views produced
    on first access; the device holds packed rows and norms.
    """

    def __init__(self, indices: np.ndarray, norms: np.ndarray, d: int, bits: int):
        idx = np.asarray(indices, dtype=np.uint8)
        self._rows = None
        self._h_indices = idx.reshape(-1, int(d))
        self._h_norms = np.asarray(norms, dtype=np.float32).reshape(-1)
        self.d = int(d)
        self.bits = int(bits)
        self.n = self._h_indices.shape[0]
        self._x_hat_rot = None

    @classmethod
    def _from_device(cls, rows: _DeviceRows) -> "CompressedVectors":
        obj = cls.__new__(cls)
        obj._rows = rows
        obj._h_indices = None
        obj._h_norms = None
        obj.d, obj.bits, obj.n = rows.d, rows.bits, rows.n
        obj._x_hat_rot = None
        return obj

    # -- device side ------------------------------------------------------
    def _device(self) -> _DeviceRows:
        if self._rows is None:
            self._rows = _DeviceRows.from_codes(self._h_indices, self._h_norms, self.d, self.bits)
        return self._rows

    # -- host views -------------------------------------------------------
    @property
    def indices(self) -> np.ndarray:
        if self._h_indices is None:
            self._h_indices = self._rows.codes().cpu().numpy()
        return self._h_indices

    @indices.setter
    def indices(self, value) -> None:
        self._h_indices = np.asarray(value, dtype=np.uint8)
        self.n = self._h_indices.shape[0]
        self._rows = None

    @property
    def norms(self) -> np.ndarray:
        if self._h_norms is None:
            self._h_norms = self._rows.norms.cpu().numpy()
        return self._h_norms

    @norms.setter
    def norms(self, value) -> None:
        self._h_norms = np.asarray(value, dtype=np.float32)
        self._rows = None

    def subset(self, idx: np.ndarray) -> "CompressedVectors":
        return CompressedVectors._from_device(self._device().subset(idx))

    @property
    def nbytes(self) -> int:
        return packed_nbytes(self.n, self.d, self.bits) + self.n * 4

    @property
    def nbytes_unpacked(self) -> int:
        return self.n * self.d + self.n * 4

    @property
    def compression_ratio(self) -> float:
        return (self.n * self.d * 4) / self.nbytes

    @property
    def resident_bytes(self) -> int:
        total = 0 if self._rows is None else self._rows.device_bytes
        if self._h_indices is not None:
            total += self._h_indices.nbytes
        if self._h_norms is not None:
            total += self._h_norms.nbytes
        return total

    def drop_cache(self) -> None:
        self._x_hat_rot = None

    def save(self, path: str) -> None:
        """Same .npz keys and arrays as remex/core.py:64-74."""
        if self._rows is not None and (self.d * self.bits) % 8 == 0:
            flat = self._rows.rows_host().ravel()
        else:
            flat = pack(self.indices.ravel(), self.bits)
        write_npz(path, flat, self.norms, self.d, self.bits, self.n)

    @classmethod
    def load(cls, path: str) -> "CompressedVectors":
        """remex/core.py:76-91 (also reads the legacy unpacked 'indices' key)."""
        data = read_npz(path)
        d, bits, n = data["d"], data["bits"], data["n"]
        norms = data["norms"]
        if "packed_indices" in data:
            flat = data["packed_indices"]
            if (d * bits) % 8 == 0:
                rows = flat[: n * packed_nbytes(1, d, bits)].reshape(n, -1) if n else \
                    np.zeros((0, packed_nbytes(1, d, bits)), np.uint8)
                return cls._from_device(_DeviceRows.from_rows(rows, norms, d, bits))
            return cls(unpack(flat, bits, n * d).reshape(n, d), norms, d, bits)
        return cls(data["indices"], norms, d, bits)

    def save_arrow(self, path: str, seed: Optional[int] = None, **extra_metadata):
        PackedVectors.from_compressed(self).save_arrow(path, seed=seed, **extra_metadata)

    @classmethod
    def load_arrow(cls, path: str) -> "CompressedVectors":
        return PackedVectors.load_arrow(path).to_compressed()


class PackedVectors:
    """Packed storage (remex/core.py:120-439), resident on the GPU."""

    def __init__(self, packed: np.ndarray, norms: np.ndarray, n: int, d: int, bits: int):
        self._rows = _DeviceRows.from_rows(np.asarray(packed, np.uint8).reshape(int(n), -1),
                                           norms, d, bits)
        self._init_meta()

    def _init_meta(self) -> None:
        r = self._rows
        self.n, self.d, self.bits = r.n, r.d, r.bits
        self._row_bytes = packed_nbytes(1, self.d, self.bits)
        self._row_aligned = (self.d * self.bits) % 8 == 0
        self._h_packed = None
        self._h_norms = None

    @classmethod
    def _wrap(cls, rows: _DeviceRows) -> "PackedVectors":
        obj = cls.__new__(cls)
        obj._rows = rows
        obj._init_meta()
        return obj

    def _device(self) -> _DeviceRows:
        return self._rows

    @property
    def _packed(self) -> np.ndarray:
        if self._h_packed is None:
            self._h_packed = self._rows.rows_host()
        return self._h_packed

    @property
    def norms(self) -> np.ndarray:
        if self._h_norms is None:
            self._h_norms = self._rows.norms.cpu().numpy()
        return self._h_norms

    def unpack_rows(self, start: int, end: int) -> np.ndarray:
        start, end = max(0, int(start)), min(self.n, int(end))
        if end <= start:
            return np.zeros((0, self.d), np.uint8)
        return self._rows.codes_at(np.arange(start, end)).cpu().numpy()

    def unpack_at(self, idx: np.ndarray) -> np.ndarray:
        idx = np.asarray(idx)
        if idx.ndim == 0:
            idx = idx.reshape(1)
        return self._rows.codes_at(idx).cpu().numpy()

    @classmethod
    def from_compressed(cls, compressed: CompressedVectors) -> "PackedVectors":
        r = compressed._device()
        return cls._wrap(_DeviceRows(r.buf.clone(), r.norms.clone(), r.n, r.d, r.bits, r.ldb,
                                     r.device))

    @classmethod
    def from_rows(cls, rows: Iterable, norms: np.ndarray, d: int, bits: int) -> "PackedVectors":
        lst = [np.frombuffer(r, dtype=np.uint8) if isinstance(r, (bytes, bytearray))
               else np.asarray(r, dtype=np.uint8) for r in rows]
        packed = np.stack(lst) if lst else np.zeros((0, packed_nbytes(1, d, bits)), np.uint8)
        return cls(packed, np.asarray(norms, dtype=np.float32), len(lst), d, bits)

    def at_precision(self, target_bits: int) -> "PackedVectors":
        if target_bits < 1 or target_bits > self.bits:
            raise ValueError(f"target_bits must be 1-{self.bits}, got {target_bits}")
        if target_bits == self.bits:
            return self
        return PackedVectors._wrap(self._rows.at_precision(target_bits))

    def to_compressed(self) -> CompressedVectors:
        r = self._rows
        return CompressedVectors._from_device(
            _DeviceRows(r.buf.clone(), r.norms.clone(), r.n, r.d, r.bits, r.ldb, r.device))

    def subset(self, idx: np.ndarray) -> "PackedVectors":
        return PackedVectors._wrap(self._rows.subset(idx))

    @property
    def nbytes(self) -> int:
        return self.n * self._row_bytes + self.n * 4

    @property
    def resident_bytes(self) -> int:
        total = self._rows.device_bytes
        if self._h_packed is not None:
            total += self._h_packed.nbytes
        if self._h_norms is not None:
            total += self._h_norms.nbytes
        return total

    @property
    def compression_ratio(self) -> float:
        return (self.n * self.d * 4) / self.nbytes

    def save(self, path: str) -> None:
        """remex/core.py:326-335: the padded rows back to back."""
        write_npz(path, self._packed.ravel(), self.norms, self.d, self.bits, self.n)

    @classmethod
    def load(cls, path: str) -> "PackedVectors":
        """remex/core.py:337-347."""
        data = read_npz(path)
        d, bits, n = data["d"], data["bits"], data["n"]
        rb = packed_nbytes(1, d, bits)
        return cls(data["packed_indices"].reshape(n, rb), data["norms"], n, d, bits)

    def save_arrow(self, path: str, seed: Optional[int] = None, **extra_metadata):
        """Arrow IPC (Feather v2) layout of remex/core.py:349-401."""
        write_arrow(path, self._packed, self.norms, self.d, self.bits, seed, **extra_metadata)

    @classmethod
    def load_arrow(cls, path: str, memory_map: bool = False) -> "PackedVectors":
        """remex/core.py:403-439."""
        rows, norms, n, d, bits = read_arrow(path, memory_map=memory_map)
        return cls(rows, norms, n, d, bits)


# ---------------------------------------------------------------------------
# Quantizer
# ---------------------------------------------------------------------------

class _DeviceParams:
    """Per-device copies of the Quantizer's tables."""

    def __init__(self, q: "Quantizer", dev: torch.device):
        self.device = dev
        self.R = torch.from_numpy(np.ascontiguousarray(q.R)).to(dev)
        self.RT = None
        self.boundaries = torch.from_numpy(np.ascontiguousarray(q.boundaries)).to(dev)
        self.cent = {p: torch.from_numpy(np.ascontiguousarray(t)).to(dev)
                     for p, t in q._nested.items()}
        self.cent[q.bits] = torch.from_numpy(np.ascontiguousarray(q.centroids)).to(dev)


class Quantizer:
    """Drop-in for remex.Quantizer (remex/core.py:442-901) on a B200."""

    def __init__(self, d: int, bits: int = 4, seed: int = 42):
        _validate_bits(bits)
        self.d = d
        self.bits = bits
        self.seed = seed
        self.R = haar_rotation(d, seed)
        self.boundaries, self.centroids = lloyd_max_codebook(d, bits)
        self._nested = nested_codebooks(d, bits)
        self._dev = {}

    # -- device state -------------------------------------------------------
    def _params(self, dev: Optional[torch.device] = None) -> _DeviceParams:
        dev = dev or require_cuda()
        key = dev.index
        if key not in self._dev:
            self._dev[key] = _DeviceParams(self, dev)
        return self._dev[key]

    def _resolve_centroids(self, compressed, precision: Optional[int]) -> np.ndarray:
        """remex/core.py:882-892."""
        if precision is None:
            return self.centroids
        if precision < 1 or precision > self.bits:
            raise ValueError(f"precision must be 1-{self.bits}, got {precision}")
        return self._nested[precision]

    def _level(self, precision: Optional[int]) -> int:
        self._resolve_centroids(None, precision)
        return self.bits if precision is None else int(precision)

    def _rotate(self, X, dev: torch.device) -> torch.Tensor:
        Xd = to_device_f32(X, dev)
        if Xd.dim() == 1:
            Xd = Xd.unsqueeze(0)
        if Xd.shape[1] != self.d:
            raise ValueError(f"Expected d={self.d}, got {Xd.shape[1]}")
        Y = torch.empty_like(Xd)
        _lib.call("pq_rotate", ptr(Xd), Xd.shape[0], self.d, ptr(self._params(dev).R), ptr(Y),
                  stream_ptr(dev))
        return Y

    @staticmethod
    def _rows_of(compressed) -> _DeviceRows:
        if isinstance(compressed, (CompressedVectors, PackedVectors)):
            return compressed._device()
        raise TypeError(f"expected CompressedVectors or PackedVectors, got "
                        f"{type(compressed).__name__}")

    def _check_corpus(self, rows: _DeviceRows) -> None:
        if rows.d != self.d or rows.bits != self.bits:
            raise ValueError(f"corpus (d={rows.d}, bits={rows.bits}) does not match quantizer "
                             f"(d={self.d}, bits={self.bits})")

    # -- encode ---------------------------------------------------------------
    def encode(self, X) -> CompressedVectors:
        """Quantize (n, d) vectors (remex/core.py:484-511) on the GPU."""
        from .encode import encode_rows
        return CompressedVectors._from_device(encode_rows(self, X))

    def decode(self, compressed, precision: Optional[int] = None) -> np.ndarray:
        """remex/core.py:513-532."""
        from .encode import decode_rows
        p = self._level(precision)
        return decode_rows(self, self._rows_of(compressed), p).cpu().numpy()

    def mse(self, X, precision: Optional[int] = None) -> float:
        """remex/core.py:780-786."""
        comp = self.encode(X)
        X_hat = self.decode(comp, precision=precision)
        Xh = np.asarray(X, np.float32)
        if Xh.ndim == 1:
            Xh = Xh[None]
        return float(np.mean(np.sum((Xh - X_hat) ** 2, axis=1)))

    # -- search -------------------------------------------------------------
    def _scan(self, rows: _DeviceRows, qrot: torch.Tensor, k: int, p: int,
              force: Optional[str] = None):
        """Top-min(k, n) ADC results for each row of qrot, on the device.

        Batches chosen by use_tensor_cores() (k <= BATCH_MAX_K) run on the
        tensor cores (pq_adc_batch); smaller ones stream the corpus once per
        query (pq_adc_scan).  `force` ("batch" / "scan") selects a path."""
        dev = rows.device
        nq = qrot.shape[0]
        K = min(int(k), rows.n)
        if K <= 0 or nq == 0:
            return (torch.empty((nq, 0), dtype=torch.float32, device=dev),
                    torch.empty((nq, 0), dtype=torch.int64, device=dev))
        cent = self._params(dev).cent[p]
        batched = (use_tensor_cores(rows.n, nq, K, rows.row_bytes, rows.bits, rows.d)
                   if force is None
                   else force == "batch")
        fn = "pq_adc_batch" if batched else "pq_adc_scan"
        ws = workspace(_lib.query(fn + "_workspace_bytes", rows.n, rows.d, nq, K), dev)
        out_s = torch.empty((nq, K), dtype=torch.float32, device=dev)
        out_i = torch.empty((nq, K), dtype=torch.int64, device=dev)
        _lib.call(fn, ptr(rows.buf), rows.ldb, ptr(rows.norms), rows.n, rows.d,
                  rows.bits, p, ptr(qrot), nq, ptr(cent), K, 0, ptr(out_s), ptr(out_i),
                  ptr(ws), ws.numel(), stream_ptr(dev))
        return out_s, out_i

    def _twostage(self, rows: _DeviceRows, qrot: torch.Tensor, k: int, candidates: int,
                  cp: int):
        dev = rows.device
        nq = qrot.shape[0]
        ck = min(int(candidates), rows.n)
        if ck <= 0 or nq == 0 or k <= 0:
            return (torch.empty((nq, 0), dtype=torch.float32, device=dev),
                    torch.empty((nq, 0), dtype=torch.int64, device=dev))
        if ck >= rows.n:
            # Every row is a candidate: stage 2 alone decides (remex/core.py:701-702).
            return self._scan(rows, qrot, min(k, rows.n), self.bits)
        K = min(int(k), ck)
        pr = self._params(dev)
        ws = workspace(_lib.query("pq_twostage_workspace_bytes", rows.n, rows.d, nq, ck), dev)
        out_s = torch.empty((nq, K), dtype=torch.float32, device=dev)
        out_i = torch.empty((nq, K), dtype=torch.int64, device=dev)
        _lib.call("pq_twostage", ptr(rows.buf), rows.ldb, ptr(rows.norms), rows.n, rows.d,
                  rows.bits, cp, ptr(qrot), nq, ptr(pr.cent[cp]), ptr(pr.cent[self.bits]), ck,
                  K, 0, ptr(out_s), ptr(out_i), ptr(ws), ws.numel(), stream_ptr(dev))
        return out_s, out_i

    def search(self, compressed, query, k: int = 10, precision: Optional[int] = None):
        """remex/core.py:534-580 (scores via the ADC scan)."""
        if isinstance(compressed, PackedVectors):
            raise TypeError(
                "PackedVectors does not support cached search(). "
                "Use search_adc() or search_twostage(), or convert "
                "with packed.to_compressed() first.")
        return self.search_adc(compressed, query, k=k, precision=precision)

    def search_adc(self, compressed, query, k: int = 10, precision: Optional[int] = None,
                   chunk_size: int = 4096):
        """remex/core.py:582-636.  chunk_size is accepted; results do not depend on it."""
        rows = self._rows_of(compressed)
        self._check_corpus(rows)
        p = self._level(precision)
        qrot = self._rotate(query, rows.device)
        s, i = self._scan(rows, qrot, k, p)
        ids, sc = topk_to_numpy(s, i)
        return ids[0], sc[0]

    def search_adc_many(self, compressed, queries, k: int = 10,
                        precision: Optional[int] = None):
        """search_adc for each row of `queries`; returns (nq, min(k, n)) arrays."""
        rows = self._rows_of(compressed)
        self._check_corpus(rows)
        p = self._level(precision)
        s, i = self._scan(rows, self._rotate(queries, rows.device), k, p)
        return topk_to_numpy(s, i)

    def search_twostage(self, compressed, query, k: int = 10, candidates: int = 500,
                        coarse_precision: Optional[int] = None, coarse_chunk_size: int = 4096):
        """remex/core.py:638-719."""
        ids, sc = self.search_twostage_many(compressed, query, k=k, candidates=candidates,
                                            coarse_precision=coarse_precision)
        return ids[0], sc[0]

    def search_twostage_many(self, compressed, queries, k: int = 10, candidates: int = 500,
                             coarse_precision: Optional[int] = None):
        if coarse_precision is None:
            coarse_precision = max(1, self.bits - 2)
        cp = self._level(coarse_precision)
        rows = self._rows_of(compressed)
        self._check_corpus(rows)
        s, i = self._twostage(rows, self._rotate(queries, rows.device), k, candidates, cp)
        return topk_to_numpy(s, i)

    # -- 1-bit popcount coarse scorer (no method of the reference; the coarse
    # tier its docs recommend, bench/RESULTS.md:153-161) ------------------------
    def _popcount(self, rows: _DeviceRows, qrot: torch.Tensor, k: int,
                  candidates: Optional[int] = None):
        dev = rows.device
        nq = qrot.shape[0]
        K = min(int(k), rows.n)
        C = None if candidates is None else min(int(candidates), rows.n)
        if K <= 0 or nq == 0 or (C is not None and C <= 0):
            return (torch.empty((nq, 0), dtype=torch.float32, device=dev),
                    torch.empty((nq, 0), dtype=torch.int64, device=dev))
        if C is not None and C >= rows.n:
            # Every row is a candidate: the full-precision stage alone decides.
            return self._scan(rows, qrot, K, self.bits)
        if C is not None:
            K = min(K, C)
        width = K if C is None else C
        if width > TOPK_MAX:
            raise ValueError(f"the popcount scorer keeps at most {TOPK_MAX} results per query "
                             f"(asked for {width})")
        sg = rows.sign_tier()
        ws = workspace(_lib.query("pq_hamming_workspace_bytes", rows.n, nq, width), dev)
        out_s = torch.empty((nq, K), dtype=torch.float32, device=dev)
        out_i = torch.empty((nq, K), dtype=torch.int64, device=dev)
        if C is None:
            _lib.call("pq_hamming_scan", ptr(sg.buf), sg.ldb, rows.n, rows.d, ptr(qrot), nq, K,
                      0, ptr(out_s), ptr(out_i), ptr(ws), ws.numel(), stream_ptr(dev))
        else:
            cent = self._params(dev).cent[self.bits]
            _lib.call("pq_hamming_twostage", ptr(sg.buf), sg.ldb, ptr(rows.buf), rows.ldb,
                      ptr(rows.norms), rows.n, rows.d, rows.bits, ptr(qrot), nq, ptr(cent), C, K,
                      0, ptr(out_s), ptr(out_i), ptr(ws), ws.numel(), stream_ptr(dev))
        return out_s, out_i

    def search_popcount_many(self, compressed, queries, k: int = 10):
        """Coarse search by 1-bit sign agreement: score = d - 2 * popcount(
        query_signs XOR row_signs), the row signs being the MSBs of its codes
        and query bit j being q_rot[j] > 0; (nq, min(k, n)) ids and scores,
        score descending, ties by row ascending.  k <= 2048."""
        rows = self._rows_of(compressed)
        self._check_corpus(rows)
        s, i = self._popcount(rows, self._rotate(queries, rows.device), k)
        return topk_to_numpy(s, i)

    def search_popcount(self, compressed, query, k: int = 10):
        ids, sc = self.search_popcount_many(compressed, query, k=k)
        return ids[0], sc[0]

    def search_twostage_popcount_many(self, compressed, queries, k: int = 10,
                                      candidates: int = 500):
        """Two-stage search with the popcount coarse scorer: the top
        `candidates` rows by sign agreement (ties by row), rescored at full
        precision exactly as search_twostage's second stage
        (remex/core.py:706-719); (nq, min(k, candidates, n)) results.
        candidates <= 2048 unless it covers the whole corpus."""
        rows = self._rows_of(compressed)
        self._check_corpus(rows)
        s, i = self._popcount(rows, self._rotate(queries, rows.device), k, candidates)
        return topk_to_numpy(s, i)

    def search_twostage_popcount(self, compressed, query, k: int = 10, candidates: int = 500):
        ids, sc = self.search_twostage_popcount_many(compressed, query, k=k,
                                                     candidates=candidates)
        return ids[0], sc[0]

    def search_batch(self, compressed, queries, k: int = 10, precision: Optional[int] = None):
        """remex/core.py:721-778: (n_queries, min(k, n)) indices and scores."""
        if isinstance(compressed, PackedVectors):
            raise TypeError(
                "PackedVectors does not support cached search_batch(). "
                "Use search_adc() or search_twostage(), or convert "
                "with packed.to_compressed() first.")
        Q = np.asarray(queries, dtype=np.float32) if not isinstance(queries, torch.Tensor) \
            else queries
        if Q.ndim == 1:
            Q = Q[None]
        return self.search_adc_many(compressed, Q, k=k, precision=precision)

"""B200 drop-in for remex.ivf.IVFCoarseIndex (remex/ivf.py:65-472).

Same constructor, attributes, methods, results and errors.  The index is
built on the GPU (cell ids by ivf_cell_ids_kernel; the CSR layout by the
library's stable counting sort, pq_ivf_build_csr) and kept there; the query
path (query cell, Hamming-ranked probe cells, gather-ADC over the probed
cells' rows, top-C, full-precision rerank) runs as one library call per
query batch (pq_ivf_search).  Host views
(``cell_ids``, ``sorted_idx``, ``cell_offsets``) are produced on demand.

LSH projections are summed exactly (f64) on the device; the reference sums
them with an f32 sgemm, so a row whose projection lies within f32 rounding of
zero can land in the neighbouring cell.  ``probe_cells`` and the host helpers
follow remex/ivf.py:252-295 exactly.
"""

from __future__ import annotations

from typing import Optional

import numpy as np
import torch

from . import _lib
from .core import CompressedVectors, PackedVectors, Quantizer
from .device import ptr, stream_ptr, to_device_f32, workspace

_VALID_MODES = ("lsh", "rotated_prefix")


class IVFCoarseIndex:
    """Inverted-file index over the coarse Matryoshka tier, resident on the GPU."""

    def __init__(self, quantizer: Quantizer, compressed, n_bits: int, mode: str = "lsh",
                 seed: int = 0):
        if n_bits < 1 or n_bits > 16:
            raise ValueError(f"n_bits must be 1-16, got {n_bits}")
        if mode not in _VALID_MODES:
            raise ValueError(f"mode must be one of {_VALID_MODES}, got {mode!r}")
        if mode == "rotated_prefix" and n_bits > quantizer.d:
            raise ValueError(f"n_bits={n_bits} exceeds quantizer.d={quantizer.d} "
                             f"for rotated_prefix mode")
        if not isinstance(compressed, (CompressedVectors, PackedVectors)):
            raise TypeError(f"compressed must be CompressedVectors or PackedVectors, "
                            f"got {type(compressed).__name__}")
        self.quantizer = quantizer
        self.compressed = compressed
        self.n_bits = int(n_bits)
        self.n_cells = 1 << int(n_bits)
        self.mode = mode
        self.seed = int(seed)
        self.n = compressed.n
        self.d = quantizer.d
        if mode == "lsh":
            rng = np.random.default_rng(seed)
            self.hyperplanes = rng.standard_normal((self.n_bits, self.d)).astype(np.float32)
        else:
            self.hyperplanes = None
        self._build()

    # -- build ------------------------------------------------------------------
    def _build(self) -> None:
        rows = self.compressed._device()
        dev = rows.device
        self._dev = dev
        self._H = None if self.hyperplanes is None else \
            torch.from_numpy(self.hyperplanes).to(dev)
        cells = torch.empty(rows.n, dtype=torch.int16, device=dev)
        st = stream_ptr(dev)
        if rows.n:
            _lib.call("pq_ivf_cell_ids", ptr(rows.buf), rows.ldb, rows.n, rows.d, rows.bits,
                      self.n_bits, 0 if self.mode == "lsh" else 1, ptr(self._H), ptr(cells), st)
        # CSR: rows grouped by cell, ascending row order within a cell
        # (remex/ivf.py:216-224: stable argsort + bincount offsets), by the
        # library's stable counting sort, together with a copy of the packed
        # rows and norms in CSR order, so the query path reads each probed
        # cell as one contiguous run instead of gathering rows through
        # sorted_idx (one more device copy of the corpus).
        self._sorted = torch.empty(rows.n, dtype=torch.int64, device=dev)
        self._offsets = torch.empty(self.n_cells + 1, dtype=torch.int64, device=dev)
        if rows.n:
            self._cell_rows = torch.zeros(rows.n * rows.ldb + 64, dtype=torch.uint8, device=dev)
            self._cell_norms = torch.empty(rows.n, dtype=torch.float32, device=dev)
        else:
            self._cell_rows = self._cell_norms = None
        ws = workspace(_lib.query("pq_ivf_csr_workspace_bytes", rows.n, self.n_bits), dev)
        _lib.call("pq_ivf_build_csr", ptr(cells), rows.n, self.n_bits, ptr(self._sorted),
                  ptr(self._offsets), ptr(rows.buf), rows.ldb, ptr(rows.norms),
                  ptr(self._cell_rows), ptr(self._cell_norms), ptr(ws), ws.numel(), st)
        self._cells = cells
        self._h_cells = self._h_sorted = self._h_offsets = None

    # -- host views (remex/ivf.py:81-89 attributes) ---------------------------
    @property
    def cell_ids(self) -> np.ndarray:
        if self._h_cells is None:
            self._h_cells = self._cells.cpu().numpy().view(np.uint16)
        return self._h_cells

    @property
    def sorted_idx(self) -> np.ndarray:
        if self._h_sorted is None:
            self._h_sorted = self._sorted.cpu().numpy()
        return self._h_sorted

    @property
    def cell_offsets(self) -> np.ndarray:
        if self._h_offsets is None:
            self._h_offsets = self._offsets.cpu().numpy()
        return self._h_offsets

    # -- query helpers (host, exactly as remex/ivf.py:230-295) ------------------
    def _query_cell_from_rot(self, q_rot: np.ndarray) -> int:
        if self.mode == "rotated_prefix":
            sb = (q_rot[: self.n_bits] > 0).astype(np.uint8)
        else:
            sb = ((self.hyperplanes.astype(np.float64) @ q_rot.astype(np.float64)) > 0)
        cid = 0
        for b in range(self.n_bits):
            cid |= int(sb[b]) << b
        return cid

    def query_cell(self, query) -> int:
        q_rot = self.quantizer._rotate(np.asarray(query, np.float32), self._dev)[0]
        return self._query_cell_from_rot(q_rot.cpu().numpy())

    def probe_cells(self, query_cell: int, nprobe: int) -> np.ndarray:
        if nprobe <= 0:
            return np.empty(0, dtype=np.int64)
        if nprobe >= self.n_cells:
            return np.arange(self.n_cells, dtype=np.int64)
        cells = np.arange(self.n_cells, dtype=np.uint32)
        x = cells ^ np.uint32(query_cell)
        hd = np.zeros(self.n_cells, dtype=np.uint8)
        for b in range(self.n_bits):
            hd += ((x >> np.uint32(b)) & 1).astype(np.uint8)
        order = np.lexsort((cells, hd))[:nprobe]
        return cells[order].astype(np.int64)

    def candidate_indices(self, query_cell: int, nprobe: int) -> np.ndarray:
        cells = self.probe_cells(query_cell, nprobe)
        if len(cells) == 0:
            return np.empty(0, dtype=np.int64)
        off, srt = self.cell_offsets, self.sorted_idx
        return np.concatenate([srt[off[c]:off[c + 1]] for c in cells])

    def candidate_count(self, query, nprobe: int) -> int:
        cells = self.probe_cells(self.query_cell(query), nprobe)
        if len(cells) == 0:
            return 0
        return int(np.diff(self.cell_offsets)[cells].sum())

    # -- search (device) ---------------------------------------------------------
    def _run(self, queries, k: int, nprobe: int, precision: int, rerank: bool,
             candidates: int):
        q = self.quantizer
        rows = self.compressed._device()
        dev = rows.device
        Qr = q._rotate(queries, dev)
        nq = Qr.shape[0]
        nprobe = int(min(max(nprobe, 0), self.n_cells))
        if nprobe <= 0 or rows.n == 0 or nq == 0 or candidates <= 0 or k <= 0:
            # No probed cell, no rows or nothing asked for: empty results, as
            # remex/ivf.py:301-436 returns for an empty candidate set.
            return (np.full((nq, 0), -1, np.int64), np.zeros((nq, 0), np.float32))
        # More than the fused limit (TOPK_MAX) candidates take the library's
        # sort-based path; the result has min(k, candidates) columns either way.
        C = int(min(candidates, rows.n))
        K = int(min(k, C))
        # Row groups per query: about 8k probed rows each (at least one).
        probed = nprobe * (rows.n / self.n_cells)
        splits = int(min(64, max(1, round(probed / 8192))))
        pr = q._params(dev)
        ws = workspace(_lib.query("pq_ivf_workspace_bytes", rows.n, nq, nprobe, splits, C), dev)
        out_s = torch.empty((nq, K), dtype=torch.float32, device=dev)
        out_i = torch.empty((nq, K), dtype=torch.int64, device=dev)
        _lib.call("pq_ivf_search", ptr(rows.buf), rows.ldb, ptr(rows.norms), rows.n, rows.d,
                  rows.bits, precision, ptr(Qr), nq, ptr(pr.cent[precision]),
                  ptr(pr.cent[q.bits]), self.n_bits, 0 if self.mode == "lsh" else 1,
                  ptr(self._H), ptr(self._sorted), ptr(self._offsets), ptr(self._cell_rows),
                  ptr(self._cell_norms), nprobe, splits, C, K,
                  1 if rerank else 0, ptr(out_s), ptr(out_i), ptr(ws), ws.numel(),
                  stream_ptr(dev))
        return out_i.cpu().numpy(), out_s.cpu().numpy()

    @staticmethod
    def _trim(ids, sc):
        keep = ids >= 0
        return ids[keep].astype(np.int64), sc[keep]

    def search_coarse_many(self, queries, k: int = 500, nprobe: int = 1,
                           precision: Optional[int] = None):
        """(nq, min(k, C)) coarse results; slots past a query's candidates hold id -1."""
        p = self.quantizer._level(precision)
        return self._run(queries, k, nprobe, p, False, max(int(k), 1))

    def search_coarse(self, query, k: int = 500, nprobe: int = 1,
                      precision: Optional[int] = None, chunk_size: int = 4096):
        """remex/ivf.py:301-374."""
        ids, sc = self.search_coarse_many(np.asarray(query, np.float32)[None], k=k,
                                          nprobe=nprobe, precision=precision)
        return self._trim(ids[0], sc[0])

    def search_twostage_many(self, queries, k: int = 10, candidates: int = 500,
                             nprobe: int = 1, coarse_precision: Optional[int] = None):
        if coarse_precision is None:
            coarse_precision = max(1, self.quantizer.bits - 2)
        cp = self.quantizer._level(coarse_precision)
        return self._run(queries, k, nprobe, cp, True, candidates)

    def search_twostage(self, query, k: int = 10, candidates: int = 500, nprobe: int = 1,
                        coarse_precision: Optional[int] = None, coarse_chunk_size: int = 4096):
        """remex/ivf.py:376-436."""
        ids, sc = self.search_twostage_many(np.asarray(query, np.float32)[None], k=k,
                                            candidates=candidates, nprobe=nprobe,
                                            coarse_precision=coarse_precision)
        return self._trim(ids[0], sc[0])

    # -- diagnostics (remex/ivf.py:442-472) -------------------------------------
    @property
    def index_nbytes(self) -> int:
        total = self.n * 2 + self.n * 8 + (self.n_cells + 1) * 8
        if self.hyperplanes is not None:
            total += self.hyperplanes.nbytes
        return int(total)

    @property
    def avg_cell_size(self) -> float:
        return self.n / self.n_cells if self.n_cells > 0 else 0.0

    def cell_size_stats(self) -> dict:
        sizes = np.diff(self.cell_offsets)
        nonempty = sizes[sizes > 0]
        return {
            "n_cells": int(self.n_cells),
            "nonempty_cells": int((sizes > 0).sum()),
            "min": int(sizes.min()),
            "max": int(sizes.max()),
            "mean": float(sizes.mean()),
            "std": float(sizes.std()),
            "median": float(np.median(sizes)),
            "p95": float(np.percentile(sizes, 95)),
            "nonempty_min": int(nonempty.min()) if len(nonempty) else 0,
        }

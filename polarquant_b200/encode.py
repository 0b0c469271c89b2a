"""Device encode and decode for the Quantizer (remex/core.py:484-532)."""

from __future__ import annotations

import ctypes

import numpy as np
import torch

from . import _lib
from .device import alloc_rows, ptr, require_cuda, row_stride, stream_ptr, to_device_f32, workspace


def _planes(q, dev, transposed: bool = False) -> torch.Tensor:
    pr = q._params(dev)
    attr = "planes_T" if transposed else "planes"
    pl = getattr(pr, attr, None)
    if pl is None:
        nb = _lib.query("pq_rotation_planes_bytes", q.d)
        pl = torch.empty(nb, dtype=torch.uint8, device=dev)
        src = rt(q, dev) if transposed else pr.R
        _lib.call("pq_prepare_rotation", ptr(src), q.d, ptr(pl), nb, stream_ptr(dev))
        setattr(pr, attr, pl)
    return pl


def rt(q, dev) -> torch.Tensor:
    pr = q._params(dev)
    if getattr(pr, "RT", None) is None:
        pr.RT = torch.from_numpy(np.ascontiguousarray(q.R.T)).to(dev)
    return pr.RT


def encode_rows(q, X):
    """(n, d) float array or tensor -> _DeviceRows of packed codes + norms."""
    from .core import _DeviceRows
    dev = require_cuda()
    if isinstance(X, torch.Tensor) and X.is_cuda:
        dev = X.device
    Xd = to_device_f32(X, dev)
    if Xd.dim() == 1:
        Xd = Xd.unsqueeze(0)
    if Xd.dim() != 2 or Xd.shape[1] != q.d:
        raise ValueError(f"Expected d={q.d}, got {Xd.shape[-1] if Xd.dim() else 0}")
    n = Xd.shape[0]
    ldb = row_stride(q.d, q.bits)
    buf = alloc_rows(n, ldb, dev)
    norms = torch.empty(n, dtype=torch.float32, device=dev)
    if n:
        pl = _planes(q, dev)
        pr = q._params(dev)
        ws = workspace(_lib.query("pq_encode_workspace_bytes", n, q.d), dev)
        _lib.call("pq_encode", ptr(Xd), n, q.d, ptr(pr.R), ptr(pl), ptr(pr.boundaries), q.bits,
                  ptr(buf), ldb, ptr(norms), ptr(ws), ws.numel(), stream_ptr(dev))
    return _DeviceRows(buf, norms, n, q.d, q.bits, ldb, dev)


def decode_rows(q, rows, precision: int) -> torch.Tensor:
    """_DeviceRows -> (n, d) f32 reconstruction on the device."""
    dev = rows.device
    out = torch.empty((rows.n, q.d), dtype=torch.float32, device=dev)
    if rows.n:
        ws = workspace(_lib.query("pq_decode_workspace_bytes", rows.n, q.d), dev)
        cent = q._params(dev).cent[precision]
        _lib.call("pq_decode", ptr(rows.buf), rows.ldb, ptr(rows.norms), rows.n, q.d, rows.bits,
                  precision, ptr(cent), ptr(rt(q, dev)), ptr(out), ptr(ws), ws.numel(),
                  stream_ptr(dev))
    return out


def rotate_tc(q, X) -> torch.Tensor:
    """Y = X @ R^T through the tensor-core encode GEMM (f32)."""
    dev = require_cuda()
    Xd = to_device_f32(X, dev)
    n = Xd.shape[0]
    Y = torch.empty((n, q.d), dtype=torch.float32, device=dev)
    if n:
        ws = workspace(_lib.query("pq_encode_workspace_bytes", n, q.d), dev)
        _lib.call("pq_rotate_tc", ptr(Xd), n, q.d, ptr(_planes(q, dev)), ptr(Y), ptr(ws),
                  ws.numel(), stream_ptr(dev))
    return Y


def alloc_corpus(q, n: int, dev):
    """An uninitialised device corpus of n rows for this quantizer (filled by encode_into)."""
    from .core import _DeviceRows
    ldb = row_stride(q.d, q.bits)
    buf = alloc_rows(n, ldb, dev)
    norms = torch.empty(int(n), dtype=torch.float32, device=dev)
    return _DeviceRows(buf, norms, int(n), q.d, q.bits, ldb, dev)


def encode_into(q, X, rows, start: int) -> None:
    """Encodes X (device f32, m x d) into rows [start, start + m) of an existing
    device corpus, so corpora larger than one f32 staging buffer are built chunk
    by chunk."""
    Xd = to_device_f32(X, rows.device)
    m = Xd.shape[0]
    if Xd.dim() != 2 or Xd.shape[1] != q.d:
        raise ValueError(f"Expected d={q.d}")
    if start < 0 or start + m > rows.n:
        raise IndexError("rows out of range")
    if m == 0:
        return
    dev = rows.device
    pr = q._params(dev)
    ws = workspace(_lib.query("pq_encode_workspace_bytes", m, q.d), dev)
    pk = ctypes.c_void_p(rows.buf.data_ptr() + int(start) * rows.ldb)
    nr = ctypes.c_void_p(rows.norms.data_ptr() + int(start) * 4)
    _lib.call("pq_encode", ptr(Xd), m, q.d, ptr(pr.R), ptr(_planes(q, dev)), ptr(pr.boundaries),
              q.bits, pk, rows.ldb, nr, ptr(ws), ws.numel(), stream_ptr(dev))

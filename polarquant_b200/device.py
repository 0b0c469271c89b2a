"""Device plumbing: torch tensors as device memory, the current CUDA stream,
and the padded row layout the kernels read.

PyTorch only allocates memory and provides streams here; every computation
on the search and encode path is a kernel of the polarquant_b200 library.
"""

from __future__ import annotations

import ctypes

import numpy as np
import torch

from . import _lib
from .packing import packed_nbytes

ROW_SLACK = 64  # bytes after the last packed row (the 3-bit reader fetches 12-byte groups)


def require_cuda() -> torch.device:
    if not torch.cuda.is_available():
        raise RuntimeError("polarquant_b200 needs a CUDA device (B200, sm_100a); none is visible")
    return torch.device("cuda", torch.cuda.current_device())


def ptr(t: torch.Tensor | None) -> ctypes.c_void_p:
    return ctypes.c_void_p(0 if t is None else t.data_ptr())


def stream_ptr(device: torch.device | None = None) -> ctypes.c_void_p:
    return ctypes.c_void_p(torch.cuda.current_stream(device).cuda_stream)


def row_stride(d: int, bits: int) -> int:
    """Device row stride: packed row bytes rounded up to 16 (128-bit loads)."""
    rb = packed_nbytes(1, d, bits)
    return max(16, (rb + 15) // 16 * 16)


def alloc_rows(n: int, ldb: int, device: torch.device) -> torch.Tensor:
    """Flat uint8 buffer for n rows of stride ldb plus the read slack."""
    return torch.empty(int(n) * int(ldb) + ROW_SLACK, dtype=torch.uint8, device=device)


def workspace(nbytes: int, device: torch.device) -> torch.Tensor:
    return torch.empty(max(256, int(nbytes)), dtype=torch.uint8, device=device)


def to_device_f32(x, device: torch.device) -> torch.Tensor:
    """Host array or tensor -> contiguous f32 tensor on `device`."""
    if isinstance(x, torch.Tensor):
        return x.to(device=device, dtype=torch.float32).contiguous()
    a = np.ascontiguousarray(np.asarray(x, dtype=np.float32))
    return torch.from_numpy(a).to(device, non_blocking=False)


def rows_to_device(rows: np.ndarray, ldb: int, device: torch.device) -> torch.Tensor:
    """(n, row_bytes) host rows -> padded device buffer of stride ldb."""
    rows = np.ascontiguousarray(rows, dtype=np.uint8)
    n, rb = rows.shape
    buf = alloc_rows(n, ldb, device)
    if n:
        host = np.zeros((n, ldb), np.uint8)
        host[:, :rb] = rows
        buf[: n * ldb].copy_(torch.from_numpy(host.ravel()))
    return buf


def rows_to_host(buf: torch.Tensor, n: int, ldb: int, rb: int) -> np.ndarray:
    """Padded device buffer -> (n, row_bytes) host rows."""
    if n == 0:
        return np.zeros((0, rb), np.uint8)
    return buf[: n * ldb].view(n, ldb)[:, :rb].cpu().numpy().copy()


def topk_to_numpy(scores: torch.Tensor, ids: torch.Tensor):
    """(nq, k) device results -> host (ids intp, scores f32)."""
    return ids.cpu().numpy().astype(np.intp, copy=False), scores.cpu().numpy()


def check_device_errors() -> None:
    code = _lib.device_status()
    if code:
        raise _lib.PQError("kernel", -5, f"device-side failure code {code}")

"""Row-sharded search across GPUs (one process per GPU, torch.distributed).

Rank r holds corpus rows [row_offset, row_offset + n_local) as a packed
shard on its GPU; queries are replicated.  The exchange steps are exact:

* ADC / batch top-k: each rank's local top-k (f32 score, global i64 id) is
  all-gathered and merged (score desc, id asc), giving the same ids and
  scores as one GPU holding the whole corpus.
* Two-stage: a first exchange all-gathers the local coarse top-C lists and
  every rank selects the same global top-C; in a second, each rank rescores
  only the candidates it owns at full precision, all-gathers those lists and
  merges the top-k.  This reproduces the single-GPU result exactly
  (remex/core.py:638-719 semantics over the whole corpus).

The collectives run on the caller's process group (NCCL over NVLink on a B200
box; gloo works for CPU tests).  The per-rank compute steps are methods so a
test can substitute a CPU implementation and check the protocol alone.
"""

from __future__ import annotations

from typing import Optional

import numpy as np
import torch
import torch.distributed as dist

from . import _lib

SENTINEL_ID = -1


def shard_bounds(n: int, world: int, rank: int):
    """Contiguous near-equal row block of `rank` (first n % world ranks get one more)."""
    base, extra = divmod(int(n), int(world))
    start = rank * base + min(rank, extra)
    return start, start + base + (1 if rank < extra else 0)


def pad_topk(s: torch.Tensor, i: torch.Tensor, k: int):
    """(nq, kl) -> (nq, k) with sentinel slots (score -inf, id -1)."""
    nq, kl = s.shape
    if kl == k:
        return s.contiguous(), i.contiguous()
    ps = torch.full((nq, k), float("-inf"), dtype=s.dtype, device=s.device)
    pi = torch.full((nq, k), SENTINEL_ID, dtype=i.dtype, device=i.device)
    ps[:, :kl] = s
    pi[:, :kl] = i
    return ps, pi


class ShardedSearch:
    """Search over a corpus whose rows are split across the ranks of `group`."""

    def __init__(self, quantizer, shard, row_offset: int, n_total: int, group=None):
        self.q = quantizer
        self.shard = shard
        self.row_offset = int(row_offset)
        self.n_total = int(n_total)
        self.group = group
        self.world = dist.get_world_size(group) if dist.is_initialized() else 1
        self.rank = dist.get_rank(group) if dist.is_initialized() else 0
        self.force = None  # "scan" / "batch" pins the per-rank ADC path

    # -- per-rank compute (CUDA library); tests may override ---------------------
    @property
    def n_local(self) -> int:
        return self.shard.n

    def rotate(self, Q) -> torch.Tensor:
        rows = self.shard._device()
        return self.q._rotate(Q, rows.device)

    def local_topk(self, qrot: torch.Tensor, k: int, precision: int):
        rows = self.shard._device()
        s, i = self.q._scan(rows, qrot, k, precision, force=self.force)
        return s, i + self.row_offset

    def local_rerank(self, qrot: torch.Tensor, cand: torch.Tensor, k: int):
        """Full-precision top-k among the candidates this rank owns."""
        rows = self.shard._device()
        nq, C = cand.shape
        s = torch.empty((nq, k), dtype=torch.float32, device=qrot.device)
        i = torch.empty((nq, k), dtype=torch.int64, device=qrot.device)
        from .device import ptr, stream_ptr
        cent = self.q._params(rows.device).cent[self.q.bits]
        _lib.call("pq_rerank", ptr(rows.buf), rows.ldb, ptr(rows.norms), rows.n, rows.d,
                  rows.bits, ptr(qrot), nq, ptr(cent), ptr(cand), C, k, self.row_offset,
                  ptr(s), ptr(i), stream_ptr(rows.device))
        return s, i

    def merge(self, s_parts: torch.Tensor, i_parts: torch.Tensor, k: int):
        """(parts, nq, kin) -> (nq, k) by the library's merge kernel."""
        from .device import ptr, stream_ptr
        parts, nq, kin = s_parts.shape
        out_s = torch.empty((nq, k), dtype=torch.float32, device=s_parts.device)
        out_i = torch.empty((nq, k), dtype=torch.int64, device=s_parts.device)
        _lib.call("pq_topk_merge", ptr(s_parts), ptr(i_parts), parts, nq, kin, k, ptr(out_s),
                  ptr(out_i), stream_ptr(s_parts.device))
        return out_s, out_i

    # -- communication ----------------------------------------------------------
    def all_gather(self, t: torch.Tensor) -> torch.Tensor:
        if self.world == 1:
            return t.unsqueeze(0)
        t = t.contiguous()
        out = torch.empty((self.world * t.shape[0],) + tuple(t.shape[1:]), dtype=t.dtype,
                          device=t.device)
        dist.all_gather_into_tensor(out, t, group=self.group)
        return out.view((self.world,) + tuple(t.shape))

    def _gathered_topk(self, s: torch.Tensor, i: torch.Tensor, k: int, k_out: int):
        s, i = pad_topk(s, i, k)
        if self.world == 1:
            return s[:, :k_out], i[:, :k_out]
        return self.merge(self.all_gather(s), self.all_gather(i), k_out)

    # -- protocol -----------------------------------------------------------------
    def search_adc_many(self, Q, k: int = 10, precision: Optional[int] = None):
        p = self.q._level(precision)
        qrot = self.rotate(Q)
        k_out = min(int(k), self.n_total)
        kl = min(k_out, self.n_local)
        if kl > 0:
            s, i = self.local_topk(qrot, kl, p)
        else:
            s = torch.empty((qrot.shape[0], 0), dtype=torch.float32, device=qrot.device)
            i = torch.empty((qrot.shape[0], 0), dtype=torch.int64, device=qrot.device)
        return self._gathered_topk(s, i, k_out, k_out)

    def search_twostage_many(self, Q, k: int = 10, candidates: int = 500,
                             coarse_precision: Optional[int] = None):
        if coarse_precision is None:
            coarse_precision = max(1, self.q.bits - 2)
        cp = self.q._level(coarse_precision)
        ck = min(int(candidates), self.n_total)
        if ck >= self.n_total:
            return self.search_adc_many(Q, k=min(k, self.n_total), precision=None)
        qrot = self.rotate(Q)
        nq = qrot.shape[0]
        kl = min(ck, self.n_local)
        if kl > 0:
            s, i = self.local_topk(qrot, kl, cp)
        else:
            s = torch.empty((nq, 0), dtype=torch.float32, device=qrot.device)
            i = torch.empty((nq, 0), dtype=torch.int64, device=qrot.device)
        _, cand = self._gathered_topk(s, i, ck, ck)        # first exchange: global top-C ids
        k_out = min(int(k), ck)
        fs, fi = self.local_rerank(qrot, cand.contiguous(), k_out)  # owned candidates only
        return self._gathered_topk(fs, fi, k_out, k_out)   # second exchange: global top-k


def to_numpy(s: torch.Tensor, i: torch.Tensor):
    return i.cpu().numpy().astype(np.intp, copy=False), s.cpu().numpy()

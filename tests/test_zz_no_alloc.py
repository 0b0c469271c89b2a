"""The allocation-free ADC scan entry point (pq_adc_scan_noalloc).

It serves callers that cannot allocate device memory (hosts that reserve the
GPU's memory for their own pool, latency-critical paths that cannot pay for
cudaMalloc): the scan's scratch is a built-in device array instead of a
caller workspace.  This file is collected last so that a failure here stops a
-x run only after every other test has run.  Each check calls the new entry
point through the C ABI and compares it with pq_adc_scan on the same inputs,
twice in a row (the second call reuses the scratch the first one left).
"""

import ctypes

import numpy as np
import pytest

from oracle import remex_oracle as O

pytestmark = pytest.mark.gpu

RTOL = 1e-4


def _corpus(bits=4, d=128, n=5000, nq=7, seed=3):
    from polarquant_b200 import CompressedVectors, Quantizer
    pq = Quantizer(d, bits=bits, seed=seed)
    rng = np.random.default_rng(seed)
    X = rng.standard_normal((n, d)).astype(np.float32)
    Q = rng.standard_normal((nq, d)).astype(np.float32)
    idx, norms = O.encode(X, pq.R, pq.boundaries)
    return pq, CompressedVectors(idx, norms, d, bits), Q


def _both(pq, cv, qrot, k, p):
    import torch
    from polarquant_b200 import _lib
    from polarquant_b200.device import ptr, stream_ptr, workspace
    rows = cv._device()
    dev = rows.device
    nq = qrot.shape[0]
    cent = pq._params(dev).cent[p]
    out = []
    for name in ("pq_adc_scan", "pq_adc_scan_noalloc"):
        s = torch.empty((nq, k), dtype=torch.float32, device=dev)
        i = torch.empty((nq, k), dtype=torch.int64, device=dev)
        args = [ptr(rows.buf), rows.ldb, ptr(rows.norms), rows.n, rows.d, rows.bits, p, ptr(qrot),
                nq, ptr(cent), k, 0, ptr(s), ptr(i)]
        if name == "pq_adc_scan":
            ws = workspace(_lib.query("pq_adc_scan_workspace_bytes", rows.n, rows.d, nq, k), dev)
            args += [ptr(ws), ws.numel()]
        _lib.call(name, *args, stream_ptr(dev))
        torch.cuda.synchronize()
        out.append((i.cpu().numpy(), s.cpu().numpy()))
    return out


def _same(a, b):
    (ia, sa), (ib, sb) = a, b
    assert ia.shape == ib.shape
    for q in range(ia.shape[0]):
        assert O.topk_equal_up_to_ties(ib[q], sb[q], ia[q], sa[q], rtol=RTOL)
        np.testing.assert_allclose(sb[q], sa[q], rtol=RTOL, atol=RTOL * np.abs(sa[q]).max())


def test_noalloc_scan_matches_workspace_scan_twice(gpu):
    pq, cv, Q = _corpus()
    dev = cv._device().device
    qrot = pq._rotate(Q, dev)
    ref1, got1 = _both(pq, cv, qrot, 10, 4)
    _same(ref1, got1)
    # ... and the oracle's search_adc (remex/core.py:582-636) on the same corpus.
    idx, norms = cv.indices, cv.norms
    for q in range(Q.shape[0]):
        ri, rs = O.search_adc(pq.R, pq.centroids, pq._nested, 4, idx, norms, Q[q], k=10)
        assert O.topk_equal_up_to_ties(got1[0][q], got1[1][q], ri, rs, rtol=RTOL), q
    # Second call in a row: other queries, other k and precision, same scratch.
    qrot2 = pq._rotate(Q[::-1].copy() * 2.0, dev)
    ref2, got2 = _both(pq, cv, qrot2, 37, 2)
    _same(ref2, got2)


def test_noalloc_scan_rejects_oversized_calls(gpu):
    from polarquant_b200 import _lib
    pq, cv, Q = _corpus(n=300, nq=2)
    rows = cv._device()
    cap = _lib.query("pq_adc_scan_noalloc_scratch_bytes")
    assert cap > 0
    P = ctypes.c_void_p
    # More scratch than the built-in array holds: many queries x large k.
    with pytest.raises(_lib.PQError, match="scratch"):
        _lib.call("pq_adc_scan_noalloc", P(rows.buf.data_ptr()), rows.ldb,
                  P(rows.norms.data_ptr()), 300000000, rows.d, rows.bits, 4, P(16), 60000,
                  P(16), 2048, 0, P(16), P(16), None)
    with pytest.raises(_lib.PQError, match="k must be"):
        _lib.call("pq_adc_scan_noalloc", P(rows.buf.data_ptr()), rows.ldb,
                  P(rows.norms.data_ptr()), rows.n, rows.d, rows.bits, 4, P(16), 1, P(16),
                  4096, 0, P(16), P(16), None)


def test_noalloc_scan_k_limit_on_a_large_corpus(gpu):
    """One query on a corpus of a few million rows: the scan then splits the
    rows into about 8 blocks per SM, each keeping k candidates in the built-in
    scratch, so the scratch bounds k below PQ_TOPK_MAX.  The largest k the
    entry point accepts (found by calling it) is above 512 -- the byte-table
    scan's tables and partial sums, which this corpus's 3M rows would make
    larger than the scratch, do not lower the bound -- its results match
    pq_adc_scan, and the next k is rejected with PQ_ERR_WORKSPACE."""
    import torch
    from polarquant_b200 import CompressedVectors, Quantizer, _lib
    from polarquant_b200.device import ptr, stream_ptr
    d, n = 64, 3_000_000
    pq = Quantizer(d, bits=4, seed=5)
    rng = np.random.default_rng(9)
    idx = rng.integers(0, 16, size=(n, d), dtype=np.uint8)
    norms = rng.uniform(0.5, 2.0, n).astype(np.float32)
    cv = CompressedVectors(idx, norms, d, 4)
    q = rng.standard_normal((1, d)).astype(np.float32)
    rows = cv._device()
    dev = rows.device
    qrot = pq._rotate(q, dev)
    cent = pq._params(dev).cent[4]

    def accepted(k):
        s = torch.empty((1, k), dtype=torch.float32, device=dev)
        i = torch.empty((1, k), dtype=torch.int64, device=dev)
        try:
            _lib.call("pq_adc_scan_noalloc", ptr(rows.buf), rows.ldb, ptr(rows.norms), rows.n, d,
                      4, 4, ptr(qrot), 1, ptr(cent), k, 0, ptr(s), ptr(i), stream_ptr(dev))
        except _lib.PQError as e:
            assert e.code == -3 and "scratch" in str(e), e
            return False
        torch.cuda.synchronize()
        return True

    assert accepted(1)
    assert not accepted(2048), "a multi-million-row corpus should bound k below PQ_TOPK_MAX"
    lo, hi = 1, 2048  # accepted(lo), not accepted(hi)
    while hi - lo > 1:
        mid = (lo + hi) // 2
        if accepted(mid):
            lo = mid
        else:
            hi = mid
    kmax = lo
    assert kmax > 512, kmax
    ref, got = _both(pq, cv, qrot, kmax, 4)
    _same(ref, got)
    assert not accepted(kmax + 1)

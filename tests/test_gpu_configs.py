"""GPU parity on the benchmark configurations' own data distributions and
production shapes, against the CPU oracle.

* d=1536, 4-bit, clustered (10,000 centres, noise 0.2/sqrt(d)), >= 2^20 rows,
  512 queries, k=100: the batched ADC runs the int8 tensor-core kernel with
  its row chunks sharing per-query thresholds, then the exact rescoring;
  checked against the oracle's search_batch (remex/core.py:721-778) on
  sampled queries and against the exact streaming scan on all of them.
* d=768, 8-bit, clustered (1,000 centres, noise 0.3/sqrt(d)), 1M rows, 96
  queries: search_twostage(coarse_precision=4, candidates=200, k=10) with the
  coarse stage on the fp16 pair kernel (remex/core.py:638-719).
* IVF: d=384, 4-bit, 1M rows from 4,096 centres (noise 0.1/sqrt(d)),
  n_bits=12 lsh, nprobe=32, coarse precision 2, 500 candidates, k=10
  (remex/ivf.py:376-436).

Corpora are generated on the GPU by the benchmark's own generator and
encoded on the GPU; the oracle then searches the same codes (search parity is
independent of the encode, which tests/test_gpu_encode.py pins).  Tolerance:
scores within 1e-4 relative; top-k ids identical except score ties.
"""

import numpy as np
import pytest

from oracle import remex_oracle as O

pytestmark = pytest.mark.gpu

RTOL = 1e-4


def _corpus(cfg, n, nq, seed=1):
    import torch
    import bench
    from polarquant_b200 import Quantizer
    from polarquant_b200.core import CompressedVectors
    from polarquant_b200.encode import alloc_corpus, encode_into
    dev = torch.device("cuda", torch.cuda.current_device())
    cfg = dict(cfg, n=n, nq=nq)
    pq = Quantizer(cfg["d"], bits=cfg["bits"], seed=42)
    centres = bench.make_centres(torch, dev, cfg, seed=7)
    rows = alloc_corpus(pq, n, dev)
    for a in range(0, n, 1 << 20):
        b = min(n, a + (1 << 20))
        X = bench.gen_rows(torch, dev, cfg, a, b, seed=seed, centres=centres)
        encode_into(pq, X, rows, a)
        del X
    Q = bench.make_queries(torch, dev, cfg, centres)
    torch.cuda.synchronize()
    return pq, CompressedVectors._from_device(rows), Q.cpu().numpy()


def test_config4_clustered_batched_adc(gpu):
    import bench
    from polarquant_b200 import _lib
    from polarquant_b200.core import use_tensor_cores
    n, nq, k = (1 << 20) + 4096, 512, 100
    pq, cv, Q = _corpus(bench.WORKLOADS["c4"], n, nq)
    rows = cv._device()
    assert use_tensor_cores(n, nq, k)
    assert _lib.query("pq_adc_batch_kernel", n, rows.d, 4, 4, k, rows.ldb) == 1, \
        "d=1536 4-bit k=100 should run the int8 pair kernel"
    GI, GS = pq.search_adc_many(cv, Q, k=k)
    assert GI.shape == (nq, k)
    # All queries against the exact streaming scan (f32 table sums).
    s, i = pq._scan(rows, pq._rotate(Q, rows.device), k, 4, force="scan")
    SI, SS = i.cpu().numpy(), s.cpu().numpy()
    bad = [q for q in range(nq) if not O.topk_equal_up_to_ties(GI[q], GS[q], SI[q], SS[q],
                                                                rtol=RTOL)]
    assert not bad, f"{len(bad)} of {nq} queries differ from the exact scan: {bad[:8]}"
    # Sampled queries (every 4th, all four 128-query quarters of each pair
    # tile) against the oracle's search_batch over the same codes.
    pick = np.arange(0, nq, 4)
    RI, RS = O.search_batch_chunked(pq.R, pq.centroids, pq._nested, 4, cv.indices, cv.norms,
                                    Q[pick], k=k)
    bad = [int(q) for j, q in enumerate(pick)
           if not O.topk_equal_up_to_ties(GI[q], GS[q], RI[j], RS[j], rtol=RTOL)]
    assert not bad, f"{len(bad)} sampled queries differ from the oracle: {bad[:8]}"


def test_config2_clustered_twostage(gpu):
    import bench
    from polarquant_b200 import _lib
    n, nq = 1_000_000, 96
    pq, cv, Q = _corpus(bench.WORKLOADS["c2"], n, nq)
    rows = cv._device()
    assert _lib.query("pq_adc_batch_kernel", n, rows.d, 8, 4, 200, rows.ldb) == 2, \
        "d=768 coarse stage should run the fp16 pair kernel"
    GI, GS = pq.search_twostage_many(cv, Q, k=10, candidates=200, coarse_precision=4)
    RI, RS = O.search_twostage_chunked(pq.R, pq.centroids, pq._nested, 8, cv.indices, cv.norms,
                                       Q, k=10, candidates=200, coarse_precision=4)
    bad = [q for q in range(nq) if not O.topk_equal_up_to_ties(GI[q], GS[q], RI[q], RS[q],
                                                                rtol=RTOL)]
    assert not bad, f"{len(bad)} of {nq} queries differ from the oracle: {bad[:8]}"


def test_config5_ivf_n_bits12(gpu):
    import bench
    from polarquant_b200 import IVFCoarseIndex
    n, nq = 1_000_000, 64
    pq, cv, Q = _corpus(bench.WORKLOADS["c5"], n, nq)
    ix = IVFCoarseIndex(pq, cv, n_bits=12, mode="lsh", seed=0)
    idx, norms = cv.indices, cv.norms
    H = ix.hyperplanes
    # The device build against the oracle's (remex/ivf.py:162-224): LSH
    # projections are summed exactly on the device and in f32 by the
    # reference, so a row within f32 rounding of a hyperplane may differ.
    cells = O.ivf_cell_ids(idx, 4, 12, "lsh", H)
    assert (cells != ix.cell_ids).mean() < 1e-4
    if (cells == ix.cell_ids).all():
        srt, off = O.ivf_csr(cells, 1 << 12)
        np.testing.assert_array_equal(ix.sorted_idx, srt)
        np.testing.assert_array_equal(ix.cell_offsets, off)
    srt, off = ix.sorted_idx, ix.cell_offsets
    ids, sc = ix.search_twostage_many(Q, k=10, candidates=500, nprobe=32, coarse_precision=2)
    bad = []
    for q in range(nq):
        ri, rs = O.ivf_search_twostage(pq.R, pq.centroids, pq._nested, 4, idx, norms, srt, off,
                                       12, "lsh", H, Q[q], k=10, candidates=500, nprobe=32,
                                       coarse_precision=2)
        keep = ids[q] >= 0
        if not O.topk_equal_up_to_ties(ids[q][keep], sc[q][keep], ri, rs, rtol=RTOL):
            bad.append(q)
    assert not bad, f"{len(bad)} of {nq} queries differ from the oracle: {bad[:8]}"


def test_batched_adc_with_threshold_pilot_pass(gpu):
    """Corpora of 4M+ rows run the int8 kernel in two passes: the first
    pass's merged lists seed every query's threshold for the second.  The
    results must not depend on it: all queries against the exact streaming
    scan, sampled ones against the oracle's search_batch."""
    import bench
    from polarquant_b200 import _lib
    cfg = dict(bench.WORKLOADS["c4"], d=1024)
    n, nq, k = (4 << 20) + 777, 300, 64
    pq, cv, Q = _corpus(cfg, n, nq)
    rows = cv._device()
    assert _lib.query("pq_adc_batch_kernel", n, rows.d, 4, 4, k, rows.ldb) == 1
    GI, GS = pq.search_adc_many(cv, Q, k=k)
    s, i = pq._scan(rows, pq._rotate(Q, rows.device), k, 4, force="scan")
    SI, SS = i.cpu().numpy(), s.cpu().numpy()
    bad = [q for q in range(nq) if not O.topk_equal_up_to_ties(GI[q], GS[q], SI[q], SS[q],
                                                                rtol=RTOL)]
    assert not bad, f"{len(bad)} of {nq} queries differ from the exact scan: {bad[:8]}"
    pick = np.arange(0, nq, 25)
    RI, RS = O.search_batch_chunked(pq.R, pq.centroids, pq._nested, 4, cv.indices, cv.norms,
                                    Q[pick], k=k)
    bad = [int(q) for j, q in enumerate(pick)
           if not O.topk_equal_up_to_ties(GI[q], GS[q], RI[j], RS[j], rtol=RTOL)]
    assert not bad, f"{len(bad)} sampled queries differ from the oracle: {bad[:8]}"

"""GPU parity of the TMA-staged streaming ADC scan (4- and 8-bit codes) against
the oracle's search_adc (remex/core.py:597-636): every Matryoshka precision,
ragged row lengths (slab padding), partial tiles and blocks, large k, and the
shapes that fall back to the generic scan."""

import numpy as np
import pytest

from oracle import remex_oracle as O

pytestmark = pytest.mark.gpu
RTOL = 1e-4


def _case(bits, d, n, nq, seed=3):
    from polarquant_b200 import CompressedVectors, Quantizer
    pq = Quantizer(d=d, bits=bits, seed=42)
    rng = np.random.default_rng(seed)
    X = rng.standard_normal((n, d)).astype(np.float32)
    X *= rng.uniform(0.5, 2.0, size=(n, 1)).astype(np.float32)
    Q = rng.standard_normal((nq, d)).astype(np.float32)
    idx, norms = O.encode(X, pq.R, pq.boundaries)
    return pq, CompressedVectors(idx, norms, d, bits), idx, norms, Q


def _kernel(cv, p, nq, k):
    from polarquant_b200 import _lib
    rows = cv._device()
    return _lib.query("pq_adc_scan_kernel", rows.n, rows.d, rows.bits, p, nq, k, rows.ldb)


@pytest.mark.parametrize("bits,d", [(4, 256), (4, 384), (4, 1000), (8, 128), (8, 200),
                                    (8, 768)])
def test_tma_scan_every_precision(gpu, bits, d):
    pq, cv, idx, norms, Q = _case(bits, d, 9001, 3)
    for p in range(1, bits + 1):
        assert _kernel(cv, p, 3, 50) == 2, (bits, d, p)
        gi, gs = pq.search_adc_many(cv, Q, k=50, precision=p)
        for qi, q in enumerate(Q):
            ri, rs = O.search_adc(pq.R, pq.centroids, pq._nested, bits, idx, norms, q, k=50,
                                  precision=p)
            assert O.topk_equal_up_to_ties(gi[qi], gs[qi], ri, rs, rtol=RTOL), (p, qi)


@pytest.mark.parametrize("bits,d,k", [(8, 768, 1500), (4, 1536, 2048), (4, 384, 1)])
def test_tma_scan_large_and_small_k(gpu, bits, d, k):
    pq, cv, idx, norms, Q = _case(bits, d, 20000, 2, seed=5)
    assert _kernel(cv, bits, 2, k) == 2
    gi, gs = pq.search_adc_many(cv, Q, k=k)
    for qi, q in enumerate(Q):
        ri, rs = O.search_adc(pq.R, pq.centroids, pq._nested, bits, idx, norms, q, k=k)
        assert O.topk_equal_up_to_ties(gi[qi], gs[qi], ri, rs, rtol=RTOL), qi


@pytest.mark.parametrize("n", [256, 257, 511, 4096, 70001])
def test_tma_scan_row_counts(gpu, n):
    pq, cv, idx, norms, Q = _case(8, 256, n, 2, seed=n)
    k = min(40, n)
    assert _kernel(cv, 4, 2, k) == 2
    for p in (4, 8):
        gi, gs = pq.search_adc_many(cv, Q, k=k, precision=p)
        for qi, q in enumerate(Q):
            ri, rs = O.search_adc(pq.R, pq.centroids, pq._nested, 8, idx, norms, q, k=k,
                                  precision=p)
            assert O.topk_equal_up_to_ties(gi[qi], gs[qi], ri, rs, rtol=RTOL), (p, qi)


def test_tma_scan_many_queries_forced(gpu):
    """Query batches above the tensor-core threshold, forced onto the scan."""
    import torch
    pq, cv, idx, norms, Q = _case(4, 512, 6000, 70, seed=9)
    rows = cv._device()
    qrot = pq._rotate(Q, rows.device)
    s, i = pq._scan(rows, qrot, 20, 3, force="scan")
    torch.cuda.synchronize()
    s, i = s.cpu().numpy(), i.cpu().numpy()
    for qi, q in enumerate(Q):
        ri, rs = O.search_adc(pq.R, pq.centroids, pq._nested, 4, idx, norms, q, k=20,
                              precision=3)
        assert O.topk_equal_up_to_ties(i[qi], s[qi], ri, rs, rtol=RTOL), qi


@pytest.mark.parametrize("bits,d,n", [(4, 128, 3000), (4, 64, 3000), (8, 96, 3000),
                                      (8, 256, 200), (3, 512, 3000)])
def test_generic_scan_fallback_shapes(gpu, bits, d, n):
    pq, cv, idx, norms, Q = _case(bits, d, n, 2)
    assert _kernel(cv, bits, 2, 10) == 1
    gi, gs = pq.search_adc_many(cv, Q, k=10)
    for qi, q in enumerate(Q):
        ri, rs = O.search_adc(pq.R, pq.centroids, pq._nested, bits, idx, norms, q, k=10)
        assert O.topk_equal_up_to_ties(gi[qi], gs[qi], ri, rs, rtol=RTOL), qi

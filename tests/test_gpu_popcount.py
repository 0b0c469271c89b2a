"""GPU parity of the 1-bit popcount coarse scorer (pq_hamming_scan /
pq_hamming_twostage) against the oracle's statement of it.  The coarse
scores are integers (d - 2 * Hamming distance of the sign bits), so the
coarse top-k must match the oracle exactly, ids and scores, ties by row; the
two-stage results (full-precision rescoring) within 1e-4 relative, top-k ids
equal up to score ties."""

import numpy as np
import pytest

from oracle import remex_oracle as O

pytestmark = pytest.mark.gpu


def _case(bits, d, n, nq=4, seed=0, clustered=False):
    from polarquant_b200 import CompressedVectors, Quantizer
    rng = np.random.default_rng(seed)
    if clustered:
        cen = rng.standard_normal((20, d)).astype(np.float32)
        X = cen[rng.integers(0, 20, n)] + 0.3 * rng.standard_normal((n, d)).astype(np.float32)
        Q = cen[rng.integers(0, 20, nq)] + 0.3 * rng.standard_normal((nq, d)).astype(np.float32)
    else:
        X = rng.standard_normal((n, d)).astype(np.float32)
        Q = rng.standard_normal((nq, d)).astype(np.float32)
    pq = Quantizer(d, bits=bits, seed=42)
    idx, norms = O.encode(X, pq.R, pq.boundaries)
    return pq, CompressedVectors(idx, norms, d, bits), idx, norms, Q


@pytest.mark.parametrize("bits,d", [(8, 768), (4, 384), (1, 128), (2, 100), (3, 40), (4, 1536)])
def test_popcount_scan_exact(gpu, bits, d):
    pq, cv, idx, norms, Q = _case(bits, d, 5000, clustered=True)
    GI, GS = pq.search_popcount_many(cv, Q, k=300)
    for q in range(len(Q)):
        ri, rs = O.search_popcount(pq.R, bits, idx, Q[q], k=300)
        np.testing.assert_array_equal(GI[q], ri)
        np.testing.assert_array_equal(GS[q], rs)


@pytest.mark.parametrize("bits,d,C", [(8, 768, 200), (4, 384, 500), (8, 256, 2048)])
def test_popcount_twostage(gpu, bits, d, C):
    pq, cv, idx, norms, Q = _case(bits, d, 8000, seed=1, clustered=True)
    GI, GS = pq.search_twostage_popcount_many(cv, Q, k=10, candidates=C)
    for q in range(len(Q)):
        ri, rs = O.search_twostage_popcount(pq.R, pq.centroids, bits, idx, norms, Q[q], k=10,
                                            candidates=C)
        assert O.topk_equal_up_to_ties(GI[q], GS[q], ri, rs, rtol=1e-4), q


def test_popcount_edges(gpu):
    from polarquant_b200 import PackedVectors
    pq, cv, idx, norms, Q = _case(8, 64, 300, seed=2)
    # k > n: every row, in order; candidates >= n: the full-precision search.
    gi, gs = pq.search_popcount(cv, Q[0], k=1000)
    ri, rs = O.search_popcount(pq.R, 8, idx, Q[0], k=1000)
    np.testing.assert_array_equal(gi, ri)
    a = pq.search_twostage_popcount(cv, Q[0], k=10, candidates=300)
    b = pq.search_adc(cv, Q[0], k=10)
    np.testing.assert_array_equal(a[0], b[0])
    # PackedVectors take the same path (their 1-bit tier is made on demand).
    pv = PackedVectors.from_compressed(cv)
    gi2, gs2 = pq.search_popcount(pv, Q[0], k=50)
    np.testing.assert_array_equal(gi2, ri[:50])
    big = _case(4, 32, 3000, seed=3)
    with pytest.raises(ValueError, match="2048"):
        big[0].search_popcount(big[1], big[4][0], k=2500)

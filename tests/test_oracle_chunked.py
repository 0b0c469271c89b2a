"""The oracle's chunked batch forms (used by the config-scale GPU parity tests,
whose corpora are too large for one (Q, n) score matrix) give the same
results as the direct restatements of remex/core.py:638-778."""

import numpy as np
import pytest

from oracle import remex_oracle as O
from polarquant_b200.params import haar_rotation, lloyd_max_codebook, nested_codebooks


@pytest.mark.parametrize("bits,prec", [(4, None), (8, 3), (2, 1)])
def test_search_batch_chunked_equals_search_batch(bits, prec):
    d = 64
    R = haar_rotation(d, 42)
    bnd, cent = lloyd_max_codebook(d, bits)
    nest = nested_codebooks(d, bits)
    rng = np.random.default_rng(bits)
    X = rng.standard_normal((5000, d)).astype(np.float32)
    Q = rng.standard_normal((9, d)).astype(np.float32)
    idx, nr = O.encode(X, R, bnd)
    I1, S1 = O.search_batch(R, cent, nest, bits, idx, nr, Q, k=33, precision=prec)
    I2, S2 = O.search_batch_chunked(R, cent, nest, bits, idx, nr, Q, k=33, precision=prec,
                                    chunk=700)
    assert I2.shape == I1.shape
    for q in range(len(Q)):
        assert O.topk_equal_up_to_ties(I2[q], S2[q], I1[q], S1[q])


def test_search_twostage_chunked_equals_search_twostage():
    d, bits = 64, 8
    R = haar_rotation(d, 42)
    bnd, cent = lloyd_max_codebook(d, bits)
    nest = nested_codebooks(d, bits)
    rng = np.random.default_rng(3)
    X = rng.standard_normal((5000, d)).astype(np.float32)
    Q = rng.standard_normal((7, d)).astype(np.float32)
    idx, nr = O.encode(X, R, bnd)
    It, St = O.search_twostage_chunked(R, cent, nest, bits, idx, nr, Q, k=10, candidates=200,
                                       coarse_precision=4, chunk=900)
    for q in range(len(Q)):
        ri, rs = O.search_twostage(R, cent, nest, bits, idx, nr, Q[q], k=10, candidates=200,
                                   coarse_precision=4)
        assert O.topk_equal_up_to_ties(It[q], St[q], ri, rs)


def test_search_batch_cached_equals_search_batch():
    d, bits = 48, 4
    R = haar_rotation(d, 42)
    bnd, cent = lloyd_max_codebook(d, bits)
    nest = nested_codebooks(d, bits)
    rng = np.random.default_rng(5)
    X = rng.standard_normal((3000, d)).astype(np.float32)
    Q = rng.standard_normal((6, d)).astype(np.float32)
    idx, nr = O.encode(X, R, bnd)
    Xh = O.x_hat_rot(cent, nest, bits, idx)
    I1, S1 = O.search_batch(R, cent, nest, bits, idx, nr, Q, k=20)
    I2, S2 = O.search_batch_cached(R, Xh, nr, Q, k=20)
    np.testing.assert_array_equal(I1, I2)
    np.testing.assert_array_equal(S1, S2)


def test_sign_scores_are_the_pm1_inner_product():
    """The popcount score d - 2 * popcount(q_signs XOR row_signs) equals the
    inner product of the +-1 sign vectors, and the 1-bit Matryoshka level
    (the code's MSB) is the sign of the rotated coordinate."""
    d, bits = 40, 4
    R = haar_rotation(d, 42)
    bnd, cent = lloyd_max_codebook(d, bits)
    rng = np.random.default_rng(9)
    X = rng.standard_normal((500, d)).astype(np.float32)
    idx, _ = O.encode(X, R, bnd)
    rot = O.rotated(X, R)
    np.testing.assert_array_equal((idx >> (bits - 1)).astype(bool), rot > 0)
    q = rng.standard_normal(d).astype(np.float32)
    qr = O.exact_q_rot(R, q)
    sq = np.where(qr > 0, 1, -1)
    sr = np.where(idx >> (bits - 1), 1, -1)
    np.testing.assert_array_equal(O.sign_scores(qr, idx, bits), sr @ sq)
    ids, sc = O.search_popcount(R, bits, idx, q, k=50)
    assert np.all(np.diff(sc) <= 0)
    ties = np.diff(sc) == 0
    assert np.all(np.diff(ids)[ties] > 0), "ties ordered by row"

"""The int8 batched kernel's candidate scheme, emulated in NumPy.

The kernel scores with 16-bit fixed point split into two int8 digits
(v = 256 hi + lo), accumulates HH = sum qhi*chi and X = sum (qhi*clo +
qlo*chi) exactly, forms v = HH + round(X / 256), and keeps the top K+32 rows
per query by float(v) * scales * norm; those are rescored exactly.  These
tests restate that arithmetic on the host and check the two facts the design
relies on: the approximate scores stay within a small absolute band of the
exact ones, and every row of the exact top K is among the approximate top
K+32 (so the exact rescoring recovers the exact top K).  They also check the
epilogue's two bounds of an 8-row group (HH + xb, then the group's largest v)
in its f32 arithmetic.
"""

import numpy as np
import pytest

from oracle import remex_oracle as O
from polarquant_b200.params import haar_rotation, lloyd_max_codebook, nested_codebooks

DIGIT_MAX = 32639
MARGIN = 32


def digits(v, mx):
    """16-bit fixed point of v (scale mx / 32639) as (hi, lo) int8 digits."""
    qi = np.clip(np.rint(v * (DIGIT_MAX / mx)), -DIGIT_MAX, DIGIT_MAX).astype(np.int64)
    hi = (qi + 128) >> 8
    return hi, qi - (hi << 8)


def approx_scores(Q, cent, codes, norms):
    mq = np.abs(Q).max(1, keepdims=True)
    qh, ql = digits(Q, mq)
    mc = np.abs(cent).max()
    ch, cl = digits(cent, mc)
    assert qh.min() >= -127 and qh.max() <= 127 and ql.min() >= -128 and ql.max() <= 127
    HH = qh @ ch[codes].T
    X = qh @ cl[codes].T + ql @ ch[codes].T
    v = HH + ((X + 128) >> 8)
    scale = (mq / DIGIT_MAX * (mc / DIGIT_MAX * 65536)).astype(np.float32)
    # the epilogue's bound: v <= HH + xb per query
    xb = (np.abs(qh).sum(1) * np.abs(cl).max() + np.abs(ql).sum(1) * np.abs(ch).max() + 128) >> 8
    assert np.all(v <= HH + xb[:, None])
    return (v.astype(np.float32) * scale) * norms.astype(np.float32)


def clustered(rng, n, d, centres, sigma):
    c = rng.standard_normal((centres, d))
    c /= np.linalg.norm(c, axis=1, keepdims=True)
    x = c[rng.integers(0, centres, n)] + rng.standard_normal((n, d)) * sigma / np.sqrt(d)
    return (x / np.linalg.norm(x, axis=1, keepdims=True)).astype(np.float32), c


@pytest.mark.parametrize("d,bits,prec,clusters", [(256, 4, 4, 0), (256, 8, 7, 0), (384, 4, 2, 64),
                                                  (512, 2, 2, 0), (1024, 4, 4, 32)])
def test_exact_topk_within_int8_candidates(d, bits, prec, clusters):
    rng = np.random.default_rng(d + bits)
    n, nq, k = 6000, 24, 64
    if clusters:
        X, cen = clustered(rng, n, d, clusters, 0.3)
        Qx = cen[rng.integers(0, clusters, nq)] + 0.3 / np.sqrt(d) * rng.standard_normal((nq, d))
        Qx = (Qx / np.linalg.norm(Qx, axis=1, keepdims=True)).astype(np.float32)
    else:
        X = rng.standard_normal((n, d)).astype(np.float32)
        X /= np.linalg.norm(X, axis=1, keepdims=True)
        Qx = rng.standard_normal((nq, d)).astype(np.float32)
        Qx /= np.linalg.norm(Qx, axis=1, keepdims=True)
    R = haar_rotation(d, 42)
    bnd, cent_full = lloyd_max_codebook(d, bits)
    cent = cent_full if prec == bits else nested_codebooks(d, bits)[prec]
    idx, norms = O.encode(X, R, bnd)
    codes = (idx >> (bits - prec)).astype(np.int64)
    Q = (Qx.astype(np.float64) @ R.T.astype(np.float64)).astype(np.float32)
    exact = (Q.astype(np.float64) @ cent[codes].T.astype(np.float64)) * norms
    approx = approx_scores(Q, cent, codes, norms)
    err = np.abs(approx - exact)
    assert err.max() < 1e-4, err.max()
    for q in range(nq):
        top = np.argsort(-exact[q], kind="stable")[:k]
        cand = set(np.argsort(-approx[q], kind="stable")[:k + MARGIN].tolist())
        assert set(top.tolist()) <= cand, q


def test_group_bounds_cover_every_score():
    """The epilogue's two bounds of an 8-row group, in the kernel's f32
    arithmetic: float(max HH + xb) * qs * (max or min norm) and
    float(max v) * qs * (max or min norm) are >= every row's
    float(v) * qs * norm, and the second is never looser than the first."""
    rng = np.random.default_rng(7)
    d, bits, n, nq = 512, 4, 4096, 8
    X = rng.standard_normal((n, d)).astype(np.float32)
    X /= np.linalg.norm(X, axis=1, keepdims=True)
    norms_all = np.exp(rng.uniform(np.log(0.5), np.log(2.0), n)).astype(np.float32)
    Q = rng.standard_normal((nq, d)).astype(np.float32)
    Q /= np.linalg.norm(Q, axis=1, keepdims=True)
    R = haar_rotation(d, 42)
    bnd, cent = lloyd_max_codebook(d, bits)
    codes, _ = O.encode(X, R, bnd)
    codes = codes.astype(np.int64)
    Qr = (Q.astype(np.float64) @ R.T.astype(np.float64)).astype(np.float32)
    mq = np.abs(Qr).max(1, keepdims=True)
    qh, ql = digits(Qr, mq)
    mc = np.abs(cent).max()
    ch, cl = digits(cent, mc)
    HH = qh @ ch[codes].T
    Xc = qh @ cl[codes].T + ql @ ch[codes].T
    v = HH + ((Xc + 128) >> 8)
    xb = (np.abs(qh).sum(1) * np.abs(cl).max() + np.abs(ql).sum(1) * np.abs(ch).max() + 128) >> 8
    qs = (mq[:, 0] / DIGIT_MAX * (mc / DIGIT_MAX * 65536)).astype(np.float32)
    f = np.float32
    for q in range(nq):
        for g0 in range(0, n, 8):
            rows = slice(g0, g0 + 8)
            nr = norms_all[rows]
            sc = (v[q, rows].astype(f) * qs[q]) * nr
            for top in (HH[q, rows].max() + xb[q], v[q, rows].max()):
                b = f(f(top) * qs[q]) * (nr.max() if top >= 0 else nr.min())
                assert np.all(sc <= b), (q, g0)
            assert v[q, rows].max() <= HH[q, rows].max() + xb[q]

"""GPU parity of the ADC scan, two-stage search, batch search and packed-row
utilities against the CPU oracle (a NumPy restatement of remex/core.py).

Corpora are encoded by the oracle on the CPU and uploaded, so these tests pin
the search kernels independently of the GPU encode.  Tolerances: scores within
1e-4 relative; top-k ids identical except where scores tie within that band.
"""

import numpy as np
import pytest

from oracle import remex_oracle as O

pytestmark = pytest.mark.gpu

RTOL = 1e-4


def unit_rows(rng, n, d):
    x = rng.standard_normal((n, d)).astype(np.float32)
    x /= np.linalg.norm(x, axis=1, keepdims=True)
    return x


def make_case(bits, d=128, n=2000, seed=42, nq=6, data_seed=42):
    from polarquant_b200 import CompressedVectors, Quantizer
    pq = Quantizer(d=d, bits=bits, seed=seed)
    rng = np.random.default_rng(data_seed)
    corpus = unit_rows(rng, n, d)
    qs = unit_rows(rng, nq, d)
    idx, norms = O.encode(corpus, pq.R, pq.boundaries)
    cv = CompressedVectors(idx, norms, d, bits)
    return pq, cv, idx, norms, qs


def assert_topk(ids, sc, ref_ids, ref_sc):
    assert len(ids) == len(ref_ids)
    assert np.all(np.diff(sc) <= 0), "scores must be descending"
    assert O.topk_equal_up_to_ties(ids, sc, ref_ids, ref_sc, rtol=RTOL), (ids, ref_ids, sc, ref_sc)


@pytest.mark.parametrize("bits", [1, 2, 3, 4, 8])
def test_search_adc_all_precisions(gpu, bits):
    pq, cv, idx, norms, qs = make_case(bits)
    for q in qs[:3]:
        for prec in [None] + list(range(1, bits + 1)):
            ri, rs = O.search_adc(pq.R, pq.centroids, pq._nested, bits, idx, norms, q, k=50,
                                  precision=prec)
            gi, gs = pq.search_adc(cv, q, k=50, precision=prec)
            assert_topk(gi, gs, ri, rs)


@pytest.mark.parametrize("bits", [4, 8])
def test_search_matches_cached(gpu, bits):
    pq, cv, idx, norms, qs = make_case(bits)
    for q in qs[:3]:
        ri, rs = O.search_cached(pq.R, pq.centroids, pq._nested, bits, idx, norms, q, k=10)
        gi, gs = pq.search(cv, q, k=10)
        assert_topk(gi, gs, ri, rs)
    assert cv._x_hat_rot is None


@pytest.mark.parametrize("bits,cands,cp", [(8, 200, None), (8, 200, 4), (4, 200, None),
                                           (4, 500, 1), (2, 100, 1), (3, 300, 2),
                                           (8, 2000, None), (8, 2048, 4)])
def test_twostage(gpu, bits, cands, cp):
    pq, cv, idx, norms, qs = make_case(bits)
    for q in qs[:3]:
        ri, rs = O.search_twostage(pq.R, pq.centroids, pq._nested, bits, idx, norms, q, k=10,
                                   candidates=cands, coarse_precision=cp)
        gi, gs = pq.search_twostage(cv, q, k=10, candidates=cands, coarse_precision=cp)
        assert_topk(gi, gs, ri, rs)


def test_twostage_candidates_n_equals_search(gpu):
    pq, cv, idx, norms, qs = make_case(8)
    for q in qs[:2]:
        i_full, _ = pq.search(cv, q, k=10)
        i_ts, _ = pq.search_twostage(cv, q, k=10, candidates=cv.n)
        np.testing.assert_array_equal(i_full, i_ts)


@pytest.mark.parametrize("bits", [1, 4, 8])
def test_search_batch(gpu, bits):
    pq, cv, idx, norms, qs = make_case(bits, nq=20)
    RI, RS = O.search_batch(pq.R, pq.centroids, pq._nested, bits, idx, norms, qs, k=25)
    GI, GS = pq.search_batch(cv, qs, k=25)
    assert GI.shape == RI.shape == (20, 25)
    for a, b, c, e in zip(GI, GS, RI, RS):
        assert_topk(a, b, c, e)


def test_matryoshka_1bit_equals_standalone_1bit(gpu):
    # remex tests/test_matryoshka.py:197-210: the MSB of an 8-bit code is the 1-bit code.
    from polarquant_b200 import CompressedVectors, Quantizer
    rng = np.random.default_rng(42)
    corpus = unit_rows(rng, 500, 128)
    qs = unit_rows(rng, 20, 128)
    pq8 = Quantizer(128, bits=8, seed=7)
    pq1 = Quantizer(128, bits=1, seed=7)
    i8, n8 = O.encode(corpus, pq8.R, pq8.boundaries)
    i1, n1 = O.encode(corpus, pq1.R, pq1.boundaries)
    a, _ = pq8.search_batch(CompressedVectors(i8, n8, 128, 8), qs, k=10, precision=1)
    b, _ = pq1.search_batch(CompressedVectors(i1, n1, 128, 1), qs, k=10)
    np.testing.assert_array_equal(a, b)


def test_packed_vectors_match_compressed(gpu):
    from polarquant_b200 import PackedVectors
    pq, cv, idx, norms, qs = make_case(4)
    pv = PackedVectors.from_compressed(cv)
    q = qs[0]
    a = pq.search_adc(cv, q, k=10)
    b = pq.search_adc(pv, q, k=10)
    np.testing.assert_array_equal(a[0], b[0])
    np.testing.assert_allclose(a[1], b[1], rtol=1e-6)
    a = pq.search_twostage(cv, q, k=10, candidates=200)
    b = pq.search_twostage(pv, q, k=10, candidates=200)
    np.testing.assert_array_equal(a[0], b[0])
    with pytest.raises(TypeError, match="PackedVectors"):
        pq.search(pv, q, k=10)
    with pytest.raises(TypeError, match="PackedVectors"):
        pq.search_batch(pv, qs, k=10)


@pytest.mark.parametrize("n", [1, 5, 7, 255, 257, 4097])
def test_edge_sizes_and_k_over_n(gpu, n):
    pq, cv, idx, norms, qs = make_case(4, d=64, n=n)
    q = qs[0]
    for k in (1, 10, n, n + 100):
        ri, rs = O.search_adc(pq.R, pq.centroids, pq._nested, 4, idx, norms, q, k=k)
        gi, gs = pq.search_adc(cv, q, k=k)
        assert len(gi) == min(k, n)
        assert_topk(gi, gs, ri, rs)
    gi, gs = pq.search_twostage(cv, q, k=3, candidates=max(1, n // 2))
    ri, rs = O.search_twostage(pq.R, pq.centroids, pq._nested, 4, idx, norms, q, k=3,
                               candidates=max(1, n // 2))
    assert_topk(gi, gs, ri, rs)


def test_empty_corpus(gpu):
    from polarquant_b200 import CompressedVectors, Quantizer
    pq = Quantizer(64, bits=4)
    cv = CompressedVectors(np.zeros((0, 64), np.uint8), np.zeros(0, np.float32), 64, 4)
    i, s = pq.search_adc(cv, np.ones(64, np.float32), k=5)
    assert i.shape == (0,) and s.shape == (0,)
    i, s = pq.search_twostage(cv, np.ones(64, np.float32), k=5)
    assert i.shape == (0,)


def test_precision_errors(gpu):
    pq, cv, idx, norms, qs = make_case(4, n=100)
    with pytest.raises(ValueError):
        pq.search(cv, qs[0], precision=0)
    with pytest.raises(ValueError):
        pq.search_adc(cv, qs[0], precision=5)
    with pytest.raises(ValueError, match="Expected d=128"):
        pq.search_adc(cv, np.ones(64, np.float32))


@pytest.mark.parametrize("bits", [1, 2, 3, 4, 8])
@pytest.mark.parametrize("d", [40, 64, 100, 384])
def test_packed_row_utilities(gpu, bits, d):
    from polarquant_b200 import CompressedVectors, PackedVectors
    rng = np.random.default_rng(bits * 1000 + d)
    n = 37
    idx = rng.integers(0, 2 ** bits, size=(n, d), dtype=np.uint8)
    norms = rng.uniform(0.5, 2, n).astype(np.float32)
    cv = CompressedVectors(idx, norms, d, bits)
    pv = PackedVectors.from_compressed(cv)
    np.testing.assert_array_equal(pv._packed, O.pack_rows(idx, bits))
    np.testing.assert_array_equal(pv.unpack_rows(0, n), idx)
    np.testing.assert_array_equal(pv.unpack_rows(3, 9), idx[3:9])
    sel = np.array([0, 5, n - 1, 2])
    np.testing.assert_array_equal(pv.unpack_at(sel), idx[sel])
    # device unpack round trip through the host view of CompressedVectors
    cv2 = pv.to_compressed()
    np.testing.assert_array_equal(cv2.indices, idx)
    np.testing.assert_array_equal(cv2.norms, norms)
    for t in range(1, bits):
        if t not in (1, 2, 3, 4):
            continue
        lo = pv.at_precision(t)
        np.testing.assert_array_equal(lo.unpack_rows(0, n), idx >> (bits - t))
        np.testing.assert_array_equal(lo._packed, O.pack_rows(idx >> (bits - t), t))
    sub = pv.subset(np.array([4, 1]))
    np.testing.assert_array_equal(sub.unpack_rows(0, 2), idx[[4, 1]])


def test_rotate_matches_f64(gpu):
    import torch
    from polarquant_b200 import Quantizer
    pq = Quantizer(384, bits=4)
    rng = np.random.default_rng(3)
    Q = rng.standard_normal((130, 384)).astype(np.float32)
    dev = torch.device("cuda")
    Y = pq._rotate(Q, dev).cpu().numpy()
    ref = (Q.astype(np.float64) @ pq.R.astype(np.float64).T)
    np.testing.assert_allclose(Y, ref, rtol=1e-6, atol=1e-6 * np.abs(ref).max())


def test_topk_merge_kernel(gpu):
    import ctypes
    import torch
    from polarquant_b200 import _lib
    from polarquant_b200.device import ptr, stream_ptr
    rng = np.random.default_rng(0)
    parts, nq, kin, k = 4, 3, 50, 37
    s = rng.standard_normal((parts, nq, kin)).astype(np.float32)
    s[1, 0, :5] = s[0, 0, :5]  # exact ties across parts
    ids = (np.arange(parts * nq * kin).reshape(parts, nq, kin)).astype(np.int64)
    ids[2, 1, 10:] = -1  # unused slots
    dev = torch.device("cuda")
    ts, ti = torch.from_numpy(s).to(dev), torch.from_numpy(ids).to(dev)
    os_, oi = torch.empty((nq, k), device=dev), torch.empty((nq, k), dtype=torch.int64,
                                                            device=dev)
    _lib.call("pq_topk_merge", ptr(ts), ptr(ti), parts, nq, kin, k, ptr(os_), ptr(oi),
              stream_ptr(dev))
    gs, gi = os_.cpu().numpy(), oi.cpu().numpy()
    for q in range(nq):
        sc = s[:, q, :].ravel()
        idq = ids[:, q, :].ravel()
        keep = idq >= 0
        order = np.lexsort((idq[keep], -sc[keep]))[:k]
        np.testing.assert_array_equal(gi[q], idq[keep][order])
        np.testing.assert_array_equal(gs[q], sc[keep][order])


def test_config1_shape_parity(gpu):
    """d=384, 4-bit, 10k unit rows (seed 42), 200 queries (seed 99), k=10."""
    from polarquant_b200 import CompressedVectors, Quantizer
    pq = Quantizer(384, bits=4, seed=42)
    corpus = unit_rows(np.random.default_rng(42), 10000, 384)
    qs = unit_rows(np.random.default_rng(99), 200, 384)
    idx, norms = O.encode(corpus, pq.R, pq.boundaries)
    cv = CompressedVectors(idx, norms, 384, 4)
    GI, GS = pq.search_adc_many(cv, qs, k=10)
    bad = 0
    for i in range(200):
        ri, rs = O.search_adc(pq.R, pq.centroids, pq._nested, 4, idx, norms, qs[i], k=10)
        bad += not O.topk_equal_up_to_ties(GI[i], GS[i], ri, rs, rtol=RTOL)
    assert bad == 0


# ---------------------------------------------------------------------------
# Tensor-core batched ADC (pq_adc_batch) and the batched coarse stage
# ---------------------------------------------------------------------------

def _batched(pq, cv, qs, k, prec, force):
    import torch
    rows = cv._device()
    qrot = pq._rotate(qs, rows.device)
    s, i = pq._scan(rows, qrot, k, pq._level(prec), force=force)
    return i.cpu().numpy(), s.cpu().numpy()


@pytest.mark.parametrize("bits", [1, 2, 3, 4, 8])
def test_batched_adc_all_precisions(gpu, bits):
    pq, cv, idx, norms, qs = make_case(bits, d=128, n=3000, nq=70)
    for prec in [None] + list(range(1, bits)):
        GI, GS = _batched(pq, cv, qs, 50, prec, "batch")
        SI, SS = _batched(pq, cv, qs, 50, prec, "scan")
        bad = 0
        for q in range(len(qs)):
            ri, rs = O.search_adc(pq.R, pq.centroids, pq._nested, bits, idx, norms, qs[q], k=50,
                                  precision=prec)
            bad += not O.topk_equal_up_to_ties(GI[q], GS[q], ri, rs, rtol=RTOL)
            assert np.all(np.diff(GS[q]) <= 0)
            np.testing.assert_allclose(GS[q], SS[q], rtol=RTOL, atol=RTOL * np.abs(SS[q]).max())
        assert bad == 0, f"{bad} queries differ at precision {prec}"


@pytest.mark.parametrize("d,n,nq,k", [(40, 77, 65, 7), (100, 1000, 130, 256), (384, 257, 64, 1),
                                      (1536, 20000, 200, 100), (768, 5000, 129, 200)])
def test_batched_adc_shapes(gpu, d, n, nq, k):
    pq, cv, idx, norms, qs = make_case(4 if d != 768 else 8, d=d, n=n, nq=nq)
    K = min(k, n)
    GI, GS = _batched(pq, cv, qs, K, None, "batch")
    assert GI.shape == (nq, K)
    bad = 0
    for q in range(nq):
        ri, rs = O.search_adc(pq.R, pq.centroids, pq._nested, pq.bits, idx, norms, qs[q], k=K)
        bad += not O.topk_equal_up_to_ties(GI[q], GS[q], ri, rs, rtol=RTOL)
    assert bad == 0


def test_search_batch_uses_tensor_cores_and_matches(gpu):
    from polarquant_b200.core import use_tensor_cores
    pq, cv, idx, norms, qs = make_case(4, d=256, n=50000, nq=100)
    # Large enough for the tensor-core path; 4,000 rows would stay on the
    # streaming scan (a batched call's fixed cost exceeds the scans').
    assert use_tensor_cores(50000, 100, 100, cv._device().row_bytes)
    assert not use_tensor_cores(4000, 100, 100, cv._device().row_bytes)
    RI, RS = O.search_batch(pq.R, pq.centroids, pq._nested, 4, idx, norms, qs, k=100)
    GI, GS = pq.search_batch(cv, qs, k=100)
    for a, b, c, e in zip(GI, GS, RI, RS):
        assert_topk(a, b, c, e)


@pytest.mark.parametrize("bits,cands,cp,d", [(8, 200, 4, 128), (4, 100, 2, 128),
                                             (8, 256, None, 128), (8, 200, 4, 1024),
                                             (4, 150, 2, 1024)])
def test_twostage_batched_coarse(gpu, bits, cands, cp, d):
    """Batched coarse stage (fp16 kernels at d=128; at d=1024 the int8 kernel,
    whose candidates are rescored exactly at the coarse precision before the
    full-precision rerank)."""
    pq, cv, idx, norms, qs = make_case(bits, d=d, n=5000, nq=80)
    GI, GS = pq.search_twostage_many(cv, qs, k=10, candidates=cands, coarse_precision=cp)
    bad = 0
    for q in range(len(qs)):
        ri, rs = O.search_twostage(pq.R, pq.centroids, pq._nested, bits, idx, norms, qs[q], k=10,
                                   candidates=cands, coarse_precision=cp)
        bad += not O.topk_equal_up_to_ties(GI[q], GS[q], ri, rs, rtol=RTOL)
    assert bad == 0


@pytest.mark.parametrize("d,bits", [(256, 1), (256, 2), (256, 3), (256, 4), (256, 8),
                                    (1024, 2), (1024, 4), (1024, 8)])
def test_batched_adc_full_query_tiles(gpu, d, bits):
    """Query batches spanning several 256-query tiles (both CTAs of each pair
    busy) over many row tiles and chunks, against the oracle's search_batch,
    three launches in a row: d=256 runs the fp16 kernels, d=1024 the int8
    kernel (2-, 4- and 8-bit codes).  These shapes exposed a timing-dependent
    loss of candidate rows when a code-tile slot was handed back to its TMA
    producer before the decoders had consumed it, and a race on the shared
    sort scratch when a one-tile task followed."""
    pq, cv, idx, norms, qs = make_case(bits, d=d, n=40000, nq=520, data_seed=bits)
    prec = max(1, bits - 1)
    RI, RS = O.search_batch(pq.R, pq.centroids, pq._nested, bits, idx, norms, qs, k=64,
                            precision=prec)
    for rep in range(3):
        GI, GS = _batched(pq, cv, qs, 64, prec, "batch")
        bad = sum(not O.topk_equal_up_to_ties(GI[q], GS[q], RI[q], RS[q], rtol=RTOL)
                  for q in range(len(qs)))
        assert bad == 0, (rep, bad)


@pytest.mark.parametrize("bits,d,k", [(8, 768, 50), (4, 768, 200), (8, 256, 200),
                                      (4, 1024, 100), (8, 1536, 64)])
def test_batched_adc_repeatable(gpu, bits, d, k):
    """Repeated launches of the batched kernel agree with the streaming scan
    every time (guards the producer/consumer hand-offs of the code-tile ring
    and the accumulator buffers, whose failures are timing dependent)."""
    pq, cv, idx, norms, qs = make_case(bits, d=d, n=5000, nq=129)
    SI, SS = _batched(pq, cv, qs, k, None, "scan")
    for rep in range(4):
        GI, GS = _batched(pq, cv, qs, k, None, "batch")
        bad = sum(not O.topk_equal_up_to_ties(GI[q], GS[q], SI[q], SS[q], rtol=RTOL)
                  for q in range(len(qs)))
        assert bad == 0, (rep, bad)


def test_small_batch_on_large_corpus_uses_tensor_cores(gpu):
    """16 queries on a corpus of 2^20+ rows take the tensor-core path by
    default (one batched pass costs a few single-query scans there) and match
    the oracle's search_adc per query."""
    from polarquant_b200 import Quantizer
    from polarquant_b200.core import use_tensor_cores
    d, n, nq, k = 64, (1 << 20) + 123, 16, 20
    rng = np.random.default_rng(11)
    X = unit_rows(rng, n, d)
    qs = unit_rows(rng, nq, d)
    pq = Quantizer(d, bits=4, seed=42)
    cv = pq.encode(X)
    assert use_tensor_cores(n, nq, k) and not use_tensor_cores(100_000, nq, k)
    GI, GS = pq.search_adc_many(cv, qs, k=k)
    idx, norms = cv.indices, cv.norms
    for q in range(nq):
        ri, rs = O.search_adc(pq.R, pq.centroids, pq._nested, 4, idx, norms, qs[q], k=k)
        assert O.topk_equal_up_to_ties(GI[q], GS[q], ri, rs, rtol=RTOL), q


@pytest.mark.parametrize("bits,cands,k,cp", [(4, 5000, 3000, 2), (8, 2500, 10, 4),
                                             (8, 2049, 2049, None)])
def test_twostage_more_than_2048_candidates(gpu, bits, cands, k, cp):
    """remex/core.py:701-704 takes any candidate count: more than the fused
    top-k limit runs the sort-based path (coarse keys of every row sorted,
    the first C rescored at full precision and sorted)."""
    pq, cv, idx, norms, qs = make_case(bits, d=96, n=12000, nq=3)
    GI, GS = pq.search_twostage_many(cv, qs, k=k, candidates=cands, coarse_precision=cp)
    assert GI.shape == (3, min(k, cands))
    for q in range(3):
        ri, rs = O.search_twostage(pq.R, pq.centroids, pq._nested, bits, idx, norms, qs[q], k=k,
                                   candidates=cands, coarse_precision=cp)
        assert_topk(GI[q], GS[q], ri, rs)

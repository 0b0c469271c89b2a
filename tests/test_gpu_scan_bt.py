"""GPU parity of the byte-table streaming scan (scan_bt_kernel: one lookup
per packed byte, tables built per query in global memory, rows streamed in
column slices) against the oracle's search_adc (remex/core.py:582-636): 1-,
2-, 4- and 8-bit codes, Matryoshka precisions (the shift folded into the
tables), rows whose bytes end inside a slice, k up to 1024, up to 64 queries,
a row count that is not a multiple of the chunk or stage.  Larger k fall
back to the other scans (checked by the diagnostic)."""

import numpy as np
import pytest

from oracle import remex_oracle as O

pytestmark = pytest.mark.gpu

RTOL = 1e-4


@pytest.mark.parametrize("bits,d,prec,k,nq", [
    (4, 384, None, 10, 3),     # two slices (192 bytes)
    (4, 384, 2, 100, 2),       # coarse precision through the tables
    (8, 200, None, 10, 2),     # 200-byte rows: the second slice ends mid-way
    (8, 200, 5, 50, 1),
    (2, 640, 1, 10, 2),
    (1, 1100, None, 20, 2),    # 138-byte rows (the last code byte half used)
    (4, 1536, None, 512, 1),   # six slices, the largest k
    (4, 256, 3, 10, 64),       # the most queries per call
])
def test_byte_table_scan_matches_oracle(gpu, bits, d, prec, k, nq):
    from polarquant_b200 import CompressedVectors, Quantizer, _lib
    n = 300_001
    rng = np.random.default_rng(bits * 100 + d)
    idx = rng.integers(0, 1 << bits, size=(n, d), dtype=np.uint8)
    norms = rng.uniform(0.5, 2.0, n).astype(np.float32)
    Q = rng.standard_normal((nq, d)).astype(np.float32)
    pq = Quantizer(d, bits=bits, seed=3)
    cv = CompressedVectors(idx, norms, d, bits)
    rows = cv._device()
    p = bits if prec is None else prec
    assert _lib.query("pq_adc_scan_kernel", n, d, bits, p, nq, k, rows.ldb) == 4
    assert _lib.query("pq_adc_scan_kernel", n, d, bits, p, nq, 513, rows.ldb) != 4
    s, i = pq._scan(rows, pq._rotate(Q, rows.device), k, p, force="scan")
    GS, GI = s.cpu().numpy(), i.cpu().numpy()
    for q in range(min(nq, 4)):
        ri, rs = O.search_adc(pq.R, pq.centroids, pq._nested, bits, idx, norms, Q[q], k=k,
                              precision=prec)
        assert np.all(np.diff(GS[q]) <= 0)
        assert O.topk_equal_up_to_ties(GI[q], GS[q], ri, rs, rtol=RTOL), q
    # Every query: the returned scores are the oracle's ADC scores of the
    # returned rows (remex/core.py:792-826).
    cent = pq.centroids if prec is None else pq._nested[prec]
    for q in range(nq):
        table = np.outer(pq.R @ Q[q], cent).astype(np.float32)
        sc = O.adc_scores(table, O.resolve_indices(idx[GI[q]], bits, prec), norms[GI[q]])
        np.testing.assert_allclose(GS[q], sc, rtol=RTOL, atol=RTOL * np.abs(sc).max())


def test_byte_table_scan_in_row_chunks(gpu):
    """64 queries over 2^20 + 777 rows of 256 bytes: the per-slice row sums
    (64 x 2 slices x 4 B per row) exceed the scan's 256 MB buffer, so the
    rows are streamed and scored in three chunks whose candidate lists share
    the merge.  Two queries against the oracle's search_adc, all of them
    through the oracle's ADC scores of the returned rows."""
    from polarquant_b200 import CompressedVectors, Quantizer, _lib
    bits, d, nq, k = 4, 512, 64, 50
    n = (1 << 20) + 777
    rng = np.random.default_rng(11)
    idx = rng.integers(0, 1 << bits, size=(n, d), dtype=np.uint8)
    norms = rng.uniform(0.5, 2.0, n).astype(np.float32)
    Q = rng.standard_normal((nq, d)).astype(np.float32)
    pq = Quantizer(d, bits=bits, seed=5)
    cv = CompressedVectors(idx, norms, d, bits)
    rows = cv._device()
    assert _lib.query("pq_adc_scan_kernel", n, d, bits, bits, nq, k, rows.ldb) == 4
    s, i = pq._scan(rows, pq._rotate(Q, rows.device), k, bits, force="scan")
    GS, GI = s.cpu().numpy(), i.cpu().numpy()
    for q in (0, nq - 1):
        ri, rs = O.search_adc(pq.R, pq.centroids, pq._nested, bits, idx, norms, Q[q], k=k)
        assert O.topk_equal_up_to_ties(GI[q], GS[q], ri, rs, rtol=RTOL), q
    for q in range(nq):
        assert np.all(np.diff(GS[q]) <= 0)
        table = np.outer(pq.R @ Q[q], pq.centroids).astype(np.float32)
        sc = O.adc_scores(table, idx[GI[q]], norms[GI[q]])
        np.testing.assert_allclose(GS[q], sc, rtol=RTOL, atol=RTOL * np.abs(sc).max())


def test_byte_table_scan_merges_chunk_lists(gpu):
    """8 queries over 140M one-bit rows of 16 bytes: the slice sums (8 x 4 B
    per row) are scored in 17 row chunks, too many for the candidate lists
    the workspace holds per query to give every chunk a full scoring grid,
    so each chunk's lists are merged into one.  Every query's result equals
    that of a single-query call (3 chunks, lists kept unmerged), and the
    scores of two queries match the oracle's ADC scores of the returned
    rows."""
    import torch
    from polarquant_b200 import Quantizer, _lib
    from polarquant_b200.core import _DeviceRows
    bits, d, nq, k = 1, 128, 8, 100
    n, ldb = 140_000_000, 16
    dev = torch.device("cuda:0")
    g = torch.Generator(device=dev)
    g.manual_seed(3)
    buf = torch.randint(0, 256, (n, ldb), dtype=torch.uint8, device=dev, generator=g)
    norms = torch.rand(n, device=dev, generator=g) + 0.5
    rows = _DeviceRows(buf, norms, n, d, bits, ldb, dev)
    assert _lib.query("pq_adc_scan_kernel", n, d, bits, bits, nq, k, ldb) == 4
    pq = Quantizer(d, bits=bits, seed=5)
    Q = np.random.default_rng(12).standard_normal((nq, d)).astype(np.float32)
    qrot = pq._rotate(Q, dev)
    s, i = pq._scan(rows, qrot, k, bits, force="scan")
    for q in range(nq):
        s1, i1 = pq._scan(rows, qrot[q:q + 1].contiguous(), k, bits, force="scan")
        assert torch.equal(i[q], i1[0]) and torch.equal(s[q], s1[0]), q
    GS, GI = s.cpu().numpy(), i.cpu().numpy()
    for q in (0, nq - 1):
        assert np.all(np.diff(GS[q]) <= 0)
        idx = O.unpack_rows(buf[i[q]].cpu().numpy(), bits, d)
        table = np.outer(pq.R @ Q[q], pq.centroids).astype(np.float32)
        sc = O.adc_scores(table, idx, norms[i[q]].cpu().numpy())
        np.testing.assert_allclose(GS[q], sc, rtol=RTOL, atol=RTOL * np.abs(sc).max())
    del buf, norms, rows
    torch.cuda.empty_cache()

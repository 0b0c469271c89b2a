"""GPU parity of the IVF coarse index (build + query path) against the
reference's golden outputs and the CPU oracle (remex/ivf.py restated)."""

import os

import numpy as np
import pytest

from oracle import remex_oracle as O

pytestmark = pytest.mark.gpu

G = os.path.join(os.path.dirname(__file__), "golden")
RTOL = 1e-4


def unit_rows(rng, n, d):
    x = rng.standard_normal((n, d)).astype(np.float32)
    x /= np.linalg.norm(x, axis=1, keepdims=True)
    return x


def golden_setup(bits, seed):
    from polarquant_b200 import CompressedVectors, Quantizer
    pq = Quantizer(128, bits=bits, seed=seed)
    rng = np.random.default_rng(42)
    corpus = unit_rows(rng, 2000, 128)
    idx, norms = O.encode(corpus, pq.R, pq.boundaries)
    return pq, CompressedVectors(idx, norms, 128, bits), idx, norms


@pytest.mark.parametrize("bits,seed", [(4, 7), (8, 11)])
@pytest.mark.parametrize("mode,nb", [("lsh", 5), ("rotated_prefix", 4), ("lsh", 8)])
def test_ivf_matches_reference_golden(gpu, bits, seed, mode, nb):
    from polarquant_b200 import IVFCoarseIndex
    z = np.load(os.path.join(G, "ivf.npz"))
    pq, cv, idx, norms = golden_setup(bits, seed)
    ix = IVFCoarseIndex(pq, cv, n_bits=nb, mode=mode, seed=0)
    tag = f"b{bits}_{mode}_n{nb}"
    np.testing.assert_array_equal(ix.cell_ids, z[f"cells_{tag}"])
    np.testing.assert_array_equal(ix.sorted_idx, z[f"sorted_{tag}"])
    np.testing.assert_array_equal(ix.cell_offsets, z[f"off_{tag}"])
    if mode == "lsh":
        np.testing.assert_array_equal(ix.hyperplanes, z[f"H_{tag}"])
    qs = z[f"queries_b{bits}"]
    for qi in range(3):
        for npb in (1, 3, ix.n_cells):
            gi, gs = ix.search_coarse(qs[qi], k=40, nprobe=npb, precision=max(1, bits - 2))
            ri, rs = z[f"coarse_{tag}_q{qi}_np{npb}_i"], z[f"coarse_{tag}_q{qi}_np{npb}_s"]
            assert O.topk_equal_up_to_ties(gi, gs, ri, rs, rtol=RTOL), (qi, npb)
            gi, gs = ix.search_twostage(qs[qi], k=10, candidates=100, nprobe=npb)
            ri, rs = z[f"ts_{tag}_q{qi}_np{npb}_i"], z[f"ts_{tag}_q{qi}_np{npb}_s"]
            assert O.topk_equal_up_to_ties(gi, gs, ri, rs, rtol=RTOL), (qi, npb)


@pytest.mark.parametrize("mode", ["lsh", "rotated_prefix"])
def test_ivf_matches_oracle_on_own_index(gpu, mode):
    """Query path parity on a larger clustered corpus, given this index's CSR."""
    from polarquant_b200 import CompressedVectors, IVFCoarseIndex, Quantizer
    d, n, nb = 384, 30000, 8
    rng = np.random.default_rng(5)
    centres = unit_rows(rng, 64, d)
    X = centres[rng.integers(0, 64, n)] + rng.standard_normal((n, d)).astype(np.float32) * (
        0.1 / np.sqrt(d))
    X /= np.linalg.norm(X, axis=1, keepdims=True)
    Q = centres[rng.integers(0, 64, 40)] + rng.standard_normal((40, d)).astype(np.float32) * (
        0.1 / np.sqrt(d))
    pq = Quantizer(d, bits=4, seed=42)
    idx, norms = O.encode(X, pq.R, pq.boundaries)
    ix = IVFCoarseIndex(pq, CompressedVectors(idx, norms, d, 4), n_bits=nb, mode=mode, seed=0)
    H = ix.hyperplanes
    # The device build equals the oracle's except for LSH projections within
    # f32 rounding of zero (none expected here).
    cells = O.ivf_cell_ids(idx, 4, nb, mode, H)
    assert (cells != ix.cell_ids).mean() < 1e-4
    srt, off = ix.sorted_idx, ix.cell_offsets
    ids, sc = ix.search_twostage_many(Q, k=10, candidates=500, nprobe=32, coarse_precision=2)
    cids, csc = ix.search_coarse_many(Q, k=200, nprobe=16, precision=2)
    for qi in range(len(Q)):
        ri, rs = O.ivf_search_twostage(pq.R, pq.centroids, pq._nested, 4, idx, norms, srt, off,
                                       nb, mode, H, Q[qi], k=10, candidates=500, nprobe=32,
                                       coarse_precision=2)
        keep = ids[qi] >= 0
        assert O.topk_equal_up_to_ties(ids[qi][keep], sc[qi][keep], ri, rs, rtol=RTOL), qi
        ri, rs = O.ivf_search_coarse(pq.R, pq.centroids, pq._nested, 4, idx, norms, srt, off,
                                     nb, mode, H, Q[qi], k=200, nprobe=16, precision=2)
        keep = cids[qi] >= 0
        assert O.topk_equal_up_to_ties(cids[qi][keep], csc[qi][keep], ri, rs, rtol=RTOL), qi


def test_ivf_full_probe_equals_flat(gpu):
    # remex tests/test_ivf.py:222-243, :299-311
    from polarquant_b200 import IVFCoarseIndex
    pq, cv, idx, norms = golden_setup(8, 11)
    ix = IVFCoarseIndex(pq, cv, n_bits=4, mode="rotated_prefix")
    qs = unit_rows(np.random.default_rng(1), 3, 128)
    for q in qs:
        a = ix.search_twostage(q, k=10, candidates=200, nprobe=ix.n_cells)
        b = pq.search_twostage(cv, q, k=10, candidates=200)
        np.testing.assert_array_equal(a[0], b[0])
        np.testing.assert_allclose(a[1], b[1], rtol=1e-5)
        a = ix.search_coarse(q, k=50, nprobe=ix.n_cells, precision=1)
        b = pq.search_adc(cv, q, k=50, precision=1)
        assert O.topk_equal_up_to_ties(a[0], a[1], b[0], b[1], rtol=RTOL)


def test_ivf_edges_and_diagnostics(gpu):
    from polarquant_b200 import IVFCoarseIndex
    pq, cv, idx, norms = golden_setup(4, 7)
    with pytest.raises(ValueError):
        IVFCoarseIndex(pq, cv, n_bits=0)
    with pytest.raises(ValueError):
        IVFCoarseIndex(pq, cv, n_bits=17)
    with pytest.raises(ValueError):
        IVFCoarseIndex(pq, cv, n_bits=4, mode="kmeans")
    with pytest.raises(TypeError):
        IVFCoarseIndex(pq, object(), n_bits=4)
    ix = IVFCoarseIndex(pq, cv, n_bits=10, mode="lsh", seed=0)
    q = unit_rows(np.random.default_rng(2), 1, 128)[0]
    i, s = ix.search_coarse(q, k=10_000 if False else 2048, nprobe=1)
    c = ix.query_cell(q)
    assert len(i) == min(2048, ix.cell_offsets[c + 1] - ix.cell_offsets[c])
    assert len(np.unique(i)) == len(i)
    i, s = ix.search_coarse(q, k=10, nprobe=0)
    assert len(i) == 0
    np.testing.assert_array_equal(ix.probe_cells(13, 1), [13])
    cells = ix.probe_cells(13, 11)
    assert cells[0] == 13 and set(cells[1:].tolist()) == {13 ^ (1 << b) for b in range(10)}
    st = ix.cell_size_stats()
    assert st["n_cells"] == 1024 and int(np.diff(ix.cell_offsets).sum()) == cv.n
    assert ix.index_nbytes > 0 and ix.candidate_count(q, 3) >= 0
    rp = IVFCoarseIndex(pq, cv, n_bits=6, mode="rotated_prefix")
    assert rp.index_nbytes < IVFCoarseIndex(pq, cv, n_bits=6, mode="lsh").index_nbytes


@pytest.mark.parametrize("mode", ["lsh", "rotated_prefix"])
def test_ivf_more_than_2048_candidates_and_k(gpu, mode):
    """remex/ivf.py:301-436 takes any k / candidate count: above the fused
    limit the probed rows are sorted by coarse score instead."""
    from polarquant_b200 import CompressedVectors, IVFCoarseIndex, Quantizer
    d, n, nb = 128, 40000, 6
    rng = np.random.default_rng(8)
    X = unit_rows(rng, n, d)
    Q = unit_rows(rng, 3, d)
    pq = Quantizer(d, bits=4, seed=42)
    idx, norms = O.encode(X, pq.R, pq.boundaries)
    ix = IVFCoarseIndex(pq, CompressedVectors(idx, norms, d, 4), n_bits=nb, mode=mode, seed=0)
    H, srt, off = ix.hyperplanes, ix.sorted_idx, ix.cell_offsets
    for q in Q:
        gi, gs = ix.search_coarse(q, k=3000, nprobe=7, precision=2)
        ri, rs = O.ivf_search_coarse(pq.R, pq.centroids, pq._nested, 4, idx, norms, srt, off, nb,
                                     mode, H, q, k=3000, nprobe=7, precision=2)
        assert O.topk_equal_up_to_ties(gi, gs, ri, rs, rtol=RTOL)
        gi, gs = ix.search_twostage(q, k=2100, candidates=5000, nprobe=9, coarse_precision=1)
        ri, rs = O.ivf_search_twostage(pq.R, pq.centroids, pq._nested, 4, idx, norms, srt, off,
                                       nb, mode, H, q, k=2100, candidates=5000, nprobe=9,
                                       coarse_precision=1)
        assert O.topk_equal_up_to_ties(gi, gs, ri, rs, rtol=RTOL)
        # One probed cell of fewer rows than asked for: every row, -1 slots trimmed.
        gi, gs = ix.search_twostage(q, k=10, candidates=4000, nprobe=1)
        ri, rs = O.ivf_search_twostage(pq.R, pq.centroids, pq._nested, 4, idx, norms, srt, off,
                                       nb, mode, H, q, k=10, candidates=4000, nprobe=1)
        assert O.topk_equal_up_to_ties(gi, gs, ri, rs, rtol=RTOL)
    i, s = ix.search_twostage(Q[0], k=10, candidates=0, nprobe=3)
    assert i.shape == (0,) and s.shape == (0,)


@pytest.mark.parametrize("n,nb", [(50000, 12), (70001, 14), (40000, 15), (30000, 16), (5, 3)])
def test_ivf_csr_build_matches_stable_argsort(gpu, n, nb):
    """pq_ivf_build_csr (stable counting sort on the device) against
    remex/ivf.py:216-224 (argsort kind='stable', bincount, cumsum), for cell
    counts that use the shared-memory counters (<= 2^14 cells) and the global
    ones, with skewed cell sizes, and the CSR-order copy of rows and norms."""
    import torch
    from polarquant_b200 import _lib
    from polarquant_b200.device import ptr, stream_ptr, workspace
    rng = np.random.default_rng(nb)
    n_cells = 1 << nb
    # Skewed: half the rows in a few cells, the rest spread out.
    cells = np.where(rng.random(n) < 0.5, rng.integers(0, 7, n),
                     rng.integers(0, n_cells, n)).astype(np.uint16)
    ldb = 32
    rows = rng.integers(0, 256, size=(n, ldb), dtype=np.uint8)
    norms = rng.random(n).astype(np.float32)
    dev = torch.device("cuda")
    c_d = torch.from_numpy(cells.view(np.int16)).to(dev)
    r_d = torch.from_numpy(rows.ravel()).to(dev)
    n_d = torch.from_numpy(norms).to(dev)
    srt = torch.empty(n, dtype=torch.int64, device=dev)
    off = torch.empty(n_cells + 1, dtype=torch.int64, device=dev)
    cr = torch.empty(n * ldb, dtype=torch.uint8, device=dev)
    cn = torch.empty(n, dtype=torch.float32, device=dev)
    ws = workspace(_lib.query("pq_ivf_csr_workspace_bytes", n, nb), dev)
    _lib.call("pq_ivf_build_csr", ptr(c_d), n, nb, ptr(srt), ptr(off), ptr(r_d), ldb, ptr(n_d),
              ptr(cr), ptr(cn), ptr(ws), ws.numel(), stream_ptr(dev))
    ref_s, ref_o = O.ivf_csr(cells, n_cells)
    np.testing.assert_array_equal(srt.cpu().numpy(), ref_s)
    np.testing.assert_array_equal(off.cpu().numpy(), ref_o)
    np.testing.assert_array_equal(cr.cpu().numpy().reshape(n, ldb), rows[ref_s])
    np.testing.assert_array_equal(cn.cpu().numpy(), norms[ref_s])

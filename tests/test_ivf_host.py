"""Host-side logic of IVFCoarseIndex on the CPU (remex/ivf.py): argument
checks (remex/ivf.py:99-130, the reference's tests/test_ivf.py construction
cases), the LSH hyperplanes against the reference's own (tests/golden/ivf.npz),
and the query-cell hash, Hamming-ranked probe order and CSR candidate lists
against the oracle.  The device build is skipped here (it runs in
test_gpu_ivf.py); these paths do not touch the GPU."""

import os

import numpy as np
import pytest

from oracle import remex_oracle as O
from polarquant_b200 import CompressedVectors, IVFCoarseIndex, Quantizer

G = os.path.join(os.path.dirname(__file__), "golden")


@pytest.fixture
def host_index(monkeypatch):
    """IVFCoarseIndex(...) with the device build replaced by a no-op."""
    monkeypatch.setattr(IVFCoarseIndex, "_build", lambda self: None)

    def make(d=128, bits=4, n_bits=5, mode="lsh", seed=0, n=10):
        pq = Quantizer(d, bits=bits, seed=7)
        rng = np.random.default_rng(1)
        cv = CompressedVectors(rng.integers(0, 1 << bits, (n, d)).astype(np.uint8),
                               np.ones(n, np.float32), d, bits)
        return IVFCoarseIndex(pq, cv, n_bits=n_bits, mode=mode, seed=seed)
    return make


def test_argument_checks():
    pq = Quantizer(8, bits=4, seed=0)
    cv = CompressedVectors(np.zeros((3, 8), np.uint8), np.ones(3, np.float32), 8, 4)
    for nb in (0, 17):
        with pytest.raises(ValueError, match="n_bits must be 1-16"):
            IVFCoarseIndex(pq, cv, n_bits=nb, mode="lsh")
    with pytest.raises(ValueError, match="mode must be one of"):
        IVFCoarseIndex(pq, cv, n_bits=4, mode="kmeans")
    with pytest.raises(ValueError, match="exceeds quantizer.d"):
        IVFCoarseIndex(pq, cv, n_bits=9, mode="rotated_prefix")
    with pytest.raises(TypeError, match="CompressedVectors or PackedVectors"):
        IVFCoarseIndex(pq, object(), n_bits=4, mode="lsh")


@pytest.mark.parametrize("nb", [5, 8])
def test_lsh_hyperplanes_match_reference(host_index, nb):
    z = np.load(os.path.join(G, "ivf.npz"))
    for bits in (4, 8):
        ix = host_index(d=128, bits=bits, n_bits=nb, mode="lsh", seed=0)
        assert ix.hyperplanes.dtype == np.float32 and ix.hyperplanes.shape == (nb, 128)
        np.testing.assert_array_equal(ix.hyperplanes, z[f"H_b{bits}_lsh_n{nb}"])


def test_lsh_seeds_and_prefix_mode(host_index):
    a = host_index(n_bits=6, seed=3).hyperplanes
    np.testing.assert_array_equal(a, host_index(n_bits=6, seed=3).hyperplanes)
    assert not np.array_equal(a, host_index(n_bits=6, seed=4).hyperplanes)
    np.testing.assert_array_equal(a, O.lsh_hyperplanes(6, 128, 3))
    ix = host_index(n_bits=4, mode="rotated_prefix")
    assert ix.hyperplanes is None and ix.n_cells == 16


@pytest.mark.parametrize("mode", ["lsh", "rotated_prefix"])
@pytest.mark.parametrize("nb", [1, 5, 12])
def test_query_cell_matches_oracle(host_index, mode, nb):
    ix = host_index(n_bits=nb, mode=mode, seed=2)
    rng = np.random.default_rng(nb)
    for _ in range(50):
        q = rng.standard_normal(128).astype(np.float32)
        want = O.ivf_query_cell(q, nb, mode, ix.hyperplanes)
        got = ix._query_cell_from_rot(q)
        assert got == want and 0 <= got < ix.n_cells


@pytest.mark.parametrize("nb", [1, 4, 5, 8, 12])
def test_probe_order_matches_oracle(host_index, nb):
    ix = host_index(n_bits=nb)
    n_cells = 1 << nb
    rng = np.random.default_rng(nb)
    for qc in rng.integers(0, n_cells, 6):
        for npb in (0, 1, 3, n_cells - 1, n_cells, n_cells + 5):
            got = ix.probe_cells(int(qc), npb)
            np.testing.assert_array_equal(got, O.ivf_probe_cells(int(qc), npb, n_cells))
        full = ix.probe_cells(int(qc), n_cells - 1)
        if len(full):
            assert full[0] == qc
            hd = [bin(int(c) ^ int(qc)).count("1") for c in full]
            assert hd == sorted(hd)


def test_candidate_lists_match_oracle(host_index):
    ix = host_index(n_bits=5)
    rng = np.random.default_rng(9)
    cells = rng.integers(0, 32, 400).astype(np.uint16)
    srt, off = O.ivf_csr(cells, 32)
    ix._h_sorted, ix._h_offsets = srt, off
    for qc in range(0, 32, 5):
        for npb in (0, 1, 4, 32):
            want = O.ivf_candidates(srt, off, O.ivf_probe_cells(qc, npb, 32))
            np.testing.assert_array_equal(ix.candidate_indices(qc, npb), want)

"""GPU parity of the tcgen05 encode (norm, normalise, rotate, Lloyd-Max code,
bit-pack), decode and tensor-core rotation against the reference's golden
outputs and the CPU oracle.

Parity rule for codes: bit-exact except coordinates whose rotated value lies
within 1e-6 of a Lloyd-Max boundary (where the reference's own f32 sgemm
rounding decides the side); such flips must be <= 1e-5 of all coordinates at
<= 4 bits.  At 8 bits the boundaries are so dense that the reference's f32
rounding alone flips ~1.0e-5 of coordinates against an exact product (the
floor for any other summation order), so the budget there is 2e-5 (each flip
still within 1e-6 of a boundary and to the neighbouring level).
Norms: identical f32 values (computed in f64 exactly as the reference).
"""

import os

import numpy as np
import pytest

from oracle import remex_oracle as O

pytestmark = pytest.mark.gpu

G = os.path.join(os.path.dirname(__file__), "golden")


def check_codes(got, ref, X, R, bnd, bits, budget=None):
    diff = got != ref
    nflip = int(diff.sum())
    if budget is None:
        budget = 1e-5 if bits <= 4 else 2e-5
    if nflip:
        rot = O.rotated(X, R)
        dist = O.boundary_distance(rot[diff], bnd)
        assert dist.max() <= 1e-6, f"flip {dist.max():.3g} away from a boundary"
        # a flip may only move to the neighbouring level
        assert np.abs(got[diff].astype(int) - ref[diff].astype(int)).max() == 1
    assert nflip <= max(1, budget * got.size), f"{nflip} flips of {got.size}"
    return nflip


@pytest.mark.parametrize("case", [(64, 300, 42, 1), (128, 500, 7, 2), (384, 400, 42, 3),
                                  (40, 77, 3, 4)])
@pytest.mark.parametrize("bits", [1, 2, 3, 4, 8])
def test_encode_matches_reference_golden(gpu, case, bits):
    from polarquant_b200 import PackedVectors, Quantizer
    d, n, seed, xseed = case
    rng = np.random.default_rng(xseed)
    X = (rng.standard_normal((n, d)) * rng.uniform(0.2, 3.0, (n, 1))).astype(np.float32)
    X[0] = 0.0
    z = np.load(os.path.join(G, "encode.npz"))
    key = f"d{d}_n{n}_s{seed}_x{xseed}_b{bits}"
    pq = Quantizer(d, bits=bits, seed=seed)
    cv = pq.encode(X)
    np.testing.assert_array_equal(cv.norms, z[f"norms_{key}"])
    check_codes(cv.indices, z[f"idx_{key}"], X, pq.R, pq.boundaries, bits)
    pv = PackedVectors.from_compressed(cv)
    if not (cv.indices != z[f"idx_{key}"]).any():
        np.testing.assert_array_equal(pv._packed, z[f"rows_{key}"])


@pytest.mark.parametrize("bits", [2, 3, 4, 8])
def test_encode_d1024_lognormal_norms(gpu, bits):
    """Config 3 distribution (N(0, I) rows scaled log-uniform in [0.5, 2]) at d=1024."""
    from polarquant_b200 import Quantizer
    d, n = 1024, 20000
    rng = np.random.default_rng(100 + bits)
    X = rng.standard_normal((n, d)).astype(np.float32)
    X /= np.linalg.norm(X, axis=1, keepdims=True)
    X *= np.exp(rng.uniform(np.log(0.5), np.log(2.0), (n, 1))).astype(np.float32)
    pq = Quantizer(d, bits=bits, seed=42)
    cv = pq.encode(X)
    ref, norms = O.encode(X, pq.R, pq.boundaries)
    np.testing.assert_array_equal(cv.norms, norms)
    check_codes(cv.indices, ref, X, pq.R, pq.boundaries, bits)


@pytest.mark.parametrize("d,bits", [(384, 4), (768, 4), (1536, 4), (600, 4), (600, 3),
                                    (200, 8)])
def test_encode_other_dims(gpu, d, bits):
    """Dimensions whose rotation output is split over several column tiles,
    including widths where a tile is not a whole number of 64 columns (d=600:
    three tiles of 224 columns, the last one ragged)."""
    from polarquant_b200 import Quantizer
    n = 3000
    rng = np.random.default_rng(d)
    X = rng.standard_normal((n, d)).astype(np.float32)
    pq = Quantizer(d, bits=bits, seed=42)
    cv = pq.encode(X)
    ref, norms = O.encode(X, pq.R, pq.boundaries)
    np.testing.assert_array_equal(cv.norms, norms)
    check_codes(cv.indices, ref, X, pq.R, pq.boundaries, bits)


def test_encode_tile_edges_and_tensor_input(gpu):
    import torch
    from polarquant_b200 import Quantizer
    pq = Quantizer(128, bits=4, seed=1)
    rng = np.random.default_rng(5)
    for n in (1, 127, 128, 129, 1000):
        X = rng.standard_normal((n, 128)).astype(np.float32)
        cv = pq.encode(torch.from_numpy(X).cuda())
        ref, norms = O.encode(X, pq.R, pq.boundaries)
        np.testing.assert_array_equal(cv.norms, norms)
        check_codes(cv.indices, ref, X, pq.R, pq.boundaries, 4)
    one = pq.encode(rng.standard_normal(128).astype(np.float32))
    assert one.n == 1
    empty = pq.encode(np.empty((0, 128), np.float32))
    assert empty.n == 0 and empty.indices.shape == (0, 128)
    with pytest.raises(ValueError, match="Expected d=128"):
        pq.encode(np.zeros((10, 64), np.float32))


def test_encode_deterministic_and_chunked(gpu):
    """Two runs give identical bytes; a corpus larger than one encode chunk too."""
    from polarquant_b200 import Quantizer
    pq = Quantizer(64, bits=3, seed=42)
    rng = np.random.default_rng(9)
    X = rng.standard_normal((140000, 64)).astype(np.float32)
    a = pq.encode(X)
    b = pq.encode(X)
    np.testing.assert_array_equal(a._rows.rows_host(), b._rows.rows_host())
    ref, norms = O.encode(X, pq.R, pq.boundaries)
    np.testing.assert_array_equal(a.norms, norms)
    check_codes(a.indices, ref, X, pq.R, pq.boundaries, 3)


@pytest.mark.parametrize("bits", [2, 4, 8])
def test_decode_and_mse(gpu, bits):
    from polarquant_b200 import Quantizer
    d, n = 256, 500
    rng = np.random.default_rng(3)
    X = rng.standard_normal((n, d)).astype(np.float32)
    pq = Quantizer(d, bits=bits, seed=0)
    cv = pq.encode(X)
    idx, norms = cv.indices, cv.norms
    for p in [None] + list(range(1, bits)):
        cent = pq.centroids if p is None else pq._nested[p]
        ref = (cent[O.resolve_indices(idx, bits, p)] @ pq.R) * norms[:, None]
        got = pq.decode(cv, precision=p)
        np.testing.assert_allclose(got, ref, rtol=1e-5, atol=1e-6 * np.abs(ref).max())
    mses = [pq.mse(X[:50], precision=p) for p in range(1, bits + 1)]
    assert all(mses[i] >= mses[i + 1] for i in range(len(mses) - 1))


def test_rotate_tc_matches_f64(gpu):
    from polarquant_b200 import Quantizer
    from polarquant_b200.encode import rotate_tc
    pq = Quantizer(1024, bits=4)
    rng = np.random.default_rng(11)
    Q = rng.standard_normal((777, 1024)).astype(np.float32) * 3.0
    Y = rotate_tc(pq, Q).cpu().numpy()
    ref = Q.astype(np.float64) @ pq.R.astype(np.float64).T
    err = np.abs(Y - ref) / (np.abs(Q).max(1, keepdims=True) * np.sqrt(1024))
    assert err.max() < 1e-6, err.max()


def test_encode_then_search_end_to_end(gpu):
    """Config 1 shape through the public API: encode on the GPU, then search."""
    from polarquant_b200 import Quantizer
    d = 384
    X = np.random.default_rng(42).standard_normal((10000, d)).astype(np.float32)
    X /= np.linalg.norm(X, axis=1, keepdims=True)
    Q = np.random.default_rng(99).standard_normal((20, d)).astype(np.float32)
    Q /= np.linalg.norm(Q, axis=1, keepdims=True)
    pq = Quantizer(d, bits=4, seed=42)
    cv = pq.encode(X)
    idx, norms = O.encode(X, pq.R, pq.boundaries)
    check_codes(cv.indices, idx, X, pq.R, pq.boundaries, 4)
    gidx = cv.indices  # search parity on the codes the GPU produced
    for q in Q:
        gi, gs = pq.search_adc(cv, q, k=10)
        ri, rs = O.search_adc(pq.R, pq.centroids, pq._nested, 4, gidx, cv.norms, q, k=10)
        assert O.topk_equal_up_to_ties(gi, gs, ri, rs, rtol=1e-4)


def test_save_load_roundtrip(gpu, tmp_path):
    from polarquant_b200 import CompressedVectors, PackedVectors, Quantizer
    for bits in (1, 2, 3, 4, 8):
        for d in (64, 40):
            pq = Quantizer(d, bits=bits)
            X = np.random.default_rng(bits).standard_normal((50, d)).astype(np.float32)
            cv = pq.encode(X)
            p = str(tmp_path / f"c{bits}_{d}.npz")
            cv.save(p)
            z = np.load(p)
            np.testing.assert_array_equal(z["packed_indices"], O.pack(cv.indices.ravel(), bits))
            lo = CompressedVectors.load(p)
            np.testing.assert_array_equal(lo.indices, cv.indices)
            np.testing.assert_array_equal(lo.norms, cv.norms)
            assert (lo.d, lo.bits, lo.n) == (d, bits, 50)
            pv = PackedVectors.from_compressed(cv)
            p2 = str(tmp_path / f"p{bits}_{d}.npz")
            pv.save(p2)
            lp = PackedVectors.load(p2)
            np.testing.assert_array_equal(lp.unpack_rows(0, 50), cv.indices)


@pytest.mark.parametrize("bits,d", [(4, 64), (3, 40), (8, 24), (2, 20)])
def test_pq_file_from_device_rows(gpu, tmp_path, bits, d):
    """A corpus encoded on the GPU writes the same .pq bytes as the host packers
    (rows streamed straight from the device when they are whole bytes), and a
    loaded file searches like the original."""
    from polarquant_b200 import CompressedVectors, Quantizer, load_pq, save_pq
    rng = np.random.default_rng(bits)
    X = rng.standard_normal((500, d)).astype(np.float32)
    pq = Quantizer(d, bits=bits, seed=42)
    cv = pq.encode(X)
    a, b = tmp_path / "dev.pq", tmp_path / "host.pq"
    save_pq(a, cv)
    save_pq(b, CompressedVectors(cv.indices, cv.norms, d, bits))
    assert a.read_bytes() == b.read_bytes()
    back = load_pq(a)
    q = X[3]
    i0, s0 = pq.search_adc(cv, q, k=10)
    i1, s1 = pq.search_adc(back, q, k=10)
    np.testing.assert_array_equal(i0, i1)
    np.testing.assert_array_equal(s0, s1)


@pytest.mark.parametrize("bits,d", [(4, 256), (8, 128), (3, 200)])
def test_encode_several_chunks(gpu, bits, d):
    """Calls spanning several 131,072-row chunks run as a pipeline (the
    normalise/split of chunk i+1 and the near-boundary fix-ups of chunk i-1 on
    a side stream while chunk i's GEMM runs), with ping-pong plane buffers;
    results must equal the one-chunk path's parity: norms bit-identical,
    codes within the boundary rule, and the tensor-core rotation likewise."""
    from polarquant_b200 import Quantizer
    from polarquant_b200.encode import rotate_tc
    n = 3 * 131072 + 1234
    rng = np.random.default_rng(bits * 7 + d)
    X = rng.standard_normal((n, d)).astype(np.float32)
    X *= np.exp(rng.uniform(np.log(0.5), np.log(2.0), (n, 1))).astype(np.float32)
    pq = Quantizer(d, bits=bits, seed=42)
    cv = pq.encode(X)
    ref, norms = O.encode(X, pq.R, pq.boundaries)
    np.testing.assert_array_equal(cv.norms, norms)
    check_codes(cv.indices, ref, X, pq.R, pq.boundaries, bits)
    # Twice more in a row: buffers and events are reused across calls.
    for _ in range(2):
        cv2 = pq.encode(X)
        np.testing.assert_array_equal(cv2.indices, cv.indices)
    Y = rotate_tc(pq, X).cpu().numpy()
    rows = np.r_[0:5, 131070:131075, n - 5:n]
    exact = X[rows].astype(np.float64) @ pq.R.astype(np.float64).T
    np.testing.assert_allclose(Y[rows], exact, rtol=1e-6, atol=1e-6 * np.abs(exact).max())

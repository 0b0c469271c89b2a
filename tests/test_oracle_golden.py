"""Pins the CPU oracle, the host parameter build and the host packing to the
reference's own outputs (fixtures written by tests/golden/make_golden.py,
which imports the reference package), plus the reference's RNG known answers.
CPU only."""

import hashlib
import json
import os

import numpy as np
import pytest

from oracle import remex_oracle as O

G = os.path.join(os.path.dirname(__file__), "golden")


def load(name):
    return np.load(os.path.join(G, name))


def meta():
    with open(os.path.join(G, "golden_meta.json")) as f:
        return json.load(f)


def sha(a):
    return hashlib.sha256(np.ascontiguousarray(a).tobytes()).hexdigest()


def test_rng_known_answers():
    # remex/mojo/tests/fixtures/{normal_f64,raw_u64}_seed42.bin: the generator
    # behind haar_rotation (remex/rotation.py:72-73).
    z = load("rng_seed42.npz")
    np.testing.assert_array_equal(np.random.default_rng(42).standard_normal(1000), z["normals"])
    np.testing.assert_array_equal(np.random.default_rng(42).bit_generator.random_raw(1000),
                                  z["raw"])


@pytest.mark.parametrize("d", [8, 64, 128])
@pytest.mark.parametrize("seed", [0, 7, 11, 42])
def test_rotation_small(d, seed):
    from polarquant_b200.params import haar_rotation
    z = load("params.npz")
    np.testing.assert_array_equal(O.haar_rotation(d, seed), z[f"R_d{d}_s{seed}"])
    np.testing.assert_array_equal(haar_rotation(d, seed), z[f"R_d{d}_s{seed}"])


@pytest.mark.parametrize("key", ["R_d256_s0", "R_d256_s42", "R_d384_s42", "R_d384_s0",
                                 "R_d768_s42", "R_d1024_s42", "R_d1536_s42"])
def test_rotation_large_digest(key):
    from polarquant_b200.params import haar_rotation
    d, s = key[3:].split("_s")
    assert sha(haar_rotation(int(d), int(s))) == meta()["R_sha256"][key]


@pytest.mark.parametrize("d", [8, 64, 128, 256, 384, 768, 1024, 1536])
@pytest.mark.parametrize("bits", [1, 2, 3, 4, 8])
def test_codebooks(d, bits):
    from polarquant_b200.params import lloyd_max_codebook, nested_codebooks
    z = load("params.npz")
    b, c = lloyd_max_codebook(d, bits)
    np.testing.assert_array_equal(b, z[f"bounds_d{d}_b{bits}"])
    np.testing.assert_array_equal(c, z[f"cent_d{d}_b{bits}"])
    nest = nested_codebooks(d, bits)
    assert sorted(nest) == list(range(1, bits + 1))
    for p in range(1, bits + 1):
        np.testing.assert_array_equal(nest[p], z[f"nested_d{d}_b{bits}_p{p}"])
    if bits <= 3 and d <= 128:  # the oracle's scalar loop is slow; spot-check it
        ob, oc = O.lloyd_max_codebook(d, bits)
        np.testing.assert_array_equal(ob, b)
        np.testing.assert_array_equal(oc, c)
        on = O.nested_codebooks(d, bits)
        for p in on:
            np.testing.assert_array_equal(on[p], nest[p])


ENC_CASES = [(64, 300, 42, 1), (128, 500, 7, 2), (384, 400, 42, 3), (40, 77, 3, 4)]


def enc_inputs(d, n, xseed):
    rng = np.random.default_rng(xseed)
    X = (rng.standard_normal((n, d)) * rng.uniform(0.2, 3.0, (n, 1))).astype(np.float32)
    X[0] = 0.0
    assert sha(X) == meta()["encode_inputs_sha256"][f"X_d{d}_n{n}_x{xseed}"]
    return X


@pytest.mark.parametrize("case", ENC_CASES)
@pytest.mark.parametrize("bits", [1, 2, 3, 4, 8])
def test_oracle_encode_and_packing(case, bits):
    from polarquant_b200 import packing as HP
    from polarquant_b200.params import haar_rotation, lloyd_max_codebook
    d, n, seed, xseed = case
    X = enc_inputs(d, n, xseed)
    z = load("encode.npz")
    key = f"d{d}_n{n}_s{seed}_x{xseed}_b{bits}"
    R = haar_rotation(d, seed)
    bnd, _ = lloyd_max_codebook(d, bits)
    idx, norms = O.encode(X, R, bnd)
    np.testing.assert_array_equal(idx, z[f"idx_{key}"])
    np.testing.assert_array_equal(norms, z[f"norms_{key}"])
    flat, rows = z[f"flat_{key}"], z[f"rows_{key}"]
    np.testing.assert_array_equal(O.pack(idx.ravel(), bits), flat)
    np.testing.assert_array_equal(O.pack_rows(idx, bits), rows)
    np.testing.assert_array_equal(O.unpack(flat, bits, n * d).reshape(n, d), idx)
    np.testing.assert_array_equal(O.unpack_rows(rows, bits, d), idx)
    # host packing of the product
    np.testing.assert_array_equal(HP.pack(idx, bits), flat)
    np.testing.assert_array_equal(HP.pack_rows(idx, bits), rows)
    np.testing.assert_array_equal(HP.unpack(flat, bits, n * d).reshape(n, d), idx)
    np.testing.assert_array_equal(HP.unpack_rows(rows, bits, d), idx)
    assert HP.packed_nbytes(n, d, bits) == len(flat) == O.packed_nbytes(n, d, bits)


SEARCH_CASES = [(4, 42), (8, 42), (2, 5), (3, 9), (1, 3)]


def search_case(bits, seed):
    from polarquant_b200.params import haar_rotation, lloyd_max_codebook, nested_codebooks
    z = load("search.npz")
    tag = f"b{bits}"
    R = haar_rotation(128, seed)
    _, cent = lloyd_max_codebook(128, bits)
    nest = nested_codebooks(128, bits)
    return z, tag, R, cent, nest


@pytest.mark.parametrize("bits,seed", SEARCH_CASES)
def test_oracle_search_matches_reference(bits, seed):
    z, tag, R, cent, nest = search_case(bits, seed)
    idx, norms, qs = z[f"idx_{tag}"], z[f"norms_{tag}"], z[f"queries_{tag}"]
    for qi in range(4):
        q = qs[qi]
        for prec in [None] + list(range(1, bits)):
            pn = "full" if prec is None else str(prec)
            i, s = O.search_adc(R, cent, nest, bits, idx, norms, q, k=50, precision=prec)
            np.testing.assert_array_equal(s, z[f"adc_{tag}_q{qi}_p{pn}_s"])
            assert O.topk_equal_up_to_ties(i, s, z[f"adc_{tag}_q{qi}_p{pn}_i"],
                                           z[f"adc_{tag}_q{qi}_p{pn}_s"], rtol=0)
        i, s = O.search_cached(R, cent, nest, bits, idx, norms, q, k=10)
        np.testing.assert_array_equal(s, z[f"cached_{tag}_q{qi}_s"])
        for C in (200, 2000):
            i, s = O.search_twostage(R, cent, nest, bits, idx, norms, q, k=10, candidates=C)
            np.testing.assert_array_equal(s, z[f"ts_{tag}_q{qi}_C{C}_s"])
            assert set(i.tolist()) == set(z[f"ts_{tag}_q{qi}_C{C}_i"].tolist()) or \
                O.topk_equal_up_to_ties(i, s, z[f"ts_{tag}_q{qi}_C{C}_i"],
                                        z[f"ts_{tag}_q{qi}_C{C}_s"], rtol=0)
    I, S = O.search_batch(R, cent, nest, bits, idx, norms, qs, k=25)
    np.testing.assert_array_equal(S, z[f"batch_{tag}_s"])


@pytest.mark.parametrize("bits,seed", [(4, 7), (8, 11)])
@pytest.mark.parametrize("mode,nb", [("lsh", 5), ("rotated_prefix", 4), ("lsh", 8)])
def test_oracle_ivf_matches_reference(bits, seed, mode, nb):
    from polarquant_b200.params import haar_rotation, lloyd_max_codebook, nested_codebooks
    z = load("ivf.npz")
    R = haar_rotation(128, seed)
    bnd, cent = lloyd_max_codebook(128, bits)
    nest = nested_codebooks(128, bits)
    rng = np.random.default_rng(42)
    corpus = rng.standard_normal((2000, 128)).astype(np.float32)
    corpus /= np.linalg.norm(corpus, axis=1, keepdims=True)
    qs = z[f"queries_b{bits}"]
    idx, norms = O.encode(corpus, R, bnd)
    tag = f"b{bits}_{mode}_n{nb}"
    H = O.lsh_hyperplanes(nb, 128, 0) if mode == "lsh" else None
    if H is not None:
        np.testing.assert_array_equal(H, z[f"H_{tag}"])
    cells = O.ivf_cell_ids(idx, bits, nb, mode, H)
    np.testing.assert_array_equal(cells, z[f"cells_{tag}"])
    srt, off = O.ivf_csr(cells, 1 << nb)
    np.testing.assert_array_equal(srt, z[f"sorted_{tag}"])
    np.testing.assert_array_equal(off, z[f"off_{tag}"])
    for qi in range(3):
        for npb in (1, 3, 1 << nb):
            i, s = O.ivf_search_coarse(R, cent, nest, bits, idx, norms, srt, off, nb, mode, H,
                                       qs[qi], k=40, nprobe=npb, precision=max(1, bits - 2))
            np.testing.assert_array_equal(s, z[f"coarse_{tag}_q{qi}_np{npb}_s"])
            i, s = O.ivf_search_twostage(R, cent, nest, bits, idx, norms, srt, off, nb, mode,
                                         H, qs[qi], k=10, candidates=100, nprobe=npb)
            np.testing.assert_array_equal(s, z[f"ts_{tag}_q{qi}_np{npb}_s"])
            assert O.topk_equal_up_to_ties(i, s, z[f"ts_{tag}_q{qi}_np{npb}_i"],
                                           z[f"ts_{tag}_q{qi}_np{npb}_s"], rtol=0)


def test_topk_helper_plants_mismatch():
    # The parity helper must reject a wrong id away from the k-th score.
    s = np.array([0.9, 0.8, 0.5], np.float32)
    assert O.topk_equal_up_to_ties([1, 2, 3], s, [1, 2, 3], s)
    assert not O.topk_equal_up_to_ties([1, 2, 4], s, [1, 3, 2], s)
    assert O.topk_equal_up_to_ties([1, 2, 4], s, [1, 2, 3], s)  # tie at the k-th
    assert not O.topk_equal_up_to_ties([1, 2, 3], s * 1.01, [1, 2, 3], s)

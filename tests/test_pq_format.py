"""The `.pq` / `.params` files (remex/pq_format.py) against files written by the
reference itself (tests/golden/pq_files.npz, made by make_pq_golden.py)."""

import os

import numpy as np
import pytest

from polarquant_b200 import CompressedVectors, Quantizer, load_pq, save_params, save_pq

G = os.path.join(os.path.dirname(__file__), "golden", "pq_files.npz")
CASES = [(b, d) for b in (1, 2, 3, 4, 8) for d in (13, 16)]


@pytest.fixture(scope="module")
def gold():
    return np.load(G)


@pytest.mark.parametrize("bits,d", CASES)
def test_save_pq_bytes_match_reference(tmp_path, gold, bits, d):
    key = f"b{bits}_d{d}"
    cv = CompressedVectors(gold[f"idx_{key}"], gold[f"norms_{key}"], d, bits)
    p = tmp_path / "x.pq"
    save_pq(p, cv)
    assert p.read_bytes() == gold[f"pq_{key}"].tobytes()


@pytest.mark.parametrize("bits,d", CASES)
def test_load_pq_reads_reference_files(tmp_path, gold, bits, d):
    key = f"b{bits}_d{d}"
    p = tmp_path / "x.pq"
    p.write_bytes(gold[f"pq_{key}"].tobytes())
    cv = load_pq(p)
    assert (cv.n, cv.d, cv.bits) == gold[f"idx_{key}"].shape + (bits,)
    np.testing.assert_array_equal(cv.indices, gold[f"idx_{key}"])
    assert cv.norms.dtype == np.float32
    np.testing.assert_array_equal(cv.norms.view(np.uint32), gold[f"norms_{key}"].view(np.uint32))


@pytest.mark.parametrize("bits", [1, 2, 3, 4, 8])
def test_save_params_bytes_match_reference(tmp_path, gold, bits):
    p = tmp_path / "x.params"
    save_params(p, Quantizer(d=16, bits=bits, seed=42))
    assert p.read_bytes() == gold[f"params_b{bits}_d16"].tobytes()


def test_load_pq_errors(tmp_path, gold):
    good = gold["pq_b4_d16"].tobytes()
    cases = [(good[:20], ".pq file too small"),
             (b"XQ" + good[2:], "bad .pq magic"),
             (good[:3] + b"\x02" + good[4:], "unsupported .pq version: 2"),
             (good[:16] + b"\x05" + good[17:], "bits=5 is not supported"),
             (good[:-1], "truncated .pq data")]
    for i, (data, msg) in enumerate(cases):
        p = tmp_path / f"bad{i}.pq"
        p.write_bytes(data)
        with pytest.raises(ValueError, match=msg):
            load_pq(p)


def test_save_params_shape_checks(tmp_path):
    q = Quantizer(d=16, bits=4, seed=42)
    q.R = q.R[:8]
    with pytest.raises(ValueError, match="R shape"):
        save_params(tmp_path / "x.params", q)


def test_empty_corpus_round_trip(tmp_path):
    cv = CompressedVectors(np.zeros((0, 12), np.uint8), np.zeros(0, np.float32), 12, 4)
    p = tmp_path / "e.pq"
    save_pq(p, cv)
    assert len(p.read_bytes()) == 32
    back = load_pq(p)
    assert back.n == 0 and back.indices.shape == (0, 12)

"""The `.npz` and Arrow IPC (Feather v2) corpus files (remex/core.py:64-116,
:326-439) against files written by the reference itself
(tests/golden/store_files.npz, made by make_store_golden.py).

The classes keep their corpora on the GPU, so these CPU tests drive the
host-side readers and writers they call (polarquant_b200.pq_format) with the
same arrays, plus the host-only CompressedVectors path for rows that are not a
whole number of bytes."""

import builtins
import os

import numpy as np
import pytest

from polarquant_b200 import CompressedVectors
from polarquant_b200.packing import pack, packed_nbytes, unpack
from polarquant_b200.pq_format import read_arrow, read_npz, write_arrow, write_npz

pa = pytest.importorskip("pyarrow")
feather = pytest.importorskip("pyarrow.feather")

G = os.path.join(os.path.dirname(__file__), "golden", "store_files.npz")
CASES = [(b, d) for b in (1, 2, 3, 4, 8) for d in (13, 16)]


@pytest.fixture(scope="module")
def gold():
    return np.load(G)


def _file(tmp_path, name, data):
    p = tmp_path / name
    p.write_bytes(data.tobytes())
    return str(p)


@pytest.mark.parametrize("bits,d", CASES)
def test_read_npz_reference_files(tmp_path, gold, bits, d):
    key = f"b{bits}_d{d}"
    idx, norms, rows = gold[f"idx_{key}"], gold[f"norms_{key}"], gold[f"rows_{key}"]
    n = idx.shape[0]
    cv = read_npz(_file(tmp_path, "cv.npz", gold[f"npz_cv_{key}"]))
    assert (cv["n"], cv["d"], cv["bits"]) == (n, d, bits)
    assert cv["packed_indices"].size == packed_nbytes(n, d, bits)
    np.testing.assert_array_equal(unpack(cv["packed_indices"], bits, n * d).reshape(n, d), idx)
    np.testing.assert_array_equal(cv["norms"].view(np.uint32), norms.view(np.uint32))
    pv = read_npz(_file(tmp_path, "pv.npz", gold[f"npz_pv_{key}"]))
    np.testing.assert_array_equal(pv["packed_indices"].reshape(rows.shape), rows)


@pytest.mark.parametrize("bits,d", CASES)
def test_write_npz_same_arrays_as_reference(tmp_path, gold, bits, d):
    key = f"b{bits}_d{d}"
    idx, norms, rows = gold[f"idx_{key}"], gold[f"norms_{key}"], gold[f"rows_{key}"]
    n = idx.shape[0]
    for name, flat in (("npz_cv", pack(idx.ravel(), bits)), ("npz_pv", rows.ravel())):
        ours = str(tmp_path / f"{name}.npz")
        write_npz(ours, flat, norms, d, bits, n)
        a = np.load(ours)
        b = np.load(_file(tmp_path, f"ref_{name}.npz", gold[f"{name}_{key}"]))
        assert sorted(a.files) == sorted(b.files)
        for k in b.files:
            assert a[k].dtype == b[k].dtype and a[k].shape == b[k].shape, k
            np.testing.assert_array_equal(a[k], b[k])


@pytest.mark.parametrize("bits,d", CASES)
def test_read_arrow_reference_files(tmp_path, gold, bits, d):
    key = f"b{bits}_d{d}"
    path = _file(tmp_path, "ref.arrow", gold[f"arrow_{key}"])
    for mm in (False, True):
        rows, norms, n, dd, bb = read_arrow(path, memory_map=mm)
        assert (n, dd, bb) == (gold[f"idx_{key}"].shape[0], d, bits)
        np.testing.assert_array_equal(rows, gold[f"rows_{key}"])
        assert norms.dtype == np.float32
        np.testing.assert_array_equal(norms.view(np.uint32),
                                      gold[f"norms_{key}"].view(np.uint32))


@pytest.mark.parametrize("bits,d", CASES)
def test_write_arrow_same_table_as_reference(tmp_path, gold, bits, d):
    key = f"b{bits}_d{d}"
    ours = str(tmp_path / "ours.arrow")
    write_arrow(ours, gold[f"rows_{key}"], gold[f"norms_{key}"], d, bits, seed=42,
                partition="shard_0")
    a = feather.read_table(ours)
    b = feather.read_table(_file(tmp_path, "ref.arrow", gold[f"arrow_{key}"]))
    assert a.schema.equals(b.schema, check_metadata=True)
    assert a.equals(b)
    meta = a.schema.metadata
    assert meta[b"seed"] == b"42" and meta[b"partition"] == b"shard_0"
    assert a.schema.field("packed_indices").type == pa.binary(packed_nbytes(1, d, bits))


def test_arrow_empty_round_trip(tmp_path):
    p = str(tmp_path / "e.arrow")
    write_arrow(p, np.zeros((0, 8), np.uint8), np.zeros(0, np.float32), 16, 4)
    rows, norms, n, d, bits = read_arrow(p)
    assert (n, d, bits) == (0, 16, 4) and rows.shape == (0, 8) and norms.size == 0


def test_arrow_row_size_checked(tmp_path):
    with pytest.raises(ValueError, match="packed rows size mismatch"):
        write_arrow(str(tmp_path / "x.arrow"), np.zeros((3, 7), np.uint8),
                    np.zeros(3, np.float32), 16, 4)


def test_arrow_needs_pyarrow(tmp_path, monkeypatch):
    real = builtins.__import__

    def fake(name, *a, **k):
        if name == "pyarrow" or name.startswith("pyarrow."):
            raise ImportError(f"No module named '{name}'")
        return real(name, *a, **k)

    monkeypatch.setattr(builtins, "__import__", fake)
    with pytest.raises(ImportError, match="pyarrow is required"):
        write_arrow(str(tmp_path / "x.arrow"), np.zeros((1, 8), np.uint8),
                    np.ones(1, np.float32), 16, 4)
    with pytest.raises(ImportError, match="pyarrow is required"):
        read_arrow(str(tmp_path / "x.arrow"))


@pytest.mark.parametrize("bits", [1, 2, 3, 4])
def test_host_compressed_vectors_npz(tmp_path, gold, bits):
    """Rows of 13 codes are not whole bytes at 1-4 bits: CompressedVectors
    saves and loads them on the host, including the reference's own files."""
    key = f"b{bits}_d13"
    idx, norms = gold[f"idx_{key}"], gold[f"norms_{key}"]
    ref = CompressedVectors.load(_file(tmp_path, "ref.npz", gold[f"npz_cv_{key}"]))
    np.testing.assert_array_equal(ref.indices, idx)
    np.testing.assert_array_equal(ref.norms, norms)
    p = str(tmp_path / "ours.npz")
    CompressedVectors(idx, norms, 13, bits).save(p)
    back = CompressedVectors.load(p)
    assert (back.n, back.d, back.bits) == (idx.shape[0], 13, bits)
    np.testing.assert_array_equal(back.indices, idx)

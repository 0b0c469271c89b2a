"""Host-side checks that need no GPU: API validation, the C-ABI library's
exports and argument checks, and host packing edge cases."""

import ctypes
import os
import re

import numpy as np
import pytest

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))


def header_functions():
    names = []
    for h in os.listdir(os.path.join(ROOT, "include")):
        if h.endswith(".h"):
            txt = open(os.path.join(ROOT, "include", h)).read()
            txt = re.sub(r"/\*.*?\*/", "", txt, flags=re.S)
            names += re.findall(r"\b(pq_[a-z0-9_]+)\s*\(", txt)
    return sorted(set(names))


@pytest.fixture(scope="module")
def lib():
    from polarquant_b200 import build, _lib
    build.build()
    return _lib.load()


def test_library_exports_every_header_symbol(lib):
    from polarquant_b200 import _lib
    names = header_functions()
    assert len(names) >= 10
    for n in names:
        assert hasattr(lib, n), f"{n} declared in include/ but not exported"
        assert n in _lib.SIGNATURES, f"{n} has no ctypes signature"
    assert set(_lib.SIGNATURES) == set(names)


def test_host_only_entry_points(lib):
    from polarquant_b200 import _lib, packing
    assert _lib.query("pq_version") >= 10000
    for d in (1, 7, 40, 384, 1536):
        for b in (1, 2, 3, 4, 8):
            assert _lib.query("pq_row_bytes", d, b) == packing.packed_nbytes(1, d, b)
    assert _lib.query("pq_row_bytes", 8, 5) == -1


def test_abi_rejects_bad_arguments_before_touching_the_device(lib):
    from polarquant_b200 import _lib
    P = ctypes.c_void_p
    rc = lib.pq_adc_scan(P(16), 16, P(16), 10, 32, 5, 1, P(16), 1, P(16), 1, 0, P(16), P(16),
                         P(16), 1 << 20, None)
    assert rc == -1 and b"bits" in lib.pq_last_error()
    rc = lib.pq_adc_scan(P(16), 8, P(16), 10, 32, 4, 1, P(16), 1, P(16), 1, 0, P(16), P(16),
                         P(16), 1 << 20, None)
    assert rc == -1 and b"ldb" in lib.pq_last_error()
    rc = lib.pq_adc_scan(P(16), 16, P(16), 10, 32, 4, 5, P(16), 1, P(16), 1, 0, P(16), P(16),
                         P(16), 1 << 20, None)
    assert rc == -1 and b"precision" in lib.pq_last_error()
    rc = lib.pq_twostage(P(16), 16, P(16), 10, 32, 4, 2, P(16), 1, P(16), P(16), 20, 5, 0,
                         P(16), P(16), P(16), 1 << 20, None)
    assert rc == -1 and b"candidates" in lib.pq_last_error()
    with pytest.raises(_lib.PQError):
        _lib.call("pq_topk_merge", P(16), P(16), 2, 1, 4, 9, P(16), P(16), None)


def test_quantizer_bit_validation():
    from polarquant_b200 import Quantizer
    for b in (0, 9):
        with pytest.raises(ValueError):
            Quantizer(16, bits=b)
    for b in (5, 6, 7):
        with pytest.raises(ValueError, match="not supported"):
            Quantizer(16, bits=b)


def test_packing_errors_and_padding():
    from polarquant_b200 import pack, packed_nbytes, unpack
    for b in (5, 6, 7):
        with pytest.raises(ValueError, match="not supported"):
            pack(np.zeros(4, np.uint8), b)
        with pytest.raises(ValueError, match="not supported"):
            unpack(np.zeros(4, np.uint8), b, 4)
        with pytest.raises(ValueError, match="not supported"):
            packed_nbytes(1, 4, b)
    rng = np.random.default_rng(99)
    from oracle import remex_oracle as O
    for b in (1, 2, 3, 4, 8):
        for n in (0, 1, 3, 9, 17, 50 * 384):
            v = rng.integers(0, 2 ** b, size=n, dtype=np.uint8)
            p = pack(v, b)
            np.testing.assert_array_equal(p, O.pack(v, b))
            np.testing.assert_array_equal(unpack(p, b, n), v)
            assert len(p) == packed_nbytes(n, 1, b)


def test_deprecated_alias():
    import polarquant_b200
    from polarquant_b200 import Quantizer
    with pytest.warns(DeprecationWarning, match="PolarQuantizer has been renamed"):
        assert polarquant_b200.PolarQuantizer is Quantizer


def test_product_does_not_import_the_oracle():
    pkg = os.path.join(ROOT, "polarquant_b200")
    for dirpath, _, files in os.walk(pkg):
        for f in files:
            if f.endswith(".py"):
                src = open(os.path.join(dirpath, f)).read()
                mods = re.findall(r"^\s*(?:from|import)\s+(\S+)", src, re.M)
                assert not any(m.split(".")[0] == "oracle" for m in mods), f

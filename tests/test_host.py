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
    # The bounded-wait self-test checks its limit before launching anything.
    assert lib.pq_selftest_wait_timeout(10, None) == -1
    assert b"limit_cycles" in lib.pq_last_error()
    assert lib.pq_selftest_wait_timeout(5_000_000_000, None) == -1


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


# One rejected call per check, for every entry point that computes: the
# status is PQ_ERR_INVALID (-1) or PQ_ERR_WORKSPACE (-3) and pq_last_error()
# names the argument.  The fake pointers (16-byte aligned, never dereferenced)
# show that each check runs before any device work.
_A = 16  # a fake aligned device address


def _abi_bad_calls():
    P = ctypes.c_void_p
    a = P(_A)
    sc = (a, a, a, 1 << 20, None)  # out_scores, out_ids, ws, ws_bytes, stream (scan shapes)
    return [
        ("pq_prepare_rotation", (a, 0, a, 1 << 20, None), -1, "d must be positive"),
        ("pq_prepare_rotation", (a, 64, a, 16, None), -1, "planes buffer too small"),
        ("pq_prepare_rotation", (a, 64, P(_A + 4), 1 << 24, None), -1, "16-byte aligned"),
        ("pq_encode", (a, 10, 32, a, a, a, 5, a, 16, a, a, 1 << 20, None), -1, "bits must be"),
        ("pq_encode", (a, 10, 32, a, a, a, 4, a, 24, a, a, 1 << 20, None), -1, "multiple of 16"),
        ("pq_encode", (a, 10, 0, a, a, a, 4, a, 16, a, a, 1 << 20, None), -1, "d must be positive"),
        ("pq_rotate_tc", (a, 10, 0, a, a, a, 1 << 20, None), -1, "d must be positive"),
        ("pq_rotate_tc", (a, -1, 8, a, a, a, 1 << 20, None), -1, "n must be >= 0"),
        ("pq_rotate", (a, 4, 0, a, a, None), -1, "d must be positive"),
        ("pq_rotate", (a, -1, 8, a, a, None), -1, "nq must be >= 0"),
        ("pq_decode", (a, 16, a, 10, 32, 4, 5, a, a, a, a, 1 << 20, None), -1, "precision must be 1-4"),
        ("pq_decode", (a, 8, a, 10, 32, 4, 4, a, a, a, a, 1 << 20, None), -1, "ldb too small"),
        ("pq_adc_scan", (a, 16, a, 10, 32, 4, 4, a, 1, a, 11, 0) + sc, -1, "exceeds n"),
        ("pq_adc_scan", (a, 16, a, 10, 32, 4, 4, a, 1, a, 0, 0) + sc, -1, "k must be >= 1"),
        ("pq_adc_scan", (P(_A + 8), 16, a, 10, 32, 4, 4, a, 1, a, 1, 0) + sc, -1,
         "16-byte aligned"),
        ("pq_adc_batch", (a, 16, a, 1000, 32, 4, 4, a, 64, a, 257, 0) + sc, -1, "k must be in"),
        ("pq_adc_batch", (a, 16, a, 1000, 32, 3, 4, a, 64, a, 10, 0) + sc, -1, "precision must be 1-3"),
        ("pq_adc_batch", (a, 16, a, -5, 32, 4, 4, a, 64, a, 10, 0) + sc, -1, "n must be >= 0"),
        ("pq_adc_scan_noalloc", (a, 16, a, 10, 32, 4, 4, a, 1, a, 2049, 0, a, a, None), -1,
         "allocation-free"),
        ("pq_adc_scan_noalloc", (a, 16, a, 1 << 24, 32, 4, 4, a, 4096, a, 2048, 0, a, a, None),
         -3, "scratch"),
        ("pq_twostage", (a, 16, a, 100, 32, 4, 2, a, 1, a, a, 200, 5, 0) + sc, -1, "candidates"),
        ("pq_twostage", (a, 16, a, 100, 32, 4, 2, a, 1, a, a, 20, 21, 0) + sc, -1, "k must be in"),
        ("pq_twostage", (a, 16, a, 100, 32, 4, 0, a, 1, a, a, 20, 5, 0) + sc, -1, "precision"),
        ("pq_rerank", (a, 16, a, 100, 32, 4, a, 1, a, a, 0, 5, 0, a, a, None), -1, "C must be in"),
        ("pq_rerank", (a, 16, a, 100, 32, 4, a, 1, a, a, 10, 2049, 0, a, a, None), -1,
         "k must be in"),
        ("pq_ivf_cell_ids", (a, 16, 10, 32, 4, 17, 0, a, a, None), -1, "n_bits must be 1-16"),
        ("pq_ivf_cell_ids", (a, 16, 10, 32, 4, 4, 2, a, a, None), -1, "mode must be"),
        ("pq_ivf_cell_ids", (a, 16, 10, 8, 4, 9, 1, None, a, None), -1, "exceeds d=8"),
        ("pq_ivf_cell_ids", (a, 16, 10, 32, 5, 4, 0, a, a, None), -1, "bits must be"),
        ("pq_ivf_probe", (a, 1, 32, 4, 0, a, 17, a, a, None), -1, "nprobe must be in"),
        ("pq_ivf_probe", (a, 1, 32, 0, 0, a, 1, a, a, None), -1, "n_bits must be 1-16"),
        ("pq_ivf_search", (a, 16, a, 100, 32, 4, 2, a, 1, a, a, 4, 0, a, a, a, None, None, 4, 65,
                           20, 5, 1, a, a, a, 1 << 20, None), -1, "splits must be in"),
        ("pq_ivf_search", (a, 16, a, 100, 32, 4, 2, a, 1, a, a, 4, 0, a, a, a, a, None, 4, 1,
                           20, 5, 1, a, a, a, 1 << 20, None), -1, "both be given"),
        ("pq_ivf_search", (a, 16, a, 100, 32, 4, 2, a, 1, a, None, 4, 0, a, a, a, None, None, 4,
                           1, 20, 5, 1, a, a, a, 1 << 20, None), -1, "full-precision"),
        ("pq_ivf_search", (a, 16, a, 100, 32, 4, 2, a, 1, a, a, 4, 0, a, a, a, None, None, 4, 1,
                           20, 5, 1, a, a, a, 64, None), -3, "workspace bytes"),
        ("pq_unpack_rows", (a, 16, 10, 32, 4, 4, a, None), -1, "shift out of range"),
        ("pq_unpack_at", (a, 16, a, 3, 32, 4, -1, a, None), -1, "shift out of range"),
        ("pq_repack", (a, 16, 10, 32, 4, 8, a, 16, None), -1, "target_bits"),
        ("pq_repack", (a, 16, 10, 32, 4, 2, a, 8, None), -1, "bad ldb_out"),
        ("pq_pack_codes", (a, 10, 32, 4, a, 8, None), -1, "bad ldb"),
        ("pq_topk_merge", (a, a, 0, 1, 4, 2, a, a, None), -1, "bad merge shape"),
    ]


@pytest.mark.parametrize("case", range(len(_abi_bad_calls())))
def test_abi_argument_checks(lib, case):
    name, args, code, msg = _abi_bad_calls()[case]
    rc = getattr(lib, name)(*args)
    assert rc == code, (name, rc, lib.pq_last_error())
    assert msg.encode() in lib.pq_last_error(), (name, lib.pq_last_error())


def test_abi_empty_inputs_do_no_device_work(lib):
    """Zero queries or zero rows succeed at once (no launch, no device query)."""
    P = ctypes.c_void_p
    a = P(_A)
    before = lib.pq_launch_count()
    calls = [
        ("pq_adc_scan", (a, 16, a, 10, 32, 4, 4, None, 0, None, 5, 0, None, None, None, 0, None)),
        ("pq_adc_batch", (a, 16, a, 10, 32, 4, 4, None, 0, None, 5, 0, None, None, None, 0, None)),
        ("pq_twostage", (a, 16, a, 100, 32, 4, 2, None, 0, None, None, 20, 5, 0, None, None,
                         None, 0, None)),
        ("pq_rerank", (a, 16, a, 100, 32, 4, None, 0, None, None, 10, 5, 0, None, None, None)),
        ("pq_encode", (None, 0, 32, None, None, None, 4, None, 16, None, None, 0, None)),
        ("pq_rotate", (None, 0, 32, None, None, None)),
        ("pq_rotate_tc", (None, 0, 32, None, None, None, 0, None)),
        ("pq_decode", (None, 16, None, 0, 32, 4, 4, None, None, None, None, 0, None)),
        ("pq_ivf_cell_ids", (None, 16, 0, 32, 4, 4, 0, None, None, None)),
        ("pq_ivf_probe", (None, 0, 32, 4, 0, None, 3, None, None, None)),
        ("pq_unpack_rows", (None, 16, 0, 32, 4, 0, None, None)),
        ("pq_unpack_at", (None, 16, None, 0, 32, 4, 0, None, None)),
        ("pq_repack", (None, 16, 0, 32, 4, 2, None, 16, None)),
        ("pq_pack_codes", (None, 0, 32, 4, None, 16, None)),
        ("pq_topk_merge", (None, None, 2, 0, 4, 3, None, None, None)),
    ]
    for name, args in calls:
        rc = getattr(lib, name)(*args)
        assert rc == 0, (name, rc, lib.pq_last_error())
    assert lib.pq_launch_count() == before


def test_api_errors_match_reference_messages():
    """The errors the reference raises before any arithmetic (remex/core.py:
    265-268, :466-472, :563-568, :748-753, :888-891), raised here before any
    device work, with the same types and messages."""
    from polarquant_b200 import PackedVectors, Quantizer
    pq = Quantizer(16, bits=4, seed=42)
    pv = PackedVectors.__new__(PackedVectors)  # no device rows: the checks come first
    pv.bits = 4
    q = np.zeros(16, np.float32)
    for fn, name in ((pq.search, "search"), (pq.search_batch, "search_batch")):
        msg = (f"PackedVectors does not support cached {name}(). Use search_adc() or "
               f"search_twostage(), or convert with packed.to_compressed() first.")
        with pytest.raises(TypeError, match=re.escape(msg)):
            fn(pv, q)
    with pytest.raises(TypeError, match="expected CompressedVectors or PackedVectors"):
        pq.search_adc(object(), q)
    for p in (0, 5):
        with pytest.raises(ValueError, match=re.escape(f"precision must be 1-4, got {p}")):
            pq._resolve_centroids(None, p)
    with pytest.raises(ValueError, match=re.escape("target_bits must be 1-4, got 5")):
        pv.at_precision(5)
    with pytest.raises(ValueError, match=re.escape("bits must be 1-4 or 8, got 9")):
        Quantizer(16, bits=9)
    with pytest.raises(ValueError, match=re.escape("bits=6 is not supported. Use 1-4 or 8 bits.")):
        Quantizer(16, bits=6)


def test_batch_routing_cost_model():
    """Large corpora route small batches by the measured cost of each path:
    the streaming scan up to the crossover, the tensor cores past it (d=1536:
    about 3 queries at 8 bits, 5 at 4, 10 at 2, 16 at 1 bit); without the
    code width the fixed 8-query rule applies, and small corpora keep the
    64-query rule."""
    from polarquant_b200.core import use_tensor_cores as route

    def first_batched(n, bits, d, rb):
        return next(nq for nq in range(1, 300) if route(n, nq, 100, rb, bits, d))

    assert first_batched(40_000_000, 8, 1536, 1536) == 3
    assert first_batched(100_000_000, 4, 1536, 768) == 5
    assert first_batched(100_000_000, 2, 1536, 384) == 10
    assert first_batched(100_000_000, 1, 1536, 192) == 16
    assert first_batched(100_000_000, 4, 1536, None) == 8
    assert first_batched(500_000, 4, 1536, 768) == 64
    assert not route(100_000_000, 200, 300, 768, 4, 1536)  # k past the batched kernels

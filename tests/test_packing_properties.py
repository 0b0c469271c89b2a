"""Property tests of the host packers (polarquant_b200.packing, the layout of
remex/packing.py:18-150 and remex/core.py:161-223) against the oracle over
random widths and shapes, including rows that are not a whole number of
bytes."""

import numpy as np
from hypothesis import given, settings
from hypothesis import strategies as st

from oracle import remex_oracle as O
from polarquant_b200.packing import pack, pack_rows, packed_nbytes, unpack, unpack_rows

BITS = st.sampled_from([1, 2, 3, 4, 8])


@settings(max_examples=150, deadline=None)
@given(bits=BITS, n=st.integers(0, 300), seed=st.integers(0, 2**32 - 1))
def test_stream_pack_matches_oracle(bits, n, seed):
    v = np.random.default_rng(seed).integers(0, 1 << bits, n).astype(np.uint8)
    p = pack(v, bits)
    np.testing.assert_array_equal(p, O.pack(v, bits))
    assert p.size == packed_nbytes(n, 1, bits) == O.packed_nbytes(n, 1, bits)
    np.testing.assert_array_equal(unpack(p, bits, n), v)


@settings(max_examples=150, deadline=None)
@given(bits=BITS, n=st.integers(0, 40), d=st.integers(1, 70), seed=st.integers(0, 2**32 - 1))
def test_row_pack_matches_oracle(bits, n, d, seed):
    idx = np.random.default_rng(seed).integers(0, 1 << bits, (n, d)).astype(np.uint8)
    rows = pack_rows(idx, bits)
    assert rows.shape == (n, packed_nbytes(1, d, bits))
    np.testing.assert_array_equal(rows, O.pack_rows(idx, bits))
    np.testing.assert_array_equal(unpack_rows(rows, bits, d), idx)
    if (d * bits) % 8 == 0:  # whole-byte rows: the row layout is the stream layout
        np.testing.assert_array_equal(rows.ravel(), pack(idx.ravel(), bits))

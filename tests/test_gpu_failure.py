"""Failure detection on the device without a fault: a kernel whose bounded
wait runs out records an error code and returns, the host reads (and clears)
it through pq_device_status, and the context stays usable.

The wait is the library's own mbar_wait_limit, the routine every mbarrier
wait of the tensor-core kernels goes through, given a short limit
(pq_selftest_wait_timeout): nothing ever arrives at its barrier, so it must
give up after ~limit SM cycles.  No trap, no illegal access, no hang."""

import numpy as np
import pytest

from oracle import remex_oracle as O

pytestmark = pytest.mark.gpu

PQ_DEVICE_ERR_WAIT_SELFTEST = 105


def test_bounded_wait_runs_out_and_is_reported(gpu):
    import time
    from polarquant_b200 import CompressedVectors, Quantizer, _lib
    assert _lib.device_status() == 0
    t = time.perf_counter()
    _lib.call("pq_selftest_wait_timeout", 2_000_000, None)  # ~1 ms of SM clock
    code = _lib.device_status()
    assert code == PQ_DEVICE_ERR_WAIT_SELFTEST
    assert time.perf_counter() - t < 30.0
    assert _lib.device_status() == 0, "pq_device_status clears the word it reported"
    # Two in a row: the first code stays until read.
    _lib.call("pq_selftest_wait_timeout", 1_000_000, None)
    _lib.call("pq_selftest_wait_timeout", 1_000_000, None)
    assert _lib.device_status() == PQ_DEVICE_ERR_WAIT_SELFTEST
    assert _lib.device_status() == 0
    # The context is still usable: a search after the timeouts matches the oracle.
    d, n = 64, 3000
    rng = np.random.default_rng(4)
    X = rng.standard_normal((n, d)).astype(np.float32)
    q = rng.standard_normal(d).astype(np.float32)
    pq = Quantizer(d, bits=4, seed=42)
    idx, norms = O.encode(X, pq.R, pq.boundaries)
    gi, gs = pq.search_adc(CompressedVectors(idx, norms, d, 4), q, k=10)
    ri, rs = O.search_adc(pq.R, pq.centroids, pq._nested, 4, idx, norms, q, k=10)
    assert O.topk_equal_up_to_ties(gi, gs, ri, rs, rtol=1e-4)
    assert _lib.device_status() == 0

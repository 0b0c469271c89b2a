"""Row-sharded search on 2 GPUs over NCCL (skipped with fewer GPUs): every
rank's results must equal the single-corpus oracle results, for the streaming
scan (few queries), the tensor-core batch path (>= 64 queries) and the exact
two-exchange two-stage merge."""

import os
import socket
import sys

import numpy as np
import pytest

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))

pytestmark = pytest.mark.gpu


def _gpus():
    try:
        import torch
        return torch.cuda.device_count()
    except Exception:
        return 0


def _free_port():
    s = socket.socket()
    s.bind(("127.0.0.1", 0))
    p = s.getsockname()[1]
    s.close()
    return p


def _data():
    from oracle import remex_oracle as O
    from polarquant_b200.params import haar_rotation, lloyd_max_codebook
    d, n, bits = 256, 20011, 8
    rng = np.random.default_rng(7)
    X = rng.standard_normal((n, d)).astype(np.float32)
    Q = rng.standard_normal((80, d)).astype(np.float32)
    R = haar_rotation(d, 42)
    bnd, _ = lloyd_max_codebook(d, bits)
    idx, norms = O.encode(X, R, bnd)
    return d, n, bits, Q, idx, norms


def _rank(rank, world, port, outdir):
    sys.path.insert(0, ROOT)
    import datetime
    import torch
    import torch.distributed as dist
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
    torch.cuda.set_device(rank)
    dist.init_process_group("nccl", rank=rank, world_size=world,
                            timeout=datetime.timedelta(seconds=120),
                            device_id=torch.device("cuda", rank))
    from polarquant_b200 import CompressedVectors, Quantizer
    from polarquant_b200.distributed import ShardedSearch, shard_bounds, to_numpy
    d, n, bits, Q, idx, norms = _data()
    r0, r1 = shard_bounds(n, world, rank)
    pq = Quantizer(d, bits=bits, seed=42)
    ss = ShardedSearch(pq, CompressedVectors(idx[r0:r1], norms[r0:r1], d, bits), r0, n)
    out = {}
    out["few_i"], out["few_s"] = to_numpy(*ss.search_adc_many(Q[:5], k=25, precision=5))
    out["bat_i"], out["bat_s"] = to_numpy(*ss.search_adc_many(Q, k=100))
    out["ts_i"], out["ts_s"] = to_numpy(*ss.search_twostage_many(Q, k=10, candidates=200,
                                                                  coarse_precision=4))
    out["ts5_i"], out["ts5_s"] = to_numpy(*ss.search_twostage_many(Q[:5], k=10, candidates=300))
    np.savez(os.path.join(outdir, f"rank{rank}.npz"), **out)
    dist.barrier()
    dist.destroy_process_group()


@pytest.mark.skipif(_gpus() < 2, reason="needs 2 GPUs")
def test_two_gpu_sharded_search_matches_oracle(gpu, tmp_path):
    import torch.multiprocessing as mp
    from oracle import remex_oracle as O
    from polarquant_b200.params import haar_rotation, lloyd_max_codebook, nested_codebooks
    mp.start_processes(_rank, args=(2, _free_port(), str(tmp_path)), nprocs=2, join=True,
                       start_method="spawn")
    d, n, bits, Q, idx, norms = _data()
    R = haar_rotation(d, 42)
    _, cent = lloyd_max_codebook(d, bits)
    nest = nested_codebooks(d, bits)
    r = [np.load(os.path.join(tmp_path, f"rank{k}.npz")) for k in range(2)]
    for key in r[0].files:
        np.testing.assert_array_equal(r[0][key], r[1][key])
    z = r[0]
    for qi in range(5):
        ri, rs = O.search_adc(R, cent, nest, bits, idx, norms, Q[qi], k=25, precision=5)
        assert O.topk_equal_up_to_ties(z["few_i"][qi], z["few_s"][qi], ri, rs, rtol=1e-4)
        ri, rs = O.search_twostage(R, cent, nest, bits, idx, norms, Q[qi], k=10, candidates=300)
        assert O.topk_equal_up_to_ties(z["ts5_i"][qi], z["ts5_s"][qi], ri, rs, rtol=1e-4)
    RI, RS = O.search_batch(R, cent, nest, bits, idx, norms, Q, k=100)
    for qi in range(len(Q)):
        assert O.topk_equal_up_to_ties(z["bat_i"][qi], z["bat_s"][qi], RI[qi], RS[qi], rtol=1e-4)
        ri, rs = O.search_twostage(R, cent, nest, bits, idx, norms, Q[qi], k=10, candidates=200,
                                   coarse_precision=4)
        assert O.topk_equal_up_to_ties(z["ts_i"][qi], z["ts_s"][qi], ri, rs, rtol=1e-4)

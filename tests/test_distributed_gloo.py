"""Row-sharded search protocol over torch.distributed ranks, on CPU (gloo).

polarquant_b200.distributed.ShardedSearch does the sharding, all-gathers and
the exact two-exchange two-stage merge; here its per-rank compute steps are
replaced by the NumPy oracle so the protocol is checked alone: 2, 3 or 4 ranks
(uneven shards, shards smaller than k, a rank without rows) must return
exactly what one process holding the whole corpus returns.  A second
test makes one rank fail before the collective and checks that the survivor
gets an error from the process-group timeout instead of hanging.
"""

import os
import socket
import sys

import numpy as np
import pytest
import torch
import torch.distributed as dist
import torch.multiprocessing as mp

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))


def _free_port():
    s = socket.socket()
    s.bind(("127.0.0.1", 0))
    p = s.getsockname()[1]
    s.close()
    return p


def _data(n=1001):
    from oracle import remex_oracle as O
    from polarquant_b200.params import haar_rotation, lloyd_max_codebook, nested_codebooks
    d, bits = 64, 4
    rng = np.random.default_rng(0)
    X = rng.standard_normal((n, d)).astype(np.float32)
    Q = rng.standard_normal((5, d)).astype(np.float32)
    R = haar_rotation(d, 42)
    bnd, cent = lloyd_max_codebook(d, bits)
    nest = nested_codebooks(d, bits)
    idx, norms = O.encode(X, R, bnd)
    return d, n, bits, Q, R, cent, nest, idx, norms


def _order(scores, ids, k):
    o = np.lexsort((ids, -scores))[:k]
    return scores[o], ids[o]


def _rank_main(rank, world, port, outdir, n, ka, ck, kt):
    sys.path.insert(0, ROOT)
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
    import datetime
    dist.init_process_group("gloo", rank=rank, world_size=world,
                            timeout=datetime.timedelta(seconds=60))
    from oracle import remex_oracle as O
    from polarquant_b200.core import Quantizer
    from polarquant_b200.distributed import ShardedSearch, shard_bounds
    d, n, bits, Q, R, cent, nest, idx, norms = _data(n)
    r0, r1 = shard_bounds(n, world, rank)

    class Shard:
        def __init__(self, m):
            self.n = m

    class CpuSharded(ShardedSearch):
        def rotate(self, Qin):
            return torch.from_numpy((np.asarray(Qin, np.float32) @ R.T).astype(np.float32))

        def local_topk(self, qrot, k, p):
            c = cent if p == bits else nest[p]
            S, I = [], []
            for q in qrot.numpy():
                sc = O.adc_scores(np.outer(q, c).astype(np.float32),
                                  O.resolve_indices(idx[r0:r1], bits, p), norms[r0:r1])
                s, i = _order(sc, np.arange(r0, r1), k)
                S.append(s)
                I.append(i)
            return torch.from_numpy(np.array(S, np.float32)), torch.from_numpy(np.array(I))

        def local_rerank(self, qrot, cand, k):
            S, I = [], []
            for q, cs in zip(qrot.numpy(), cand.numpy()):
                own = cs[(cs >= r0) & (cs < r1)]
                sc = (cent[idx[own]] @ q) * norms[own]
                s, i = _order(sc, own, k)
                pad = k - len(s)
                S.append(np.concatenate([s, np.full(pad, -np.inf, np.float32)]))
                I.append(np.concatenate([i, np.full(pad, -1, np.int64)]))
            return torch.from_numpy(np.array(S, np.float32)), torch.from_numpy(np.array(I))

        def merge(self, s_parts, i_parts, k):
            S, I = [], []
            for q in range(s_parts.shape[1]):
                s = s_parts[:, q].reshape(-1).numpy()
                i = i_parts[:, q].reshape(-1).numpy()
                keep = i >= 0
                s, i = _order(s[keep], i[keep], k)
                S.append(s)
                I.append(i)
            return torch.from_numpy(np.array(S, np.float32)), torch.from_numpy(np.array(I))

    pq = Quantizer.__new__(Quantizer)
    pq.d, pq.bits, pq.seed = d, bits, 42
    pq.R, pq.centroids, pq._nested = R, cent, nest
    ss = CpuSharded(pq, Shard(r1 - r0), r0, n)
    a_s, a_i = ss.search_adc_many(Q, k=ka, precision=3)
    t_s, t_i = ss.search_twostage_many(Q, k=kt, candidates=ck, coarse_precision=2)
    np.savez(os.path.join(outdir, f"rank{rank}.npz"), a_s=a_s.numpy(), a_i=a_i.numpy(),
             t_s=t_s.numpy(), t_i=t_i.numpy())
    dist.barrier()
    dist.destroy_process_group()


# (ranks, rows, k, candidates, two-stage k): uneven shards; shards with fewer
# rows than k (padded with sentinel slots before the exchange); a rank that
# holds no rows at all.
@pytest.mark.parametrize("world,n,ka,ck,kt", [(2, 1001, 17, 50, 7), (3, 40, 17, 30, 7),
                                              (4, 3, 2, 2, 1)])
def test_sharded_protocol_equals_single_process(tmp_path, world, n, ka, ck, kt):
    from oracle import remex_oracle as O
    port = _free_port()
    mp.start_processes(_rank_main, args=(world, port, str(tmp_path), n, ka, ck, kt),
                       nprocs=world, join=True, start_method="spawn")
    d, n, bits, Q, R, cent, nest, idx, norms = _data(n)
    r = [np.load(os.path.join(tmp_path, f"rank{k}.npz")) for k in range(world)]
    for name in ("a_s", "a_i", "t_s", "t_i"):
        for k in range(1, world):
            np.testing.assert_array_equal(r[0][name], r[k][name])  # every rank agrees
    assert r[0]["a_i"].shape == (len(Q), min(ka, n))
    assert (r[0]["a_i"] >= 0).all() and (r[0]["t_i"] >= 0).all()
    for qi, q in enumerate(Q):
        ri, rs = O.search_adc(R, cent, nest, bits, idx, norms, q, k=ka, precision=3)
        assert O.topk_equal_up_to_ties(r[0]["a_i"][qi], r[0]["a_s"][qi], ri, rs, rtol=1e-6)
        ri, rs = O.search_twostage(R, cent, nest, bits, idx, norms, q, k=kt, candidates=ck,
                                   coarse_precision=2)
        assert O.topk_equal_up_to_ties(r[0]["t_i"][qi], r[0]["t_s"][qi], ri, rs, rtol=1e-6)


def _failing_rank(rank, world, port, outdir):
    sys.path.insert(0, ROOT)
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
    import datetime
    dist.init_process_group("gloo", rank=rank, world_size=world,
                            timeout=datetime.timedelta(seconds=3))
    if rank == 1:
        os._exit(0)  # leaves between steps, before the collective
    try:
        t = torch.zeros(4)
        out = torch.empty(8)
        dist.all_gather_into_tensor(out, t)
        status = "completed"
    except Exception as e:  # gloo reports the dead peer or the timeout
        status = "error: " + type(e).__name__
    with open(os.path.join(outdir, "rank0.txt"), "w") as f:
        f.write(status)
    os._exit(0)


def test_dead_rank_surfaces_as_error(tmp_path):
    port = _free_port()
    ctx = mp.start_processes(_failing_rank, args=(2, port, str(tmp_path)), nprocs=2,
                             join=False, start_method="spawn")
    for p in ctx.processes:
        p.join(timeout=60)
    for p in ctx.processes:
        if p.is_alive():
            p.kill()
    with open(os.path.join(tmp_path, "rank0.txt")) as f:
        assert f.read().startswith("error")

"""Parity counts of the GPU path against the CPU oracle on every benchmark
configuration's own data distribution (run on a B200; prints one JSON line
per configuration and writes them all to the file given by --out).

    python tests/parity_report.py [--out parity.json] [--only c1,c2,c3,c4,c5]

What is counted (the parity rules of the encode and search paths):

* encode (c3: d=1024, 4M rows N(0,I) x log-uniform norms, bits 2/3/4/8; also
  the c1 corpus): codes that differ from the oracle's (remex/core.py:484-511),
  how many of those lie within 1e-6 of a Lloyd-Max boundary (all must), the
  largest level jump, and the norms' largest relative difference.
* search (c1, c2, c4, c5): queries whose top-k differs from the oracle's
  after score ties (scores within 1e-4 of the list's largest |score|), queries
  whose id lists differ at all, and the largest score difference relative to
  the list's largest |score|.  c1: all 200 queries, search_adc
  (remex/core.py:582-636).  c2: 1M rows, 256 of the 1,000 queries,
  search_twostage(cp=4, C=200, k=10) (core.py:638-719).  c4: the int8
  batched ADC on 2^21 rows of the d=1536 clustered corpus with 1,024 queries
  (k=100), 128 sampled queries against the oracle's search_batch
  (core.py:721-778) and all of them against the exact streaming scan.  c5:
  the full 10M-row IVF corpus (n_bits=12, nprobe=32, cp=2, C=500, k=10), cell
  ids of every row against the oracle's (remex/ivf.py:162-224) and 128 sampled
  queries against its search_twostage (remex/ivf.py:376-436).

Inputs come from the benchmark's seeded generators (bench.py), so the counts
describe the benchmarked data.  This is test infrastructure: it imports the
oracle as the checker.
"""

from __future__ import annotations

import argparse
import json
import os
import sys
import time

import numpy as np

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
sys.path.insert(0, ROOT)

from oracle import remex_oracle as O  # noqa: E402

RTOL = 1e-4


def search_counts(GI, GS, RI, RS):
    bad = diff = 0
    rel = 0.0
    for q in range(len(RI)):
        keep = GI[q] >= 0
        gi, gs = GI[q][keep], GS[q][keep]
        bad += not O.topk_equal_up_to_ties(gi, gs, RI[q], RS[q], rtol=RTOL)
        diff += (len(gi) != len(RI[q])) or bool(np.any(gi != RI[q]))
        if len(gi) == len(RI[q]) and len(gi):
            den = max(1e-30, float(np.abs(RS[q]).max()))
            rel = max(rel, float(np.abs(gs.astype(np.float64) - RS[q]).max()) / den)
    return {"queries": int(len(RI)), "topk_mismatch_after_ties": int(bad),
            "id_lists_differing": int(diff), "max_score_rel_diff": rel, "rtol": RTOL}


def encode_counts(got_idx, got_norms, X, R, bnd, ref_idx, ref_norms):
    d = got_idx != ref_idx
    nflip = int(d.sum())
    out = {"coords": int(got_idx.size), "flips": nflip, "flip_frac": nflip / got_idx.size}
    if nflip:
        rot = O.rotated(X, R)
        dist = O.boundary_distance(rot[d], bnd)
        out["flips_within_1e-6_of_boundary"] = int((dist <= 1e-6).sum())
        out["max_flip_boundary_distance"] = float(dist.max())
        out["max_level_jump"] = int(np.abs(got_idx[d].astype(int) - ref_idx[d].astype(int)).max())
    den = np.maximum(np.abs(ref_norms), 1e-30)
    out["norms_max_rel_diff"] = float((np.abs(got_norms - ref_norms) / den).max())
    out["norms_bit_identical"] = bool(np.array_equal(got_norms, ref_norms))
    return out


def corpus(torch, dev, cfg, n, nq, seed=1):
    import bench
    from polarquant_b200 import Quantizer
    from polarquant_b200.core import CompressedVectors
    from polarquant_b200.encode import alloc_corpus, encode_into
    cfg = dict(cfg, n=n, nq=nq)
    pq = Quantizer(cfg["d"], bits=cfg["bits"], seed=42)
    centres = bench.make_centres(torch, dev, cfg, seed=7)
    rows = alloc_corpus(pq, n, dev)
    for a in range(0, n, 1 << 20):
        b = min(n, a + (1 << 20))
        X = bench.gen_rows(torch, dev, cfg, a, b, seed=seed, centres=centres)
        encode_into(pq, X, rows, a)
        del X
    Q = bench.make_queries(torch, dev, cfg, centres) if nq else None
    torch.cuda.synchronize()
    return pq, CompressedVectors._from_device(rows), (Q.cpu().numpy() if nq else None), centres


def report_c3(torch, dev):
    import bench
    from polarquant_b200 import Quantizer
    cfg = bench.WORKLOADS["c3"]
    # 16 blocks of 4,096 rows spread over the 4M-row corpus.
    starts = np.linspace(0, cfg["n"] - 4096, 16).astype(np.int64)
    X = np.concatenate([bench.gen_rows(torch, dev, cfg, int(a), int(a) + 4096, seed=3,
                                       centres=None).cpu().numpy() for a in starts])
    out = {"config": "c3 " + cfg["name"], "rows_checked": int(len(X)), "widths": {}}
    for b in cfg["widths"]:
        pq = Quantizer(cfg["d"], bits=b, seed=42)
        cv = pq.encode(X)
        ref, rn = O.encode(X, pq.R, pq.boundaries)
        out["widths"][str(b)] = encode_counts(cv.indices, cv.norms, X, pq.R, pq.boundaries, ref,
                                              rn)
    return out


def report_c1(torch, dev):
    import bench
    from polarquant_b200 import Quantizer
    cfg = bench.WORKLOADS["c1"]
    X = bench.gen_rows(torch, dev, cfg, 0, cfg["n"], seed=1, centres=None).cpu().numpy()
    Q = bench.make_queries(torch, dev, cfg, None).cpu().numpy()
    pq = Quantizer(cfg["d"], bits=4, seed=42)
    cv = pq.encode(X)
    ref, rn = O.encode(X, pq.R, pq.boundaries)
    enc = encode_counts(cv.indices, cv.norms, X, pq.R, pq.boundaries, ref, rn)
    GI, GS = pq.search_adc_many(cv, Q, k=10)
    RI = np.empty((len(Q), 10), np.intp)
    RS = np.empty((len(Q), 10), np.float32)
    for q in range(len(Q)):
        RI[q], RS[q] = O.search_adc(pq.R, pq.centroids, pq._nested, 4, cv.indices, cv.norms,
                                    Q[q], k=10)
    return {"config": "c1 " + cfg["name"], "encode": enc, "search_adc": search_counts(GI, GS,
                                                                                      RI, RS)}


def report_c2(torch, dev):
    import bench
    cfg = bench.WORKLOADS["c2"]
    pq, cv, Q, _ = corpus(torch, dev, cfg, cfg["n"], cfg["nq"])
    GI, GS = pq.search_twostage_many(cv, Q, k=10, candidates=200, coarse_precision=4)
    pick = np.linspace(0, len(Q) - 1, 256).astype(np.int64)
    RI, RS = O.search_twostage_chunked(pq.R, pq.centroids, pq._nested, 8, cv.indices, cv.norms,
                                       Q[pick], k=10, candidates=200, coarse_precision=4)
    return {"config": "c2 " + cfg["name"],
            "search_twostage": search_counts(GI[pick], GS[pick], RI, RS)}


def report_c4(torch, dev):
    import bench
    cfg = bench.WORKLOADS["c4"]
    n, nq, k = 1 << 21, 1024, 100
    pq, cv, Q, _ = corpus(torch, dev, cfg, n, nq)
    rows = cv._device()
    GI, GS = pq.search_adc_many(cv, Q, k=k)
    s, i = pq._scan(rows, pq._rotate(Q, rows.device), k, 4, force="scan")
    vs_scan = search_counts(GI, GS, i.cpu().numpy(), s.cpu().numpy())
    pick = np.linspace(0, nq - 1, 128).astype(np.int64)
    RI, RS = O.search_batch_chunked(pq.R, pq.centroids, pq._nested, 4, cv.indices, cv.norms,
                                    Q[pick], k=k)
    return {"config": f"c4 distribution at {n} rows x {nq} queries: " + cfg["name"],
            "batched_vs_oracle": search_counts(GI[pick], GS[pick], RI, RS),
            "batched_vs_exact_scan": vs_scan}


def report_c5(torch, dev):
    import bench
    from polarquant_b200 import IVFCoarseIndex
    cfg = bench.WORKLOADS["c5"]
    pq, cv, Q, _ = corpus(torch, dev, cfg, cfg["n"], cfg["nq"])
    ix = IVFCoarseIndex(pq, cv, n_bits=12, mode="lsh", seed=0)
    idx, norms = cv.indices, cv.norms
    cells = O.ivf_cell_ids(idx, 4, 12, "lsh", ix.hyperplanes)
    cell_diff = int((cells != ix.cell_ids).sum())
    ids, sc = ix.search_twostage_many(Q, k=10, candidates=500, nprobe=32, coarse_precision=2)
    pick = np.linspace(0, len(Q) - 1, 128).astype(np.int64)
    ref = []
    for j, q in enumerate(pick):
        ri, rs = O.ivf_search_twostage(pq.R, pq.centroids, pq._nested, 4, idx, norms,
                                       ix.sorted_idx, ix.cell_offsets, 12, "lsh",
                                       ix.hyperplanes, Q[q], k=10, candidates=500, nprobe=32,
                                       coarse_precision=2)
        ref.append((ri, rs))
    out = {"config": "c5 " + cfg["name"], "rows": int(cfg["n"]),
           "cell_ids_differing_from_oracle": cell_diff}
    bad = diff = 0
    rel = 0.0
    for j, q in enumerate(pick):
        ri, rs = ref[j]
        keep = ids[q] >= 0
        gi, gs = ids[q][keep], sc[q][keep]
        bad += not O.topk_equal_up_to_ties(gi, gs, ri, rs, rtol=RTOL)
        diff += (len(gi) != len(ri)) or bool(np.any(gi != ri))
        if len(gi) == len(ri) and len(gi):
            rel = max(rel, float(np.abs(gs.astype(np.float64) - rs).max()) /
                      max(1e-30, float(np.abs(rs).max())))
    out["ivf_search_twostage"] = {"queries": int(len(pick)), "topk_mismatch_after_ties": int(bad),
                                  "id_lists_differing": int(diff), "max_score_rel_diff": rel,
                                  "rtol": RTOL}
    return out


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--out", default="")
    ap.add_argument("--only", default="c3,c1,c2,c4,c5")
    args = ap.parse_args()
    import torch
    torch.cuda.set_device(0)
    dev = torch.device("cuda", 0)
    fns = {"c1": report_c1, "c2": report_c2, "c3": report_c3, "c4": report_c4, "c5": report_c5}
    lines = []
    env = {"numpy": np.__version__, "torch": torch.__version__, "host_cores": os.cpu_count()}
    try:
        import numpy.__config__ as nc
        blas = nc.CONFIG.get("Build Dependencies", {}).get("blas", {})
        env["blas"] = f"{blas.get('name')} {blas.get('version')}"
    except Exception:
        pass
    for name in args.only.split(","):
        t = time.perf_counter()
        r = fns[name](torch, dev)
        r["wall_s"] = round(time.perf_counter() - t, 1)
        r["env"] = env
        print(json.dumps(r), flush=True)
        lines.append(r)
        torch.cuda.empty_cache()
    if args.out:
        with open(args.out, "w") as f:
            for r in lines:
                f.write(json.dumps(r) + "\n")


if __name__ == "__main__":
    main()

"""Benchmark of the B200 encode + ADC-search path.

    python bench.py [--gpus N] [--steps K] [--warmup W] [--impl ours|reference]
                    [--workload c4|c3|c2|c5|c1|c4s] [--quick] [--no-extra]

One JSON line on rank 0.  Workloads (synthetic, seeded, generated on the GPU):

  c4 (default): d=1536, bits=4, 100,000,000 corpus vectors = 10,000 unit
      centres + N(0, (0.2/sqrt(d))^2) noise, re-normalised, row-sharded across
      the ranks; 10,000 queries drawn the same way; batched ADC with k=100 and
      an NCCL all-gather merge.  A step = the whole 10,000-query batch.
  c2: d=768, bits=8, 1,000,000 corpus vectors = 1,000 unit centres
      + N(0, (0.3/sqrt(d))^2) noise, re-normalised; 1,000 queries drawn the
      same way with another seed; search_twostage(coarse_precision=4,
      candidates=200, k=10).  A step = the whole 1,000-query batch.  The
      corpus (768 MB) is larger than L2, so no flush is needed between steps.
  c3: encode sweep, d=1024, 4,000,000 N(0, I) rows scaled by norms drawn
      log-uniform in [0.5, 2]; a step encodes all rows at bits = 2, 3, 4 and 8.
      Metric: vectors/s (16M encodes per step).
  c5: IVF (lsh, 12 bits = 4096 cells), d=384, bits=4, 10,000,000 rows from
      4,096 centres (noise 0.1/sqrt(d)), nprobe=32, 2-bit coarse, 500
      candidates, 4-bit rerank, k=10, 1,000 queries (one GPU).
  c1: d=384, bits=4, 10,000 N(0,1) unit vectors, 200 queries, search_adc k=10
      (L2-resident corpus).
  c4s: the c4 kernel on a 4M-row slice (for ncu captures).

The default run (c4 on one GPU) also measures c1, c2, c3 and c5 after the
headline and records them under "configs" (one sub-record each, with its own
roofline and CPU baseline); --no-extra skips them.

Multi-GPU: rows are sharded contiguously across ranks (torch.distributed,
NCCL); each step runs the exact merge (all-gather of the per-rank top-k).
Timing: CUDA events on the compute stream, barrier + synchronize around the
timed steps, max over ranks.

--impl reference times the reference algorithm's CPU path (the NumPy oracle,
a restatement of remex's own code) on the host cores over a bounded sample of
the same workload, on rank 0 only.
"""

from __future__ import annotations

import argparse
import gc
import json
import os
import subprocess
import sys
import threading
import time

import numpy as np

ROOT = os.path.dirname(os.path.abspath(__file__))
sys.path.insert(0, ROOT)

WORKLOADS = {
    "c2": dict(d=768, bits=8, n=1_000_000, nq=1000, n_centres=1000, sigma=0.3, k=10,
               candidates=200, coarse_precision=4, mode="twostage",
               name="twostage d=768 bits=8 n=1M clustered(1000, 0.3/sqrt(d)) q=1000 "
                    "C=200 cp=4 k=10"),
    "c3": dict(d=1024, bits=4, n=4_000_000, nq=0, n_centres=0, sigma=0.0, k=0, lognorm=True,
               candidates=0, coarse_precision=None, mode="encode", widths=(2, 3, 4, 8),
               name="encode d=1024 n=4M N(0,I) x lognormal-norm[0.5,2], bits 2/3/4/8"),
    "c1": dict(d=384, bits=4, n=10_000, nq=200, n_centres=0, sigma=0.0, k=10,
               candidates=0, coarse_precision=None, mode="adc",
               name="search_adc d=384 bits=4 n=10k N(0,1) unit q=200 k=10"),
    "c4": dict(d=1536, bits=4, n=100_000_000, nq=10_000, n_centres=10_000, sigma=0.2, k=100,
               candidates=0, coarse_precision=None, mode="batch",
               name="batched ADC d=1536 bits=4 n=100M clustered(10000, 0.2/sqrt(d)) q=10000 "
                    "k=100"),
    "c5": dict(d=384, bits=4, n=10_000_000, nq=1000, n_centres=4096, sigma=0.1, k=10,
               candidates=500, coarse_precision=2, mode="ivf", n_bits=12, nprobe=32,
               name="IVF lsh n_bits=12 (4096 cells) nprobe=32 d=384 bits=4 n=10M "
                    "clustered(4096, 0.1/sqrt(d)) q=1000 cp=2 C=500 k=10"),
    # The c4 kernel on a 4M-row slice of the same distribution: small enough
    # for a full ncu capture (3 GB on the device).
    "c4s": dict(d=1536, bits=4, n=4_000_000, nq=10_000, n_centres=10_000, sigma=0.2, k=100,
                candidates=0, coarse_precision=None, mode="batch",
                name="batched ADC d=1536 bits=4 n=4M clustered(10000, 0.2/sqrt(d)) q=10000 "
                     "k=100"),
}

CHUNK = 65536

# DRAM bytes (read + write) per launch of the dominant batched-ADC kernel,
# from an ncu capture of pair_i8_kernel on the 4M-row slice of the d=1536
# workload at 10,000 queries (27.6 GB read + 2.06 GB written), scaled to other
# row counts of the same workload by rows (traffic grows with the row tiles at
# a fixed query batch).
PROFILED_TRAFFIC = {"rows": 4_000_000, "bytes": 29.67e9, "queries": 10_000, "d": 1536,
                    "source": "ncu dram__bytes_read.sum + dram__bytes_write.sum of "
                              "pair_i8_kernel on the 4M-row slice, scaled by rows"}


def log(*a):
    print(*a, file=sys.stderr, flush=True)


def gen_rows(torch, device, cfg, start, stop, seed, centres):
    """Rows [start, stop) of the synthetic corpus, generated chunk-by-chunk with
    per-chunk seeds so any rank can produce its own rows."""
    d = cfg["d"]
    out = torch.empty((stop - start, d), dtype=torch.float32, device=device)
    c0 = start // CHUNK
    c1 = (stop + CHUNK - 1) // CHUNK
    for c in range(c0, c1):
        a, b = c * CHUNK, min((c + 1) * CHUNK, cfg["n"])
        g = torch.Generator(device=device)
        g.manual_seed(seed * 1_000_003 + c)
        x = torch.randn((b - a, d), generator=g, device=device, dtype=torch.float32)
        if centres is not None:
            lab = torch.randint(0, centres.shape[0], (b - a,), generator=g, device=device)
            x = centres[lab] + x * (cfg["sigma"] / np.sqrt(d))
        x = x / torch.linalg.vector_norm(x, dim=1, keepdim=True)
        if cfg.get("lognorm"):
            u = torch.rand((b - a, 1), generator=g, device=device)
            x = x * torch.exp(np.log(0.5) + u * (np.log(2.0) - np.log(0.5)))
        lo, hi = max(a, start), min(b, stop)
        out[lo - start:hi - start] = x[lo - a:hi - a]
    return out


def make_centres(torch, device, cfg, seed):
    if not cfg["n_centres"]:
        return None
    g = torch.Generator(device=device)
    g.manual_seed(seed)
    c = torch.randn((cfg["n_centres"], cfg["d"]), generator=g, device=device)
    return c / torch.linalg.vector_norm(c, dim=1, keepdim=True)


def make_queries(torch, device, cfg, centres):
    qcfg = dict(cfg, n=cfg["nq"])
    return gen_rows(torch, device, qcfg, 0, cfg["nq"], seed=99, centres=centres)


class ClockSampler:
    """nvidia-smi clock/throttle samples during the timed region."""

    FIELDS = ("index,clocks.sm,clocks.max.sm,power.draw,clocks_event_reasons.active,"
              "clocks_event_reasons.hw_slowdown,clocks_event_reasons.hw_thermal_slowdown,"
              "clocks_event_reasons.sw_thermal_slowdown,clocks_event_reasons.sw_power_cap")

    def __init__(self, gpu_index: int):
        self.gpu = gpu_index
        self.proc = None
        self.lines = []

    def start(self):
        try:
            self.proc = subprocess.Popen(
                ["nvidia-smi", "-i", str(self.gpu), f"--query-gpu={self.FIELDS}",
                 "--format=csv,noheader,nounits", "-lms", "200"],
                stdout=subprocess.PIPE, stderr=subprocess.DEVNULL, text=True)
            self.t = threading.Thread(target=self._read, daemon=True)
            self.t.start()
        except OSError:
            self.proc = None

    def _read(self):
        for line in self.proc.stdout:
            self.lines.append(line.strip())

    def stop(self):
        if self.proc is None:
            return {"sm_mhz": None, "sm_max_mhz": None, "reasons": ["nvidia-smi unavailable"]}
        time.sleep(0.3)
        self.proc.terminate()
        try:
            self.proc.wait(timeout=5)
        except subprocess.TimeoutExpired:
            self.proc.kill()
        sm, smax, reasons = [], None, set()
        names = ["hw_slowdown", "hw_thermal_slowdown", "sw_thermal_slowdown", "sw_power_cap"]
        for ln in self.lines:
            f = [x.strip() for x in ln.split(",")]
            if len(f) < 9:
                continue
            try:
                sm.append(float(f[1]))
                smax = float(f[2])
            except ValueError:
                continue
            for nm, v in zip(names, f[5:9]):
                if v.lower().startswith("active"):
                    reasons.add(nm)
        return {"sm_mhz": float(np.median(sm)) if sm else None, "sm_max_mhz": smax,
                "reasons": sorted(reasons), "samples": len(sm)}


def measured_peaks():
    """HBM GB/s, dense bf16 TFLOP/s burst and sustained, and where they came from."""
    try:
        with open(os.path.join(ROOT, "MEASURED_PEAKS.json")) as f:
            p = json.load(f)
        bf = float(p["bf16_tflops"])
        return {"hbm": float(p["hbm_gbs"]), "bf16": bf,
                "bf16_sustained": float(p.get("bf16_tflops_sustained", bf)), "kind": "measured"}
    except (OSError, KeyError, ValueError):
        return {"hbm": 6650.0, "bf16": 1590.0, "bf16_sustained": 1400.0, "kind": "fallback"}


def tensor_peak(pk, launch_ms):
    """The bf16 denominator for a kernel: the sustained figure for launches
    long enough to run under the power cap (>= 1 s), else the burst one."""
    if launch_ms >= 1000.0:
        return pk["bf16_sustained"], f"{pk['kind']} dense bf16 (sustained)"
    return pk["bf16"], f"{pk['kind']} dense bf16 (burst)"


def topk_agree(ids_a, s_a, ids_b, s_b, rtol=1e-4):
    """Two descending top-k lists agree up to score ties: scores equal within
    rtol of the list's largest |score|, and ids outside the other list only
    where their score ties the k-th score within that band."""
    ids_a, ids_b = np.asarray(ids_a), np.asarray(ids_b)
    s_a, s_b = np.asarray(s_a, np.float64), np.asarray(s_b, np.float64)
    if ids_a.shape != ids_b.shape:
        return False
    if ids_a.size == 0:
        return True
    tol = rtol * max(1e-30, float(np.abs(s_b).max()))
    if np.abs(s_a - s_b).max() > tol:
        return False
    kth = s_b[-1]
    sa, sb = set(ids_a.tolist()), set(ids_b.tolist())
    for i, s in zip(ids_a.tolist(), s_a.tolist()):
        if i not in sb and abs(s - kth) > tol:
            return False
    for i, s in zip(ids_b.tolist(), s_b.tolist()):
        if i not in sa and abs(s - kth) > tol:
            return False
    return True


def compare_topk(s_a, i_a, s_b, i_b, rtol=1e-4):
    """Mismatch count (up to ties) and the largest score difference relative
    to each list's largest |score|, over the rows of two (m, k) result sets."""
    bad, rel = 0, 0.0
    for q in range(len(i_a)):
        bad += not topk_agree(i_a[q], s_a[q], i_b[q], s_b[q], rtol)
        den = max(1e-30, float(np.abs(s_b[q]).max()))
        rel = max(rel, float(np.abs(s_a[q].astype(np.float64) - s_b[q]).max()) / den)
    return bad, rel


# ---------------------------------------------------------------------------
# CPU baseline (oracle = NumPy restatement of the reference path)
# ---------------------------------------------------------------------------

def cpu_baseline(cfg, X_sample, Q_host, pq, budget_s=20.0):
    """The reference algorithm on the host cores (the NumPy oracle, which runs the
    reference's own NumPy calls) over a bounded sample of the corpus rows.
    Search cost is linear in the corpus rows, so queries/s for the full corpus
    is the sample rate scaled by sample_rows / n (stated in `sample`).

    batch: Quantizer.search_batch as the reference runs it -- the dequantised
    X_hat_rot built once per corpus and cached (remex/core.py:861-880, built
    outside the timed loop), then one sgemm per block of 1,000 queries and a
    per-row argpartition top-k (remex/core.py:756-778).  adc / twostage / ivf:
    the reference's single-query calls, one query at a time (its API takes one
    query per call); the IVF index is built before the timed loop."""
    from oracle import remex_oracle as O
    t_enc = time.perf_counter()
    codes, norms = O.encode(X_sample, pq.R, pq.boundaries)
    t_enc = time.perf_counter() - t_enc
    m = len(norms)
    scale = m / cfg["n"]
    mode = cfg["mode"]
    prep = ""
    if mode == "batch":
        t = time.perf_counter()
        Xh = O.x_hat_rot(pq.centroids, pq._nested, cfg["bits"], codes)
        prep = f"; X_hat_rot cache built once in {time.perf_counter() - t:.1f} s (not timed)"
    elif mode == "ivf":
        t = time.perf_counter()
        H = O.lsh_hyperplanes(cfg["n_bits"], cfg["d"], 0)
        cells = O.ivf_cell_ids(codes, cfg["bits"], cfg["n_bits"], "lsh", H)
        srt, off = O.ivf_csr(cells, 1 << cfg["n_bits"])
        prep = f"; IVF index built in {time.perf_counter() - t:.1f} s (not timed)"
    block = 1000
    nq_done, t0 = 0, time.perf_counter()
    while nq_done < len(Q_host) and (time.perf_counter() - t0) < budget_s:
        if mode == "batch":
            Qb = Q_host[nq_done:nq_done + block]
            O.search_batch_cached(pq.R, Xh, norms, Qb, k=cfg["k"])
            nq_done += len(Qb)
            continue
        q = Q_host[nq_done]
        if mode == "twostage":
            O.search_twostage(pq.R, pq.centroids, pq._nested, cfg["bits"], codes, norms, q,
                              k=cfg["k"], candidates=cfg["candidates"],
                              coarse_precision=cfg["coarse_precision"])
        elif mode == "ivf":
            O.ivf_search_twostage(pq.R, pq.centroids, pq._nested, cfg["bits"], codes, norms,
                                  srt, off, cfg["n_bits"], "lsh", H, q, k=cfg["k"],
                                  candidates=cfg["candidates"], nprobe=cfg["nprobe"],
                                  coarse_precision=cfg["coarse_precision"])
        else:
            O.search_adc(pq.R, pq.centroids, pq._nested, cfg["bits"], codes, norms, q,
                         k=cfg["k"])
        nq_done += 1
    dt = time.perf_counter() - t0
    how = (f"search_batch over {nq_done} queries in blocks of {block} (one sgemm per block)"
           if mode == "batch" else f"{nq_done} single-query calls")
    return {"value": nq_done / dt * scale, "unit": "queries/s", "cores": os.cpu_count(),
            "kind": "port",
            "sample": f"{how} over a {m}-row sample of the {cfg['n']}-row corpus in {dt:.1f} s, "
                      f"scaled by {m}/{cfg['n']}"
                      + (" (extrapolated)" if m < cfg["n"] else "") + prep
                      + f"; NumPy encode of the sample {m / t_enc:.0f} vectors/s",
            "encode_vectors_per_s": m / t_enc}


# ---------------------------------------------------------------------------
# Encode sweep (c3)
# ---------------------------------------------------------------------------

def encode_sweep(args, cfg, torch, dist, dev, world, rank, steps, warmup, with_cpu,
                 cpu_rows=100_000):
    """Every step encodes this rank's rows at each width (remex/core.py:484-511).
    Returns the result record (not printed)."""
    from polarquant_b200 import Quantizer, _lib
    from polarquant_b200.distributed import shard_bounds
    from polarquant_b200.encode import alloc_corpus, encode_into
    widths = cfg["widths"]
    qz = {b: Quantizer(cfg["d"], bits=b, seed=42) for b in widths}
    sample_rows = cpu_rows
    r0, r1 = shard_bounds(cfg["n"], world, rank)
    X = gen_rows(torch, dev, cfg, r0, r1, seed=3, centres=None)
    corp = {b: alloc_corpus(qz[b], r1 - r0, dev) for b in widths}

    def barrier():
        if world > 1:
            dist.barrier()
        torch.cuda.synchronize()

    for _ in range(max(3, warmup)):
        for b in widths:
            encode_into(qz[b], X, corp[b], 0)
    barrier()
    launches0 = _lib.query("pq_launch_count")
    clk = ClockSampler(dev.index)
    clk.start()
    barrier()
    t0, t1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    per = {b: [] for b in widths}
    t0.record()
    for _ in range(steps):
        for b in widths:
            a_, b_ = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
            a_.record()
            encode_into(qz[b], X, corp[b], 0)
            b_.record()
            per[b].append((a_, b_))
    t1.record()
    barrier()
    clocks = clk.stop()
    launches = _lib.query("pq_launch_count") - launches0
    ms = t0.elapsed_time(t1) / steps
    ms_t = torch.tensor([ms], device=dev)
    if world > 1:
        dist.all_reduce(ms_t, op=dist.ReduceOp.MAX)
    ms = float(ms_t.item())
    nrows = cfg["n"] * len(widths)
    pk = measured_peaks()
    flops_w = 2.0 * (r1 - r0) * cfg["d"] ** 2
    per_w = {}
    for b in widths:
        wms = float(np.mean([x.elapsed_time(y) for x, y in per[b]]))
        tf = flops_w / (wms / 1e3) / 1e12
        per_w[str(b)] = {"vectors_per_s": (r1 - r0) * world / (wms / 1e3), "ms": wms,
                         "tflops": tf, "frac": tf / pk["bf16"]}
    flops = flops_w * len(widths)
    ach = flops / (ms / 1e3) / 1e12
    line = {"metric": "encode vectors/s", "value": nrows / (ms / 1e3), "unit": "vectors/s",
            "n_gpus": world, "steps": steps, "warmup": max(3, warmup),
            "ms_per_step": ms, "higher_is_better": True, "scaling": "strong",
            "vs_baseline": None, "dtype": "f32 in, fp16 hi/lo split on tcgen05, codes out",
            "data": "synthetic",
            "config": {"workload": cfg["name"], "global_batch": cfg["n"],
                       "parallelism": f"row-shard x{world}",
                       "l2": "16.8 GB input, larger than L2"},
            "per_width": per_w,
            "roofline": {"bound": "tensor", "achieved": ach, "peak": pk["bf16"],
                         "unit": "TFLOP/s", "frac": ach / pk["bf16"], "traffic": None,
                         "kernel": "encode_prep_kernel + encode_gemm_kernel (whole encode; 3 "
                                   "MMAs per algorithmic MAC)",
                         "peak_kind": f"{pk['kind']} dense bf16 (burst)",
                         "alg_flops_per_step": flops},
            "gpu_launches": int(launches), "clocks": clocks}
    if not args.quick:
        # e2e: host f32 rows in, packed codes + norms back (one width per step).
        sub = min(r1 - r0, 1_000_000)
        Xh = torch.empty((sub, cfg["d"]), dtype=torch.float32, pin_memory=True)
        Xh.copy_(X[:sub].cpu())
        q4 = qz[4]
        q4.encode(Xh[:1024])
        barrier()
        e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        e0.record()
        cv = q4.encode(Xh.to(dev, non_blocking=True))
        packed = cv._rows.buf[: sub * cv._rows.ldb].cpu()
        nrm = cv._rows.norms.cpu()
        e1.record()
        barrier()
        ems = e0.elapsed_time(e1)
        line["e2e"] = {"value": sub * world / (ems / 1e3), "unit": "vectors/s",
                       "h2d_bytes_per_step": int(sub * cfg["d"] * 4),
                       "d2h_bytes_per_step": int(packed.numel() + nrm.numel() * 4),
                       "note": "public encode() on 1M host rows at bits=4, results copied back"}
        del cv, packed, nrm, Xh
    if with_cpu and rank == 0 and world == 1:
        Xs = X[:sample_rows].cpu().numpy()
        from oracle import remex_oracle as O
        t0_ = time.perf_counter()
        for b in widths:
            O.encode(Xs, qz[b].R, qz[b].boundaries)
        dt = time.perf_counter() - t0_
        line["cpu_baseline"] = {"value": sample_rows * len(widths) / dt,
                                "unit": "vectors/s", "cores": os.cpu_count(),
                                "kind": "port",
                                "sample": f"NumPy encode of {sample_rows} rows at each of "
                                          f"bits {list(widths)} in {dt:.1f} s"}
    del X, corp
    return line


def encode_reference_line(args, cfg, torch, dev, world):
    from polarquant_b200 import Quantizer
    from oracle import remex_oracle as O
    widths = cfg["widths"]
    sample_rows = 100_000
    Xs = gen_rows(torch, dev, cfg, 0, sample_rows, seed=3, centres=None).cpu().numpy()
    t0 = time.perf_counter()
    for b in widths:
        qb = Quantizer(cfg["d"], bits=b, seed=42)
        O.encode(Xs, qb.R, qb.boundaries)
    dt = time.perf_counter() - t0
    v = sample_rows * len(widths) / dt
    return {"metric": "encode vectors/s", "value": v, "unit": "vectors/s",
            "impl": "reference", "n_gpus": world, "steps": args.steps, "warmup": args.warmup,
            "higher_is_better": True, "dtype": "f32", "data": "synthetic",
            "config": {"workload": cfg["name"]},
            "cpu_baseline": {"value": v, "unit": "vectors/s", "cores": os.cpu_count(),
                             "kind": "port",
                             "sample": f"NumPy encode of {sample_rows} rows at each of bits "
                                       f"{list(widths)} in {dt:.1f} s"},
            "e2e": {"value": v, "unit": "vectors/s", "h2d_bytes_per_step": 0,
                    "d2h_bytes_per_step": 0}}


# ---------------------------------------------------------------------------
# Search workloads (c1, c2, c4, c5)
# ---------------------------------------------------------------------------

def scan_kernel_name(rows, nq, k, p):
    from polarquant_b200 import _lib
    kind = _lib.query("pq_adc_scan_kernel", rows.n, rows.d, rows.bits, p, nq, k, rows.ldb)
    return {4: "scan_bt_kernel (byte tables) + bt_score_kernel", 2: "scan2_kernel (TMA-staged)",
            1: "scan_topk_kernel", 3: "score_keys + sort"}.get(
        kind, "?")


def scan_rate(pq, rows, qrot, k, p, torch, reps=3):
    """One pq_adc_scan launch over the corpus for qrot's queries: ms per launch."""
    pq._scan(rows, qrot, k, p, force="scan")
    torch.cuda.synchronize()
    k0, k1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    k0.record()
    for _ in range(reps):
        pq._scan(rows, qrot, k, p, force="scan")
    k1.record()
    torch.cuda.synchronize()
    return k0.elapsed_time(k1) / reps


def search_workload(args, cfg, torch, dist, dev, world, rank, steps, warmup, headline,
                    with_cpu):
    """Builds this rank's shard, times `steps` steps of the workload and returns
    the result record (printed by the caller)."""
    from polarquant_b200 import Quantizer, _lib
    from polarquant_b200.core import CompressedVectors
    from polarquant_b200.distributed import ShardedSearch, shard_bounds
    from polarquant_b200.encode import alloc_corpus, encode_into

    pq = Quantizer(cfg["d"], bits=cfg["bits"], seed=42)
    centres = make_centres(torch, dev, cfg, seed=7)
    Q = make_queries(torch, dev, cfg, centres)
    sample_rows = min(cfg["n"], 100_000 if headline else 20_000)

    # ---- this rank's shard (generated and encoded chunk by chunk) -----------
    r0, r1 = shard_bounds(cfg["n"], world, rank)
    rows = alloc_corpus(pq, r1 - r0, dev)
    enc_ms = 0.0
    step_rows = 1 << 20
    for a in range(r0, r1, step_rows):
        b = min(r1, a + step_rows)
        X = gen_rows(torch, dev, cfg, a, b, seed=1, centres=centres)
        if a == r0:
            encode_into(pq, X[: min(len(X), 4096)], rows, 0)  # warm the encode path
        e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        e0.record()
        encode_into(pq, X, rows, a - r0)
        e1.record()
        torch.cuda.synchronize()
        enc_ms += e0.elapsed_time(e1)
        del X
    enc_vps = (r1 - r0) / (enc_ms / 1e3)
    cv = CompressedVectors._from_device(rows)
    ss = ShardedSearch(pq, cv, r0, cfg["n"])
    if args.path != "auto" and headline:
        ss.force = args.path
    kern_ms = []
    _local_topk = ss.local_topk

    def timed_local_topk(qrot, k, p):
        a_, b_ = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        a_.record()
        out = _local_topk(qrot, k, p)
        b_.record()
        kern_ms.append((a_, b_))
        return out
    ss.local_topk = timed_local_topk

    ivf = None
    if cfg["mode"] == "ivf":
        from polarquant_b200 import IVFCoarseIndex
        if world > 1:
            raise SystemExit("the ivf workload runs on one GPU")
        ivf = IVFCoarseIndex(pq, cv, n_bits=cfg["n_bits"], mode="lsh", seed=0)

    def step(Qin):
        if ivf is not None:
            a_, b_ = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
            a_.record()
            out = ivf.search_twostage_many(Qin, k=cfg["k"], candidates=cfg["candidates"],
                                           nprobe=cfg["nprobe"],
                                           coarse_precision=cfg["coarse_precision"])
            b_.record()
            kern_ms.append((a_, b_))
            return out
        if cfg["mode"] == "twostage":
            return ss.search_twostage_many(Qin, k=cfg["k"], candidates=cfg["candidates"],
                                           coarse_precision=cfg["coarse_precision"])
        return ss.search_adc_many(Qin, k=cfg["k"])

    qrot0 = pq._rotate(Q, dev)
    p_scan = cfg["coarse_precision"] or cfg["bits"]
    k_scan = min(cfg["candidates"] or cfg["k"], rows.n)
    from polarquant_b200.core import use_tensor_cores
    batched = (cfg["mode"] != "ivf"
               and use_tensor_cores(rows.n, cfg["nq"], k_scan, rows.row_bytes, rows.bits, rows.d)
               and args.path != "scan") or (headline and args.path == "batch")

    def barrier():
        if world > 1:
            dist.barrier()
        torch.cuda.synchronize()

    for _ in range(max(3, warmup)):
        res = step(Q)
    barrier()
    kern_ms.clear()
    launches0 = _lib.query("pq_launch_count")
    clk = ClockSampler(dev.index)
    clk.start()
    barrier()
    t0, t1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    t0.record()
    for _ in range(steps):
        res = step(Q)
    t1.record()
    barrier()
    clocks = clk.stop()
    ms = t0.elapsed_time(t1) / steps
    launches = _lib.query("pq_launch_count") - launches0
    kms = sum(a_.elapsed_time(b_) for a_, b_ in kern_ms) / max(1, len(kern_ms))
    ms_t = torch.tensor([ms], device=dev)
    if world > 1:
        dist.all_reduce(ms_t, op=dist.ReduceOp.MAX)
    ms = float(ms_t.item())
    qps = cfg["nq"] / (ms / 1e3)

    if args.quick:
        return {"metric": "queries/s", "value": qps, "ms_per_step": ms, "kernel_ms": kms,
                "n_gpus": world, "quick": True, "encode_vectors_per_s": enc_vps * world,
                "config": {"workload": cfg["name"], "corpus_rows": cfg["n"]}, "clocks": clocks}

    line = {
        "metric": "queries/s", "value": qps, "unit": "queries/s", "n_gpus": world,
        "steps": steps, "warmup": max(3, warmup), "ms_per_step": ms,
        "higher_is_better": True, "scaling": "strong", "vs_baseline": None,
        "dtype": "u8 codes, f32 scores", "data": "synthetic",
        "config": {"workload": cfg["name"], "global_batch": cfg["nq"],
                   "corpus_rows": cfg["n"], "parallelism": f"row-shard x{world}",
                   "l2": "corpus larger than L2 (no flush needed)"
                   if cfg["n"] * (rows.row_bytes + 4) > 126e6 else "corpus L2-resident"},
    }

    # ---- parity of the timed path against the exact streaming scan ---------
    # (rank 0 of a one-GPU run; the exact scan's scores are the f32 table sums
    # that the oracle-pinned GPU tests check).  Batched ADC: the int8
    # candidates + exact rescoring against an exact scan of the whole corpus.
    # Two-stage: the batched coarse stage + rerank against the same search
    # with the coarse stage on the exact scan.
    if world == 1 and cfg["mode"] in ("batch", "twostage"):
        ns = min(16, cfg["nq"])
        pick = np.linspace(0, cfg["nq"] - 1, ns).astype(np.int64)
        s_got, i_got = res
        s_got, i_got = s_got.cpu().numpy()[pick], i_got.cpu().numpy()[pick]
        qsel = Q[torch.from_numpy(pick).to(dev)]
        if cfg["mode"] == "batch":
            es, ei = pq._scan(rows, pq._rotate(qsel, dev), cfg["k"], cfg["bits"], force="scan")
            what = "batched ADC (int8 candidates + exact rescoring) vs pq_adc_scan"
        else:
            ss.force = "scan"
            es, ei = ss.search_twostage_many(qsel, k=cfg["k"], candidates=cfg["candidates"],
                                             coarse_precision=cfg["coarse_precision"])
            ss.force = None
            what = "twostage with batched coarse vs twostage with the exact scan coarse"
        bad, rel = compare_topk(s_got, i_got, es.cpu().numpy(), ei.cpu().numpy())
        line["parity"] = {"queries_checked": int(ns), "check": what,
                          "topk_mismatch_after_ties": int(bad), "max_score_rel_diff": rel,
                          "rtol": 1e-4}

    # ---- end to end through the public API with host buffers ---------------
    if headline:
        Qh = torch.empty(Q.shape, dtype=torch.float32, pin_memory=True)
        Qh.copy_(Q.cpu())
        barrier()
        ee0, ee1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        d2h = 0
        e2e_steps = max(1, min(steps, int(np.ceil(10_000.0 / max(ms, 1.0)))))
        ee0.record()
        for _ in range(e2e_steps):
            Qd = Qh.to(dev, non_blocking=True)
            out = step(Qd)
            if ivf is not None:
                ids, sc = out
                d2h = ids.size * 8 + sc.size * 4
            else:
                s, i = out
                ids, sc = i.cpu(), s.cpu()
                d2h = ids.numel() * 8 + sc.numel() * 4
        ee1.record()
        barrier()
        e2e_ms = ee0.elapsed_time(ee1) / e2e_steps
        e2e_t = torch.tensor([e2e_ms], device=dev)
        if world > 1:
            dist.all_reduce(e2e_t, op=dist.ReduceOp.MAX)
        e2e_ms = float(e2e_t.item())
        line["e2e"] = {"value": cfg["nq"] / (e2e_ms / 1e3), "unit": "queries/s",
                       "h2d_bytes_per_step": int(Q.numel() * 4), "d2h_bytes_per_step": int(d2h)}

    # ---- dominant kernel ----------------------------------------------------
    # Batches of >= 64 queries (>= 8 on corpora of 2^20+ rows) run the per-rank
    # ADC on the tensor cores (pq_adc_batch: pair_i8_kernel for 2/4/8-bit codes
    # at d >= 1024, then the exact rescoring of its candidates; timed inside
    # the steps above, all of its launches): bound = tensor, algorithmic work
    # 2*nq*n_local*d flops per call (each MAC counted once; the int8 split
    # issues three int8 MMAs per MAC), against the measured dense bf16 peak --
    # the int8 pipe's nominal rate is twice that.
    pk = measured_peaks()
    row_bytes = rows.row_bytes + 4
    roof = None
    if batched:
        flops = 2.0 * cfg["nq"] * rows.n * cfg["d"]
        ach = flops / (kms / 1e3) / 1e12
        peak, pkind = tensor_peak(pk, kms)
        pt = PROFILED_TRAFFIC
        same = (cfg["d"] == pt["d"] and cfg["nq"] == pt["queries"] and cfg["bits"] == 4)
        traffic = pt["bytes"] * rows.n / pt["rows"] if same else None
        i8 = cfg["d"] >= 1024 and cfg["bits"] in (2, 4, 8)
        roof = {"bound": "tensor", "achieved": ach, "peak": peak, "unit": "TFLOP/s",
                "frac": ach / peak, "frac_of_burst_peak": ach / pk["bf16"], "traffic": traffic,
                "traffic_source": pt["source"] if same else None,
                "kernel": ("pair_i8_kernel (tcgen05 kind::i8 CTA pairs, 3 int8 MMAs per MAC) + "
                           "exact rescoring of K+32 candidates" if i8 else
                           "pair_adc_kernel / batched_adc_kernel (tcgen05 kind::f16, fp16 hi/lo "
                           "split, 3 MMAs per MAC)") + " (whole per-rank batched call)",
                "peak_kind": pkind, "alg_flops_per_launch": flops, "launch_ms": kms,
                "alg_flops_basis": "2*d per (query, row) pair"}
    # The streaming single-query scan (pq_adc_scan) on the same corpus: HBM-bound.
    # nq=1 is search_adc's own case; 8 queries per launch share each row in L2.
    scan_roofs = {}
    for nsq in (1, 8 if rows.n > 5_000_000 else min(64, cfg["nq"])):
        qs = qrot0[:nsq].contiguous()
        sms = scan_rate(pq, rows, qs, k_scan, p_scan, torch)
        sbytes = nsq * rows.n * row_bytes
        sgbs = sbytes / (sms / 1e3) / 1e9
        scan_roofs[nsq] = {"bound": "hbm", "achieved": sgbs, "peak": pk["hbm"], "unit": "GB/s",
                           "frac": sgbs / pk["hbm"], "queries_per_launch": nsq,
                           "launch_ms": sms,
                           "kernel": scan_kernel_name(rows, nsq, k_scan, p_scan) +
                                     " + merge, whole pq_adc_scan call, one corpus pass per query",
                           "peak_kind": pk["kind"], "alg_bytes_per_launch": sbytes,
                           "alg_bytes_basis": "row_bytes + 4 per row per query"}
    scan_roof = scan_roofs[1]
    if ivf is not None:
        # IVF: the gather-scan visits the probed cells' rows (row_bytes + 4 +
        # 8-byte CSR id each); algorithmic bytes per launch from the index.
        sizes = np.diff(ivf.cell_offsets)
        Qh_ = Q.cpu().numpy()
        visited = 0
        for qi in range(cfg["nq"]):
            visited += int(sizes[ivf.probe_cells(ivf.query_cell(Qh_[qi]),
                                                 cfg["nprobe"])].sum())
        ibytes = visited * (row_bytes + 8)
        roof = {"bound": "hbm", "achieved": ibytes / (kms / 1e3) / 1e9, "peak": pk["hbm"],
                "unit": "GB/s", "frac": ibytes / (kms / 1e3) / 1e9 / pk["hbm"], "traffic": None,
                "kernel": "ivf_group_scan_kernel + rerank (whole pq_ivf_search call)",
                "peak_kind": pk["kind"], "alg_bytes_per_launch": ibytes, "launch_ms": kms,
                "rows_visited_per_query": visited / cfg["nq"]}
    elif not batched:
        roof = dict(scan_roofs[max(scan_roofs)], traffic=None)
    alg_bytes = cfg["nq"] * rows.n * row_bytes
    line.update({
        "scan_gbs": alg_bytes / (ms / 1e3) / 1e9,
        "roofline": roof,
        "scan_roofline": scan_roof,
        "scan_roofline_multi": scan_roofs[max(scan_roofs)],
        "encode": {"vectors_per_s": enc_vps * world, "ms": enc_ms, "rows_per_rank": r1 - r0},
        "gpu_launches": int(launches),
        "clocks": clocks,
    })
    if with_cpu and rank == 0 and world == 1:
        Xs = gen_rows(torch, dev, cfg, 0, sample_rows, seed=1, centres=centres).cpu().numpy()
        line["cpu_baseline"] = cpu_baseline(cfg, Xs, Q.cpu().numpy(), pq,
                                            budget_s=20.0 if headline else 5.0)
    del ss, cv, rows, ivf, res
    return line


def reference_line(args, cfg, torch, dev, world):
    from polarquant_b200 import Quantizer
    pq = Quantizer(cfg["d"], bits=cfg["bits"], seed=42)
    centres = make_centres(torch, dev, cfg, seed=7)
    Q = make_queries(torch, dev, cfg, centres)
    sample_rows = min(cfg["n"], 100_000)
    Xs = gen_rows(torch, dev, cfg, 0, sample_rows, seed=1, centres=centres).cpu().numpy()
    cb = cpu_baseline(cfg, Xs, Q.cpu().numpy(), pq, budget_s=max(10.0, 2.0 * args.steps))
    return {"metric": "queries/s", "value": cb["value"], "unit": "queries/s",
            "impl": "reference", "n_gpus": world, "steps": args.steps,
            "warmup": args.warmup, "higher_is_better": True, "dtype": "f32",
            "data": "synthetic", "config": {"workload": cfg["name"]},
            "cpu_baseline": cb,
            "e2e": {"value": cb["value"], "unit": "queries/s", "h2d_bytes_per_step": 0,
                    "d2h_bytes_per_step": 0}}


def free_device(torch):
    gc.collect()
    torch.cuda.synchronize()
    torch.cuda.empty_cache()


# ---------------------------------------------------------------------------

def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=3)
    ap.add_argument("--warmup", type=int, default=3)
    ap.add_argument("--impl", default="ours", choices=["ours", "reference"])
    ap.add_argument("--workload", default="c4", choices=sorted(WORKLOADS))
    ap.add_argument("--path", default="auto", choices=["auto", "scan", "batch"],
                    help="force the streaming scan or the tensor-core batch path")
    ap.add_argument("--queries", type=int, default=0, help="override the query count")
    ap.add_argument("--rows", type=int, default=0,
                    help="override the corpus row count (small cases for ncu captures)")
    ap.add_argument("--quick", action="store_true",
                    help="timed steps only (no e2e, scan roofline, parity or CPU baseline); "
                         "for profiling")
    ap.add_argument("--no-extra", action="store_true",
                    help="skip the other configs' sub-records of the default run")
    args = ap.parse_args()
    cfg = dict(WORKLOADS[args.workload])
    if args.queries:
        cfg["nq"] = args.queries
    if args.rows:
        cfg["n"] = args.rows

    import torch
    import torch.distributed as dist

    world = int(os.environ.get("WORLD_SIZE", "1"))
    rank = int(os.environ.get("RANK", "0"))
    local = int(os.environ.get("LOCAL_RANK", "0"))
    if world > 1:
        import datetime
        torch.cuda.set_device(local)
        dist.init_process_group("nccl", timeout=datetime.timedelta(seconds=300),
                                device_id=torch.device("cuda", local))
    else:
        torch.cuda.set_device(0)
    dev = torch.device("cuda", torch.cuda.current_device())

    if args.impl == "reference":
        if rank == 0:
            line = (encode_reference_line(args, cfg, torch, dev, world)
                    if cfg["mode"] == "encode" else reference_line(args, cfg, torch, dev, world))
            print(json.dumps(line), flush=True)
        if world > 1:
            dist.destroy_process_group()
        return

    if cfg["mode"] == "encode":
        line = encode_sweep(args, cfg, torch, dist, dev, world, rank, args.steps, args.warmup,
                            with_cpu=not args.quick)
    else:
        line = search_workload(args, cfg, torch, dist, dev, world, rank, args.steps, args.warmup,
                               headline=True, with_cpu=not args.quick)
    extra = (world == 1 and not args.quick and not args.no_extra and args.workload == "c4"
             and not args.rows and not args.queries)
    if extra:
        # The other configs, measured after the headline on the same GPU.
        free_device(torch)
        subs = {}
        for name in ("c3", "c2", "c5", "c1"):
            c = dict(WORKLOADS[name])
            t = time.perf_counter()
            if c["mode"] == "encode":
                sub = encode_sweep(args, c, torch, dist, dev, world, rank, steps=5, warmup=3,
                                   with_cpu=True, cpu_rows=20_000)
            else:
                sub = search_workload(args, c, torch, dist, dev, world, rank, steps=10,
                                      warmup=3, headline=False, with_cpu=True)
            sub["wall_s"] = time.perf_counter() - t
            subs[name] = sub
            free_device(torch)
        line["configs"] = subs
        line["encode_sweep"] = {
            "workload": subs["c3"]["config"]["workload"],
            "vectors_per_s": subs["c3"]["value"],
            "per_width": subs["c3"]["per_width"],
            "tensor_frac": subs["c3"]["roofline"]["frac"],
            "peak_kind": subs["c3"]["roofline"]["peak_kind"]}
    if rank == 0:
        print(json.dumps(line), flush=True)
    if world > 1:
        dist.barrier()
        dist.destroy_process_group()


if __name__ == "__main__":
    main()

"""Generate golden fixtures by running the reference ``remex`` package.

Run from the repository root with the reference checked out read-only:

    PYTHONDONTWRITEBYTECODE=1 python tests/golden/make_golden.py <reference checkout>

It imports the reference (pure NumPy/SciPy) and records its outputs on seeded
inputs: parameters (rotation, codebooks, nested tables), encode results,
packed bytes, and the search / twostage / batch / IVF results that the CUDA
library and the CPU oracle are checked against.  Large arrays are stored as
SHA-256 digests.  The RNG known-answer fixtures shipped with the reference's
Mojo tests (1000 f64 normals and 1000 raw u64 draws at seed 42) are copied
into ``rng_seed42.npz`` so the NumPy generator feeding the rotation is pinned.

The fixtures are small and committed; this script only needs to be rerun when
the fixture set changes.  Nothing at test time reads the reference tree.
"""

from __future__ import annotations

import hashlib
import json
import os
import sys

import numpy as np

HERE = os.path.dirname(os.path.abspath(__file__))


def sha(a: np.ndarray) -> str:
    return hashlib.sha256(np.ascontiguousarray(a).tobytes()).hexdigest()


def unit_rows(rng, n, d):
    x = rng.standard_normal((n, d)).astype(np.float32)
    x /= np.linalg.norm(x, axis=1, keepdims=True)
    return x


def main(ref_root: str) -> None:
    sys.dont_write_bytecode = True
    sys.path.insert(0, ref_root)
    import remex
    from remex import Quantizer, IVFCoarseIndex, PackedVectors
    from remex.codebook import lloyd_max_codebook, nested_codebooks
    from remex.rotation import haar_rotation
    from remex.packing import pack

    meta = {"numpy": np.__version__, "remex": getattr(remex, "__version__", "?")}

    # --- RNG known answers from the reference's own fixtures --------------
    fx = os.path.join(ref_root, "remex", "mojo", "tests", "fixtures")
    normals = np.fromfile(os.path.join(fx, "normal_f64_seed42.bin"), dtype="<f8")
    raw = np.fromfile(os.path.join(fx, "raw_u64_seed42.bin"), dtype="<u8")
    np.savez_compressed(os.path.join(HERE, "rng_seed42.npz"), normals=normals, raw=raw)

    # --- parameters --------------------------------------------------------
    params = {}
    for d in (8, 64, 128):
        for seed in (0, 7, 11, 42):
            params[f"R_d{d}_s{seed}"] = haar_rotation(d, seed)
    for d in (8, 64, 128, 256, 384, 768, 1024, 1536):
        for bits in (1, 2, 3, 4, 8):
            b, c = lloyd_max_codebook(d, bits)
            params[f"bounds_d{d}_b{bits}"] = b
            params[f"cent_d{d}_b{bits}"] = c
            nest = nested_codebooks(d, bits)
            for p, t in nest.items():
                params[f"nested_d{d}_b{bits}_p{p}"] = t
    np.savez_compressed(os.path.join(HERE, "params.npz"), **params)
    digests = {}
    for d, seed in ((256, 0), (256, 42), (384, 42), (768, 42), (1024, 42), (1536, 42),
                    (384, 0)):
        digests[f"R_d{d}_s{seed}"] = sha(haar_rotation(d, seed))
    meta["R_sha256"] = digests

    # --- encode ------------------------------------------------------------
    enc = {}
    enc_meta = {}
    for d, n, seed, xseed in ((64, 300, 42, 1), (128, 500, 7, 2), (384, 400, 42, 3),
                              (40, 77, 3, 4)):
        rng = np.random.default_rng(xseed)
        X = (rng.standard_normal((n, d)) * rng.uniform(0.2, 3.0, (n, 1))).astype(np.float32)
        X[0] = 0.0  # zero row: norm 0, divided by the 1e-8 floor
        enc_meta[f"X_d{d}_n{n}_x{xseed}"] = sha(X)
        for bits in (1, 2, 3, 4, 8):
            pq = Quantizer(d=d, bits=bits, seed=seed)
            cv = pq.encode(X)
            key = f"d{d}_n{n}_s{seed}_x{xseed}_b{bits}"
            enc[f"idx_{key}"] = cv.indices
            enc[f"norms_{key}"] = cv.norms
            enc[f"flat_{key}"] = pack(cv.indices.ravel(), bits)
            enc[f"rows_{key}"] = PackedVectors.from_compressed(cv)._packed
    np.savez_compressed(os.path.join(HERE, "encode.npz"), **enc)
    meta["encode_inputs_sha256"] = enc_meta

    # --- search on the reference tests' shapes -----------------------------
    srch = {}
    for bits, seed in ((4, 42), (8, 42), (2, 5), (3, 9), (1, 3)):
        rng = np.random.default_rng(42)
        d, n = 128, 2000
        pq = Quantizer(d=d, bits=bits, seed=seed)
        corpus = unit_rows(rng, n, d)
        qs = unit_rows(rng, 8, d)
        cv = pq.encode(corpus)
        tag = f"b{bits}"
        srch[f"idx_{tag}"] = cv.indices
        srch[f"norms_{tag}"] = cv.norms
        for qi in range(4):
            q = qs[qi]
            for prec in [None] + list(range(1, bits)):
                pn = "full" if prec is None else str(prec)
                i, s = pq.search_adc(cv, q, k=50, precision=prec)
                srch[f"adc_{tag}_q{qi}_p{pn}_i"] = i
                srch[f"adc_{tag}_q{qi}_p{pn}_s"] = s
            i, s = pq.search(cv, q, k=10)
            srch[f"cached_{tag}_q{qi}_i"] = i
            srch[f"cached_{tag}_q{qi}_s"] = s
            cv.drop_cache()
            for C in (200, n):
                i, s = pq.search_twostage(cv, q, k=10, candidates=C)
                srch[f"ts_{tag}_q{qi}_C{C}_i"] = i
                srch[f"ts_{tag}_q{qi}_C{C}_s"] = s
        I, S = pq.search_batch(cv, qs, k=25)
        cv.drop_cache()
        srch[f"batch_{tag}_i"] = I
        srch[f"batch_{tag}_s"] = S
        srch[f"queries_{tag}"] = qs
    np.savez_compressed(os.path.join(HERE, "search.npz"), **srch)

    # --- IVF ---------------------------------------------------------------
    ivf = {}
    rng = np.random.default_rng(42)
    d, n = 128, 2000
    for bits, seed in ((4, 7), (8, 11)):
        pq = Quantizer(d=d, bits=bits, seed=seed)
        rng = np.random.default_rng(42)
        corpus = unit_rows(rng, n, d)
        qs = unit_rows(rng, 6, d)
        cv = pq.encode(corpus)
        for mode, nb in (("lsh", 5), ("rotated_prefix", 4), ("lsh", 8)):
            ix = IVFCoarseIndex(pq, cv, n_bits=nb, mode=mode, seed=0)
            tag = f"b{bits}_{mode}_n{nb}"
            ivf[f"cells_{tag}"] = ix.cell_ids
            ivf[f"sorted_{tag}"] = ix.sorted_idx
            ivf[f"off_{tag}"] = ix.cell_offsets
            if ix.hyperplanes is not None:
                ivf[f"H_{tag}"] = ix.hyperplanes
            for qi in range(3):
                q = qs[qi]
                for npb in (1, 3, ix.n_cells):
                    i, s = ix.search_coarse(q, k=40, nprobe=npb,
                                            precision=max(1, bits - 2))
                    ivf[f"coarse_{tag}_q{qi}_np{npb}_i"] = i
                    ivf[f"coarse_{tag}_q{qi}_np{npb}_s"] = s
                    i, s = ix.search_twostage(q, k=10, candidates=100, nprobe=npb)
                    ivf[f"ts_{tag}_q{qi}_np{npb}_i"] = i
                    ivf[f"ts_{tag}_q{qi}_np{npb}_s"] = s
        ivf[f"queries_b{bits}"] = qs
    np.savez_compressed(os.path.join(HERE, "ivf.npz"), **ivf)

    with open(os.path.join(HERE, "golden_meta.json"), "w") as f:
        json.dump(meta, f, indent=1, sort_keys=True)
    print("wrote fixtures to", HERE)


if __name__ == "__main__":
    if len(sys.argv) != 2:
        sys.exit(f"usage: python {os.path.relpath(__file__)} <path of the reference checkout>")
    main(sys.argv[1])

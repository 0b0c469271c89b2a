"""Generate `.npz` and Arrow IPC golden files by running the reference writers.

Run from the repository root with the reference checked out read-only:

    PYTHONDONTWRITEBYTECODE=1 python tests/golden/make_store_golden.py <reference checkout>

For each width and two shapes (d=13: rows that are not a whole number of
bytes at 1-4 bits; d=16: whole-byte rows) it writes seeded codes and norms
with the reference's CompressedVectors.save, PackedVectors.save and
PackedVectors.save_arrow (seed 42 and one extra metadata pair), and stores
the file bytes, the inputs and the reference's packed rows in
``store_files.npz``.  Nothing at test time reads the reference tree.
"""

from __future__ import annotations

import os
import sys
import tempfile

import numpy as np

HERE = os.path.dirname(os.path.abspath(__file__))


def main(ref_root: str) -> None:
    sys.dont_write_bytecode = True
    sys.path.insert(0, ref_root)
    from remex import CompressedVectors, PackedVectors

    out = {}
    rng = np.random.default_rng(2025)
    with tempfile.TemporaryDirectory() as tmp:
        for bits in (1, 2, 3, 4, 8):
            for d, n in ((13, 7), (16, 5)):
                idx = rng.integers(0, 1 << bits, (n, d)).astype(np.uint8)
                norms = rng.uniform(0.1, 3.0, n).astype(np.float32)
                key = f"b{bits}_d{d}"
                cv = CompressedVectors(idx, norms, d, bits)
                pv = PackedVectors.from_compressed(cv)
                files = {"npz_cv": (cv.save, "cv.npz"), "npz_pv": (pv.save, "pv.npz")}
                for name, (fn, fname) in files.items():
                    p = os.path.join(tmp, fname)
                    fn(p)
                    out[f"{name}_{key}"] = np.frombuffer(open(p, "rb").read(), np.uint8)
                p = os.path.join(tmp, "pv.arrow")
                pv.save_arrow(p, seed=42, partition="shard_0")
                out[f"arrow_{key}"] = np.frombuffer(open(p, "rb").read(), np.uint8)
                out[f"idx_{key}"] = idx
                out[f"norms_{key}"] = norms
                out[f"rows_{key}"] = np.asarray(pv._packed, np.uint8)
    np.savez_compressed(os.path.join(HERE, "store_files.npz"), **out)


if __name__ == "__main__":
    if len(sys.argv) != 2:
        sys.exit(f"usage: python {os.path.relpath(__file__)} <path of the reference checkout>")
    main(sys.argv[1])

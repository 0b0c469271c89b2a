"""Generate the `.pq` / `.params` golden files by running the reference writer.

Run from the repository root with the reference checked out read-only:

    PYTHONDONTWRITEBYTECODE=1 python tests/golden/make_pq_golden.py <reference checkout>

For each width and two shapes (d=13: rows that are not a whole number of
bytes at 1-4 bits; d=16: whole-byte rows) it writes seeded codes and norms
with the reference's save_pq, and the parameters of Quantizer(d, bits, 42)
with its save_params, and stores the file bytes together with the inputs in
``pq_files.npz``.  Nothing at test time reads the reference tree.
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
    from remex import CompressedVectors, Quantizer
    from remex.pq_format import save_params, save_pq

    out = {}
    rng = np.random.default_rng(2024)
    with tempfile.TemporaryDirectory() as tmp:
        for bits in (1, 2, 3, 4, 8):
            for d, n in ((13, 7), (16, 5)):
                idx = rng.integers(0, 1 << bits, (n, d)).astype(np.uint8)
                norms = rng.uniform(0.1, 3.0, n).astype(np.float32)
                p = os.path.join(tmp, "x.pq")
                save_pq(p, CompressedVectors(idx, norms, d, bits))
                key = f"b{bits}_d{d}"
                out[f"pq_{key}"] = np.frombuffer(open(p, "rb").read(), np.uint8)
                out[f"idx_{key}"] = idx
                out[f"norms_{key}"] = norms
            q = Quantizer(d=16, bits=bits, seed=42)
            p = os.path.join(tmp, "x.params")
            save_params(p, q)
            out[f"params_b{bits}_d16"] = np.frombuffer(open(p, "rb").read(), np.uint8)
    np.savez_compressed(os.path.join(HERE, "pq_files.npz"), **out)


if __name__ == "__main__":
    if len(sys.argv) != 2:
        sys.exit(f"usage: python {os.path.relpath(__file__)} <path of the reference checkout>")
    main(sys.argv[1])

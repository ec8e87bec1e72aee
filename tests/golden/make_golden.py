"""Generate tests/golden/qmm_golden.npz.

Run from the repo root:  python tests/golden/make_golden.py

What it holds (all outputs computed by the C oracle, which restates the
reference's Rust CPU path bit for bit and is itself pinned by the reference's
own known-answer tests in tests/test_oracle.py):
  * the reference unit tests' fixtures (rce-op-qmm/src/lib.rs:2267-2616):
    weight bytes, activations, mm_batched output and the dequantised rows;
  * the seeded benchmark-distribution cases (tests/refcases.py SEEDED_CASES):
    sha256 of the generated weight and activation bytes (so a change in the
    generator is detected) and the oracle's output over every row.
The real reference cannot run here (no Rust toolchain), so these vectors are
the oracle's; their role is to pin the GPU path and to catch regressions of
the oracle itself.
"""
from __future__ import annotations

import hashlib
import os
import sys

import numpy as np

HERE = os.path.dirname(os.path.abspath(__file__))
ROOT = os.path.dirname(os.path.dirname(HERE))
sys.path.insert(0, ROOT)
sys.path.insert(0, os.path.join(ROOT, "tests"))

import oracle as O  # noqa: E402
import refcases  # noqa: E402


def sha(a: np.ndarray) -> str:
    return hashlib.sha256(np.ascontiguousarray(a).tobytes()).hexdigest()


def main() -> None:
    out = {}
    for name, build in refcases.REFERENCE_CASES.items():
        w, dt, n, k, x = build()
        t = x.shape[0]
        out[f"{name}__w"] = w
        out[f"{name}__x"] = x
        out[f"{name}__shape"] = np.array([dt, n, k, t], dtype=np.int64)
        out[f"{name}__y"] = O.mm_batched(x, t, w, dt, n, k)
        out[f"{name}__deq"] = O.dequant(w, dt, n * k).reshape(n, k)
    for name, dt, n, k, m, seed in refcases.SEEDED_CASES:
        w, _, _, _, x = refcases.seeded_case(dt, n, k, m, seed)
        out[f"{name}__shape"] = np.array([dt, n, k, m, seed], dtype=np.int64)
        out[f"{name}__wsha"] = np.frombuffer(sha(w).encode(), dtype=np.uint8)
        out[f"{name}__xsha"] = np.frombuffer(sha(x).encode(), dtype=np.uint8)
        out[f"{name}__y"] = O.mm_batched(x, m, w, dt, n, k, nthreads=os.cpu_count() or 1)
    path = os.path.join(HERE, "qmm_golden.npz")
    np.savez_compressed(path, **out)
    print(f"wrote {path} ({os.path.getsize(path)} bytes, {len(out)} arrays)")


if __name__ == "__main__":
    main()

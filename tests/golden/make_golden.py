"""Generates tests/golden/smoke_golden.npz + smoke_golden.json from the
REFERENCE's own host code (kernels/smoke_test.cu generate_weight,
generate_activation, compute_reference), compiled in place into
oracle/_ref/libref_oracle.so by oracle/Makefile.

Run in a container that has the reference checkout:
    make -C oracle ref && python tests/golden/make_golden.py

Stored per case: SHA-256 of the generated weight / weight-scale / activation /
activation-scale bytes (the generators are checked by hash, so the fixture
stays small) and the reference output as bf16 bit patterns.  The shapes are
the reference smoke test's four shapes with their seeds
(kernels/smoke_test.cu:502-507) at M in {1, 8}, plus small shapes covering
ragged N (not a multiple of 128) and every M bucket.
"""

from __future__ import annotations

import hashlib
import json
import os
import sys

import numpy as np

HERE = os.path.dirname(os.path.abspath(__file__))
sys.path.insert(0, os.path.dirname(os.path.dirname(HERE)))

import oracle  # noqa: E402

CASES = [
    # (name, N, K, shape seed, M)
    *[(f"{name}_m{m}", n, k, seed, m) for name, (n, k, seed) in oracle.SMOKE_SHAPES.items() for m in (1, 8)],
    *[(f"small_n200_k384_m{m}", 200, 384, 7, m) for m in (1, 3, 8)],
    *[(f"small_n640_k1024_m{m}", 640, 1024, 11, m) for m in (1, 16, 33, 64, 128)],
]


def sha(a: np.ndarray) -> str:
    return hashlib.sha256(np.ascontiguousarray(a).tobytes()).hexdigest()


def f32_to_bf16_bits(x: np.ndarray) -> np.ndarray:
    bits = np.ascontiguousarray(x, np.float32).view(np.uint32)
    assert np.all((bits & 0xFFFF) == 0), "reference outputs are bf16-rounded"
    return (bits >> 16).astype(np.uint16)


def main() -> None:
    ref = oracle.load_ref()
    if ref is None:
        raise SystemExit("oracle/_ref/libref_oracle.so is missing: run `make -C oracle ref` first")
    manifest = {"source": "reference kernels/smoke_test.cu host code via oracle/ref_shim.cu", "cases": []}
    arrays = {}
    weights = {}
    for name, n, k, seed, m in CASES:
        if (n, k, seed) not in weights:
            weights[(n, k, seed)] = oracle.gen_weight_smoke(n, k, seed, lib=ref)
        w, ws = weights[(n, k, seed)]
        a_seed = oracle.smoke_act_seed(seed, m)
        a, as_ = oracle.gen_activation_smoke(m, k, a_seed, lib=ref)
        out = oracle.compute_reference(a, as_, w, ws, lib=ref)
        arrays[name] = f32_to_bf16_bits(out)
        manifest["cases"].append({
            "name": name, "N": n, "K": k, "M": m, "weight_seed": seed, "act_seed": a_seed,
            "sha_weight": sha(w), "sha_weight_scales": sha(ws),
            "sha_act": sha(a), "sha_act_scales": sha(as_),
        })
        print(name, flush=True)
    np.savez_compressed(os.path.join(HERE, "smoke_golden.npz"), **arrays)
    with open(os.path.join(HERE, "smoke_golden.json"), "w") as f:
        json.dump(manifest, f, indent=1)


if __name__ == "__main__":
    main()

"""Generates the golden vectors in this directory from the reference's OWN code
(oracle/_ref/libridge_ref.so, compiled from the reference sources by
oracle/Makefile). Run where the reference is available:

    python tests/golden/make_golden.py

Writes reference_gemm.json: for the reference harness's six correctness shapes
and seeds (bench/check-gemm.cu:87-94, :266-267), fingerprints of the fills
(bench/check-gemm.cu:139-145) and of the FP64 referenceGemm output
(bench/check-gemm.cu:98-108) -- full-matrix sums plus sampled elements -- and
the checker self-test statistics (bench/check-gemm.cu:201-259) computed by the
reference's errorStats.
"""

import hashlib
import json
import sys
from pathlib import Path

import numpy as np

HERE = Path(__file__).resolve().parent
sys.path.insert(0, str(HERE.parent.parent))

import oracle  # noqa: E402

SHAPES = [(256, 256, 64), (256, 512, 128), (512, 256, 192), (1024, 1024, 64), (1024, 512, 1024),
          (2048, 2048, 2048)]


def sha(a: np.ndarray) -> str:
    return hashlib.sha256(np.ascontiguousarray(a).tobytes()).hexdigest()


def main():
    ref = oracle.Reference()
    rng = np.random.default_rng(12345)
    out = {"source": "reference code via oracle/_ref (check-gemm.cu referenceGemm, "
                     "fillDeterministic, errorStats)", "shapes": []}
    for M, N, K in SHAPES:
        a = ref.fill(M * K, 0x1234 + M)
        b = ref.fill(K * N, 0x9ABC + N)
        c = ref.gemm_f64(a.reshape(M, K), b.reshape(K, N), threads=8)
        idx = [(int(i), int(j)) for i, j in zip(rng.integers(0, M, 48), rng.integers(0, N, 48))]
        idx += [(0, 0), (M - 1, N - 1), (M - 1, 0), (0, N - 1)]
        out["shapes"].append({
            "M": M, "N": N, "K": K, "seed_a": 0x1234 + M, "seed_b": 0x9ABC + N,
            "a_sha256": sha(a), "b_sha256": sha(b), "a_head": a[:16].tolist(),
            "c_sum": float(c.sum()), "c_abs_sum": float(np.abs(c).sum()),
            "c_sq_sum": float((c * c).sum()),
            "samples": [[i, j, float(c[i, j])] for i, j in idx],
        })
    # checker self-test vectors (check-gemm.cu:201-259)
    n = 4096
    s = 0xC0FFEE
    refv = np.empty(n, np.float64)
    for i in range(n):
        s = (s * 1664525 + 1013904223) & 0xFFFFFFFF
        refv[i] = ((s >> 16) & 0x7FFF) / 32767.0 - 0.5
    cases = {}
    cases["exact copy"] = refv.astype(np.float32)
    cases["systematic 5% scale"] = (refv * 1.05).astype(np.float32)
    bad = refv.astype(np.float32).copy()
    bad[int(n * 0.97):] = (refv[int(n * 0.97):] * 0.5).astype(np.float32)
    cases["last 3% of outputs halved"] = bad
    bad = refv.astype(np.float32).copy()
    bad[n // 3] = np.float32(refv[n // 3] + 1.0)
    cases["one element off by a full unit"] = bad
    out["self_test"] = {k: list(ref.error_stats(v, refv)) for k, v in cases.items()}
    (HERE / "reference_gemm.json").write_text(json.dumps(out, indent=1))
    print("wrote", HERE / "reference_gemm.json")


if __name__ == "__main__":
    main()

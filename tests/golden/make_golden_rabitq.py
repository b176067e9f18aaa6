"""Writes tests/golden/rabitq/*.npz: the reference's own RaBitQ quantizer
(rabitq_quantize<1>, run by oracle/_ref/bin/ref_rabitq, built from the
unmodified reference headers by oracle/build_ref.sh) applied to seeded rows.
Run on a GPU machine from the repository root:

    python tests/golden/make_golden_rabitq.py

Each fixture stores the generator and seeds of its inputs (the test
regenerates them and checks their hash) and the reference's node store."""
import hashlib
import subprocess
import sys
import tempfile
from pathlib import Path

import numpy as np

ROOT = Path(__file__).resolve().parents[2]
sys.path.insert(0, str(ROOT))
OUT = Path(__file__).resolve().parent / "rabitq"
DRIVER = ROOT / "oracle" / "_ref" / "bin" / "ref_rabitq"

# name, n, dim, metric, centroid ("mean" | "zero"), rows ("normal" | "relu_sphere"), rotation seed (-1 = identity)
CASES = [
    ("l2_d32_mean", 16, 32, 0, "mean", "normal", -1),
    ("l2_d64_zero", 64, 64, 0, "zero", "normal", -1),
    ("ip_d100_mean", 64, 100, 1, "mean", "normal", -1),   # dim % 4 != 0 faults the reference (misaligned shared memory)
    # the reference's quantizer launches 64 tiles x 5 * dim bytes of dynamic
    # shared memory without raising the 48 KB default, so dim <= 153 only
    ("ip_d152_relu", 256, 152, 1, "mean", "relu_sphere", -1),
    ("l2_d128_rot42", 128, 128, 0, "mean", "normal", 42),
]


def case_inputs(n, dim, centroid, rows, seed):
    rng = np.random.default_rng(seed)
    if rows == "normal":
        X = rng.standard_normal((n, dim)).astype(np.float32)
    else:
        C = rng.standard_normal((8, dim)).astype(np.float32)
        X = C[rng.integers(0, 8, n)] + 0.3 * rng.standard_normal((n, dim)).astype(np.float32)
        X = np.maximum(X, 0)
        X /= np.maximum(np.linalg.norm(X, axis=1, keepdims=True), 1e-12)
        X = X.astype(np.float32)
    c = X.mean(0).astype(np.float32) if centroid == "mean" else np.zeros(dim, np.float32)
    return X, c


def rotation(dim, seed):
    from jasper_b200 import _lib
    P = np.zeros(dim * dim, np.float32)
    _lib.call("jb_rotation_matrix", dim, seed, P.ctypes.data)
    return P


def main():
    OUT.mkdir(exist_ok=True)
    for i, (name, n, dim, metric, centroid, rows, rot) in enumerate(CASES):
        seed = 700 + i
        X, c = case_inputs(n, dim, centroid, rows, seed)
        with tempfile.TemporaryDirectory() as td:
            fin, fout = Path(td) / "in.bin", Path(td) / "out.bin"
            with open(fin, "wb") as f:
                f.write(np.array([n, dim, metric, 1 if rot >= 0 else 0], np.uint32).tobytes())
                f.write(X.tobytes())
                f.write(c.tobytes())
                if rot >= 0:
                    f.write(rotation(dim, rot).tobytes())
            subprocess.run([str(DRIVER), str(fin), str(fout)], check=True)
            store = np.fromfile(fout, np.uint8)
        np.savez_compressed(OUT / f"{name}.npz", n=n, dim=dim, metric=metric, centroid=centroid,
                            rows=rows, seed=seed, rotation_seed=rot,
                            x_sha=hashlib.sha256(X.tobytes()).hexdigest(), store=store)
        print(name, store.size, "bytes")


if __name__ == "__main__":
    main()

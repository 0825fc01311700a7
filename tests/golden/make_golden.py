"""Generate the committed golden digests from the reference's own CPU implementation.

    make -C oracle && python tests/golden/make_golden.py [tiny] [short] [full]

For each model configuration (demucs_cuda_b200.synth: seeded random-init weights with
layer_scale 0.3 so every residual branch shows in the output; input = config 0's
U[-0.5, 0.5] segment, seed 0) this runs oracle/_ref (backend_cpu.c + the reference's model
code, unmodified) with per-stage dumps and writes <name>_digest.json: for every stage of
test_compare.c's list its shape, float64 sum and sum of squares, and 512 evenly strided
samples.  The reference itself cannot run on the GPU box's tests at full size in seconds,
so these digests pin both the numpy port (tests/test_oracle.py) and the GPU engine
(tests/test_gpu_model.py) to the reference's actual outputs.
"""
import json
import os
import sys
import time

import numpy as np

HERE = os.path.dirname(os.path.abspath(__file__))
ROOT = os.path.dirname(os.path.dirname(HERE))
sys.path.insert(0, ROOT)

from demucs_cuda_b200 import synth  # noqa: E402
from oracle import ref  # noqa: E402

NSAMP = 512
CFGS = {"tiny": synth.TINY, "short": synth.SHORT, "full": synth.FULL}


def digest(a: np.ndarray) -> dict:
    a = np.ascontiguousarray(a, dtype=np.float32)
    flat = a.ravel()
    idx = np.linspace(0, flat.size - 1, min(NSAMP, flat.size)).astype(np.int64)
    return {"shape": list(a.shape), "sum": float(flat.astype(np.float64).sum()),
            "sumsq": float((flat.astype(np.float64) ** 2).sum()),
            "idx_count": int(idx.size), "samples": [float(v) for v in flat[idx]]}


def sample_index(n: int) -> np.ndarray:
    return np.linspace(0, n - 1, min(NSAMP, n)).astype(np.int64)


def make(name: str, cache: str):
    cfg = CFGS[name]
    w, c = synth.write_model(os.path.join(cache, f"{name}_s1_ls0.3"), cfg, seed=1,
                             layer_scale=0.3)
    ref.load(w, c)
    mix = synth.segment_input(cfg, 1, 0)
    t0 = time.time()
    stems, st = ref.forward(mix, stages=True)
    dt = time.time() - t0
    out = {"config": name, "weights_seed": 1, "layer_scale": 0.3, "input_seed": 0,
           "reference_seconds": dt, "stages": {k: digest(v) for k, v in st.items()}}
    path = os.path.join(HERE, f"{name}_digest.json")
    with open(path, "w") as f:
        json.dump(out, f)
    print(f"{name}: reference forward {dt:.1f}s -> {path}")


if __name__ == "__main__":
    names = sys.argv[1:] or ["tiny", "short", "full"]
    cache = os.environ.get("DCB_TEST_CACHE", "/tmp/demucs_b200_test_models")
    for n in names:
        make(n, cache)

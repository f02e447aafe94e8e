"""Generate the config-scale parity fixtures (tests/golden/config_<case>.npz).

The CPU oracle needs minutes per chunk at the benchmark configurations (a
dim-512 depth-12 chunk is ~19 TFLOP of fp64-accumulated arithmetic), which is
too slow to repeat inside every GPU test run.  This script runs it once, here,
on seeded inputs that the GPU tests rebuild bit-exactly:

* weights: `csm_tool.make_random_csm(path, preset, seed)` (numpy PCG64 stream);
* audio: `csm_tool.pink_noise` / `csm_tool.uniform_noise16` quantised to
  16-bit levels, so tiny FFT rounding differences between hosts vanish.

Each fixture keeps the SHA-256 of the .csm bytes and of the input samples (the
test checks both before it compares), the full output shape, and every
`stride`-th sample of the oracle's flattened output (about 131 072 samples: an
SNR over that many samples is within ~0.01 dB of the SNR over all of them).

Cases (BASELINE configurations, one chunk batch each):
  std       fp16 weights, dim 384, depth 6, 8x64, one 8 s chunk (T = 801)
  large     fp16 weights, dim 512, depth 12, 16x64, 2 stems, one 11 s chunk (T = 1101)
  two_stem  bf16 weights, dim 384, depth 12, 2 stems, chunk-batch 4 (four 8 s
            chunks); also the oracle's reference-bf16 mode (weight_dtype 4),
            which rounds activations where the reference's bf16 path stores them

Usage:  python tests/golden/make_config_golden.py [case ...]   (default: all)
"""
from __future__ import annotations

import hashlib
import os
import sys
import tempfile
import time

import numpy as np

HERE = os.path.dirname(os.path.abspath(__file__))
ROOT = os.path.dirname(os.path.dirname(HERE))
for p in (os.path.join(ROOT, "mbr-cuda-tile_b200"), os.path.join(ROOT, "oracle")):
    if p not in sys.path:
        sys.path.insert(0, p)

SR = 44100
TARGET_SAMPLES = 131072

CASES = {
    "std": dict(preset="std", seed=101, wdt=1, dtype="fp16", seconds=8.0, audio_seeds=[201]),
    "large": dict(preset="large", seed=102, wdt=1, dtype="fp16", seconds=11.0, audio_seeds=[202]),
    "two_stem": dict(preset="two_stem", seed=103, wdt=3, dtype="bf16", seconds=8.0,
                     audio_seeds=[203, 204, 205, 206], ref_bf16_wdt=4),
}


def case_audio(case: dict) -> np.ndarray:
    import csm_tool

    return np.stack([csm_tool.pink_noise(case["seconds"], s, 2, SR) for s in case["audio_seeds"]])


def sha256_file(path: str) -> str:
    h = hashlib.sha256()
    with open(path, "rb") as f:
        for blk in iter(lambda: f.read(1 << 20), b""):
            h.update(blk)
    return h.hexdigest()


def sha256_array(a: np.ndarray) -> str:
    return hashlib.sha256(np.ascontiguousarray(a).tobytes()).hexdigest()


def fixture_path(name: str) -> str:
    return os.path.join(HERE, f"config_{name}.npz")


def subsample(ref: np.ndarray, stride: int) -> np.ndarray:
    return np.ascontiguousarray(ref.reshape(-1)[::stride], np.float32)


def make(name: str) -> None:
    import csm_tool
    import oracle

    case = CASES[name]
    with tempfile.TemporaryDirectory() as d:
        path = os.path.join(d, f"{name}.csm")
        csm_tool.make_random_csm(path, case["preset"], case["seed"])
        x = case_audio(case)
        out = dict(case=name, preset=case["preset"], seed=case["seed"], wdt=case["wdt"],
                   audio_seeds=np.array(case["audio_seeds"]), csm_sha=sha256_file(path),
                   input_sha=sha256_array(x))
        t0 = time.time()
        ref = oracle.Model(path, case["wdt"]).forward(x)
        stride = max(1, ref.size // TARGET_SAMPLES)
        out.update(shape=np.array(ref.shape), stride=stride, ref=subsample(ref, stride),
                   ref_energy=float(np.sum(ref.astype(np.float64) ** 2)))
        print(f"{name}: oracle forward {ref.shape} in {time.time() - t0:.0f} s "
              f"({oracle.threads()} threads)", flush=True)
        if "ref_bf16_wdt" in case:
            t0 = time.time()
            rb = oracle.Model(path, case["ref_bf16_wdt"]).forward(x)
            out.update(ref_bf16=subsample(rb, stride))
            diff = np.sum((rb.astype(np.float64) - ref) ** 2)
            print(f"{name}: reference-bf16 oracle in {time.time() - t0:.0f} s, "
                  f"SNR vs the fp32 oracle {10 * np.log10(out['ref_energy'] / diff):.2f} dB", flush=True)
        np.savez_compressed(fixture_path(name), **out)


def main(argv):
    names = argv or list(CASES)
    for n in names:
        if n not in CASES:
            raise SystemExit(f"unknown case {n}; choose from {sorted(CASES)}")
    for n in names:
        make(n)


if __name__ == "__main__":
    main(sys.argv[1:])

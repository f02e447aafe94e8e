"""Generates the committed golden fixtures of tests/golden/.

Run from the repository root:  python tests/golden/make_golden.py

 - band_map.npz: freq_indices / num_freqs_per_band / num_bands_per_freq of the
   60-band slaney mel split (sr 44100, n_fft 2048, stereo) from csm_tool.
   Their distinct 8*nf values are checked against the reference's hard-coded
   mask-estimator width whitelist (src/mbr_cuda_tile.cu:2289-2311) in the tests.
 - stft.npz: a seeded signal and torch.stft / torch.istft of it with the
   reference's STFT settings (n_fft 2048, hop 441, periodic Hann, center,
   reflect pad, onesided, unnormalised; src/stft_cuda_tile.cu:530-715), in fp64.
 - chunk_plans.json: chunk starts / border / padded length of the reference
   chunk driver (src/inference_app.cpp:46-89) for a set of track lengths,
   from an independent Python restatement in this file.
"""
import json
import math
import os
import sys

import numpy as np

HERE = os.path.dirname(os.path.abspath(__file__))
ROOT = os.path.dirname(os.path.dirname(HERE))
sys.path.insert(0, os.path.join(ROOT, "mbr-cuda-tile_b200"))


def resolve_step(chunk, overlap, default):
    # src/inference_app.cpp:46-57; std::lround rounds half away from zero
    if 0.0 < overlap < 1.0:
        v = chunk * np.float32(1.0 - np.float32(overlap))
        step = int(math.floor(abs(v) + 0.5)) * (1 if v >= 0 else -1)
        return max(1, step)
    n = default
    if overlap >= 1.0:
        n = max(1, int(math.floor(overlap + 0.5)))
    return max(1, chunk // max(1, n))


def chunk_plan(N, chunk, overlap, default):
    step = resolve_step(chunk, overlap, default)
    border = chunk - step
    padded = N > 2 * border and border > 0
    total = N + 2 * border if padded else N
    return dict(N=N, chunk=chunk, overlap=overlap, default=default, step=step,
                border=border if padded else 0, total=total, starts=list(range(0, total, step)))


def main():
    import csm_tool
    import torch

    fi, nfpb, nbpf = csm_tool.mel_band_map(44100, 2048, 60, True)
    np.savez(os.path.join(HERE, "band_map.npz"), freq_indices=fi, num_freqs_per_band=nfpb, num_bands_per_freq=nbpf)

    rng = np.random.default_rng(1234)
    x = rng.uniform(-0.5, 0.5, (2, 6000)).astype(np.float32)
    w = torch.hann_window(2048, periodic=True, dtype=torch.float64)
    S = torch.stft(torch.from_numpy(x).double(), 2048, 441, 2048, w, center=True, pad_mode="reflect",
                   normalized=False, onesided=True, return_complex=True)
    y = torch.istft(S, 2048, 441, 2048, w, center=True)
    np.savez(os.path.join(HERE, "stft.npz"), x=x, spec=torch.view_as_real(S).numpy().astype(np.float32),
             y=y.numpy().astype(np.float32))

    cases = []
    for N, chunk, ov, d in [(1323000, 352800, -1.0, 4), (1323000, 352800, 4.0, 1), (100000, 44100, 0.5, 2),
                            (44100 * 3 + 1234, 44100, -1.0, 2), (44100 * 3 + 1234, 44100, 4.0, 2),
                            (44100 * 3 + 1234, 44100, 0.5, 2), (60000, 44100, -1.0, 2), (352800, 352800, -1.0, 4),
                            (7938000, 352800, 4.0, 4), (26460000, 485100, 2.0, 2), (88200, 44100, 0.25, 1)]:
        cases.append(chunk_plan(N, chunk, ov, d))
    with open(os.path.join(HERE, "chunk_plans.json"), "w") as f:
        json.dump(cases, f)
    print("wrote", os.listdir(HERE))


if __name__ == "__main__":
    main()

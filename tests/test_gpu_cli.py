"""End-to-end check of the cudasep_infer CLI (reference flags): 16-bit WAV in,
float32 stem WAVs out, compared with the CPU oracle's chunked separation."""
import os
import subprocess
import wave

import numpy as np
import pytest

from metrics import rel_max_err

pytestmark = pytest.mark.gpu
ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
CLI = os.path.join(ROOT, "mbr-cuda-tile_b200", "cudasep_infer")


def test_cli_separates_wav_like_the_oracle(tmp_path, make_csm):
    import torch

    if not torch.cuda.is_available():
        pytest.skip("no CUDA device")
    import oracle
    from test_wav import _read

    path = make_csm("tiny2", seed=41)  # 2 stems
    rng = np.random.default_rng(5)
    pcm = rng.integers(-12000, 12000, size=(3 * 44100 + 99, 2), dtype=np.int16)
    wav = tmp_path / "in.wav"
    with wave.open(str(wav), "wb") as w:
        w.setnchannels(2)
        w.setsampwidth(2)
        w.setframerate(44100)
        w.writeframes(pcm.tobytes())
    out = tmp_path / "out"
    r = subprocess.run([CLI, "--model", path, "--input", str(wav), "--output", str(out), "--stem", "-1", "--fp32",
                        "--overlap", "2"], capture_output=True, text=True, timeout=600)
    assert r.returncode == 0, r.stdout + r.stderr
    assert "RTF" in r.stdout
    track = (pcm.T.astype(np.float32) / 32768.0).astype(np.float32)
    ref = oracle.Model(path).separate(track, 2.0, 1)
    for s, name in enumerate(["vocals", "instrumental"]):
        sr, y = _read(out / f"{name}.wav")
        assert sr == 44100 and y.shape == track.shape
        assert rel_max_err(ref[s], y) <= 1e-4
    bad = subprocess.run([CLI, "--model", path], capture_output=True, text=True)
    assert bad.returncode == 1 and "--input is required" in bad.stderr

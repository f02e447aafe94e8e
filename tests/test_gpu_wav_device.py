"""GPU WAV path (PCM -> planar fp32 conversion on the device, and the device
interleave of the float WAV writer) against the host reader and writer: the
converted samples must be bit-identical (src/audio_io.cpp:200-334 scales
integer PCM by 1/2^(bits-1) on the host; the kernels do the same arithmetic)."""
import struct
import wave

import numpy as np
import pytest

pytestmark = pytest.mark.gpu


@pytest.fixture(scope="module")
def torch_cuda():
    import torch

    if not torch.cuda.is_available():
        pytest.skip("no CUDA device")
    return torch


def _host_read(path):
    import ctypes

    import cudasep

    L = cudasep.lib()
    sr, ch, n = ctypes.c_int(), ctypes.c_int(), ctypes.c_int64()
    assert L.mbr_wav_info(str(path).encode(), ctypes.byref(sr), ctypes.byref(ch), ctypes.byref(n)) == 0
    out = np.empty((ch.value, n.value), np.float32)
    assert L.mbr_wav_read(str(path).encode(), out.ctypes.data, out.size) == 0
    return out, sr.value


@pytest.mark.parametrize("width,channels", [(2, 2), (3, 2), (4, 1), (2, 3)])
def test_device_pcm_matches_host_reader(torch_cuda, tmp_path, width, channels):
    import cudasep

    bits = 8 * width
    x = np.random.default_rng(bits + channels).integers(-(1 << (bits - 1)), 1 << (bits - 1),
                                                         size=(4099, channels), dtype=np.int64)
    p = tmp_path / f"pcm{bits}_{channels}.wav"
    with wave.open(str(p), "wb") as w:
        w.setnchannels(channels)
        w.setsampwidth(width)
        w.setframerate(44100)
        w.writeframes(b"".join(int(v).to_bytes(width, "little", signed=True) for v in x.reshape(-1)))
    host, sr_h = _host_read(p)
    dev, sr_d = cudasep.wav_read_device(str(p))
    torch_cuda.cuda.synchronize()
    assert sr_h == sr_d == 44100 and tuple(dev.shape) == host.shape
    assert np.array_equal(dev.cpu().numpy(), host)


def test_device_float_wav_and_writer(torch_cuda, tmp_path):
    import cudasep

    torch = torch_cuda
    x = np.random.default_rng(5).uniform(-1, 1, (2, 12345)).astype(np.float32)
    # a float WAV with an extra chunk ahead of "data" (odd-sized, padded)
    inter = x.T.reshape(-1).tobytes()
    fmt = struct.pack("<HHIIHH", 3, 2, 48000, 48000 * 8, 8, 32)
    body = b"WAVE" + b"fmt " + struct.pack("<I", 16) + fmt + b"LIST" + struct.pack("<I", 3) + b"abc\x00" + \
        b"data" + struct.pack("<I", len(inter)) + inter
    p = tmp_path / "f.wav"
    p.write_bytes(b"RIFF" + struct.pack("<I", len(body)) + body)
    dev, sr = cudasep.wav_read_device(str(p))
    assert sr == 48000 and np.array_equal(dev.cpu().numpy(), x)
    # device interleave + write, read back on the host
    q = tmp_path / "g.wav"
    cudasep.wav_write_device(str(q), torch.from_numpy(x).cuda(), 48000)
    back, sr2 = _host_read(q)
    assert sr2 == 48000 and np.array_equal(back, x)


def test_pcm_to_planar_on_device_bytes(torch_cuda):
    """Raw interleaved 16-bit PCM already on the device."""
    import cudasep

    torch = torch_cuda
    x = np.random.default_rng(9).integers(-32768, 32768, size=(777, 2), dtype=np.int16)
    d_pcm = torch.from_numpy(x.reshape(-1).view(np.uint8).copy()).cuda()
    out = torch.empty((2, 777), dtype=torch.float32, device="cuda")
    cudasep.pcm_to_planar(d_pcm, 777, 2, 16, False, out)
    assert np.array_equal(out.cpu().numpy(), (x.T.astype(np.float32) / np.float32(32768)))

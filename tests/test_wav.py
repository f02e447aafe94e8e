"""WAV I/O of the C ABI (host only): PCM 16/24/32-bit and float32 input with the
reference's scaling (src/audio_io.cpp:200-255), float32 output."""
import ctypes
import struct
import wave

import numpy as np
import pytest


def _lib():
    import cudasep

    L = cudasep.lib()
    L.mbr_wav_info.argtypes = [ctypes.c_char_p, ctypes.POINTER(ctypes.c_int), ctypes.POINTER(ctypes.c_int),
                               ctypes.POINTER(ctypes.c_int64)]
    L.mbr_wav_read.argtypes = [ctypes.c_char_p, ctypes.c_void_p, ctypes.c_int64]
    L.mbr_wav_write.argtypes = [ctypes.c_char_p, ctypes.c_void_p, ctypes.c_int, ctypes.c_int64, ctypes.c_int]
    return L


def _read(path):
    L = _lib()
    sr, ch, n = ctypes.c_int(), ctypes.c_int(), ctypes.c_int64()
    assert L.mbr_wav_info(str(path).encode(), ctypes.byref(sr), ctypes.byref(ch), ctypes.byref(n)) == 0
    out = np.empty((ch.value, n.value), np.float32)
    assert L.mbr_wav_read(str(path).encode(), out.ctypes.data, out.size) == 0
    return sr.value, out


@pytest.mark.parametrize("width", [2, 3, 4])
def test_pcm_scaling(tmp_path, width):
    rng = np.random.default_rng(width)
    bits = 8 * width
    x = rng.integers(-(1 << (bits - 1)), 1 << (bits - 1), size=(1000, 2), dtype=np.int64)
    raw = b"".join(int(v).to_bytes(width, "little", signed=True) for v in x.reshape(-1))
    p = tmp_path / "a.wav"
    with wave.open(str(p), "wb") as w:
        w.setnchannels(2)
        w.setsampwidth(width)
        w.setframerate(44100)
        w.writeframes(raw)
    sr, y = _read(p)
    assert sr == 44100 and y.shape == (2, 1000)
    assert np.array_equal(y, (x.T.astype(np.float32) / np.float32(1 << (bits - 1))).astype(np.float32))


def test_float_write_read_roundtrip(tmp_path):
    L = _lib()
    x = np.random.default_rng(0).uniform(-1, 1, (2, 777)).astype(np.float32)
    p = tmp_path / "f.wav"
    assert L.mbr_wav_write(str(p).encode(), x.ctypes.data, 2, 777, 48000) == 0
    sr, y = _read(p)
    assert sr == 48000 and np.array_equal(x, y)
    # also a float WAV written by hand with an extra chunk before "data"
    inter = x.T.reshape(-1).tobytes()
    fmt = struct.pack("<HHIIHH", 3, 2, 22050, 22050 * 8, 8, 32)
    body = b"WAVE" + b"fmt " + struct.pack("<I", 16) + fmt + b"LIST" + struct.pack("<I", 3) + b"abc\x00" + \
        b"data" + struct.pack("<I", len(inter)) + inter
    q = tmp_path / "g.wav"
    q.write_bytes(b"RIFF" + struct.pack("<I", len(body)) + body)
    sr, y = _read(q)
    assert sr == 22050 and np.array_equal(x, y)


def test_bad_files_report_errors(tmp_path):
    L = _lib()
    p = tmp_path / "bad.wav"
    p.write_bytes(b"RIFX0000WAVE")
    sr, ch, n = ctypes.c_int(), ctypes.c_int(), ctypes.c_int64()
    assert L.mbr_wav_info(str(p).encode(), ctypes.byref(sr), ctypes.byref(ch), ctypes.byref(n)) != 0
    assert b"RIFF" in L.mbr_last_error()
    assert L.mbr_wav_info(b"/nonexistent.wav", ctypes.byref(sr), ctypes.byref(ch), ctypes.byref(n)) != 0

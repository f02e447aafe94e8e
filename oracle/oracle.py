"""ctypes binding of the CPU oracle (oracle/_build/libmbr_oracle.so).

TEST INFRASTRUCTURE ONLY: used by tests/, __graft_entry__.smoke() and the
cpu_baseline leg of bench.py as the checker.  The product never imports it.
"""
from __future__ import annotations

import ctypes
import os
import subprocess

import numpy as np

HERE = os.path.dirname(os.path.abspath(__file__))
LIB_PATH = os.path.join(HERE, "_build", "libmbr_oracle.so")

_lib = None


def build() -> str:
    subprocess.run(["make", "-s", "-C", HERE], check=True)
    return LIB_PATH


def lib():
    global _lib
    if _lib is None:
        if not os.path.exists(LIB_PATH):
            build()
        L = ctypes.CDLL(LIB_PATH)
        i64p = ctypes.POINTER(ctypes.c_int64)
        fp = ctypes.POINTER(ctypes.c_float)
        L.orc_last_error.restype = ctypes.c_char_p
        L.orc_band_map.argtypes = [ctypes.c_int, ctypes.c_int, ctypes.c_int, ctypes.c_int, i64p, ctypes.c_int64,
                                   i64p, i64p, i64p]
        L.orc_stft.argtypes = [fp, ctypes.c_int64, ctypes.c_int64, ctypes.c_int, ctypes.c_int, fp, i64p]
        L.orc_istft.argtypes = [fp, ctypes.c_int64, ctypes.c_int64, ctypes.c_int, ctypes.c_int, ctypes.c_int64, fp,
                                i64p]
        L.orc_model_load.restype = ctypes.c_void_p
        L.orc_model_load.argtypes = [ctypes.c_char_p, ctypes.c_int]
        L.orc_model_free.argtypes = [ctypes.c_void_p]
        L.orc_model_info.restype = ctypes.c_int64
        L.orc_model_info.argtypes = [ctypes.c_void_p, ctypes.c_int]
        L.orc_forward.argtypes = [ctypes.c_void_p, fp, ctypes.c_int, ctypes.c_int64, fp, i64p]
        L.orc_forward_tap.argtypes = [ctypes.c_void_p, fp, ctypes.c_int, ctypes.c_int64, ctypes.c_int, fp, i64p]
        L.orc_separate.argtypes = [ctypes.c_void_p, fp, ctypes.c_int64, ctypes.c_float, ctypes.c_int, fp]
        L.orc_chunk_plan.restype = ctypes.c_int64
        L.orc_chunk_plan.argtypes = [ctypes.c_int64, ctypes.c_int, ctypes.c_float, ctypes.c_int, i64p,
                                     ctypes.c_int64, i64p, i64p, i64p]
        L.orc_set_threads.argtypes = [ctypes.c_int]
        L.orc_attention.argtypes = [fp, fp, fp, ctypes.c_int64, ctypes.c_int64, ctypes.c_int, ctypes.c_float, fp]
        L.orc_get_threads.restype = ctypes.c_int
        _lib = L
    return _lib


def _fp(a):
    return a.ctypes.data_as(ctypes.POINTER(ctypes.c_float))


def _ip(a):
    return a.ctypes.data_as(ctypes.POINTER(ctypes.c_int64))


def _check(rc):
    if rc != 0:
        raise RuntimeError("oracle: " + lib().orc_last_error().decode())


def set_threads(n: int) -> None:
    lib().orc_set_threads(int(n))


def threads() -> int:
    return lib().orc_get_threads()


def band_map(sr=44100, n_fft=2048, num_bands=60, stereo=True):
    nf = n_fft // 2 + 1
    cap = 2 * nf * num_bands
    fi = np.zeros(cap, np.int64)
    n = np.zeros(1, np.int64)
    nfpb = np.zeros(num_bands, np.int64)
    nbpf = np.zeros(nf, np.int64)
    _check(lib().orc_band_map(sr, n_fft, num_bands, int(stereo), _ip(fi), cap, _ip(n), _ip(nfpb), _ip(nbpf)))
    return fi[: int(n[0])].copy(), nfpb, nbpf


def stft(sig: np.ndarray, n_fft=2048, hop=441) -> np.ndarray:
    sig = np.ascontiguousarray(sig, np.float32)
    lead, L = sig.shape[:-1], sig.shape[-1]
    n = int(np.prod(lead)) if lead else 1
    T = np.zeros(1, np.int64)
    _check(lib().orc_stft(_fp(sig), n, L, n_fft, hop, None, _ip(T)))
    out = np.zeros((n, n_fft // 2 + 1, int(T[0]), 2), np.float32)
    _check(lib().orc_stft(_fp(sig), n, L, n_fft, hop, _fp(out), _ip(T)))
    return out.reshape(*lead, n_fft // 2 + 1, int(T[0]), 2)


def istft(spec: np.ndarray, n_fft=2048, hop=441, length=-1) -> np.ndarray:
    spec = np.ascontiguousarray(spec, np.float32)
    lead = spec.shape[:-3]
    T = spec.shape[-2]
    n = int(np.prod(lead)) if lead else 1
    lo = np.zeros(1, np.int64)
    _check(lib().orc_istft(_fp(spec), n, T, n_fft, hop, length, None, _ip(lo)))
    out = np.zeros((n, int(lo[0])), np.float32)
    _check(lib().orc_istft(_fp(spec), n, T, n_fft, hop, length, _fp(out), _ip(lo)))
    return out.reshape(*lead, int(lo[0]))


def attention(q: np.ndarray, k: np.ndarray, v: np.ndarray, scale: float) -> np.ndarray:
    """softmax(q k^T * scale) v over [..., L, dh] slices (fp64 sums)."""
    q, k, v = (np.ascontiguousarray(a, np.float32) for a in (q, k, v))
    L, dh = q.shape[-2:]
    nsh = int(np.prod(q.shape[:-2])) if q.ndim > 2 else 1
    out = np.empty_like(q)
    _check(lib().orc_attention(_fp(q), _fp(k), _fp(v), nsh, L, dh, scale, _fp(out)))
    return out


def chunk_plan(N, chunk_size, overlap, default_overlap):
    step, border, total = (np.zeros(1, np.int64) for _ in range(3))
    n = lib().orc_chunk_plan(N, chunk_size, overlap, default_overlap, None, 0, _ip(step), _ip(border), _ip(total))
    starts = np.zeros(max(n, 1), np.int64)
    lib().orc_chunk_plan(N, chunk_size, overlap, default_overlap, _ip(starts), n, _ip(step), _ip(border),
                         _ip(total))
    return starts[:n], int(step[0]), int(border[0]), int(total[0])


class Model:
    """Oracle model loaded from a .csm file.  weight_dtype 0 keeps the stored
    weights, 1/3 round 2-D fp32 tensors to fp16/bf16 like the reference's
    --fp16/--bf16 load path."""

    INFO = dict(dim=0, depth=1, num_stems=2, channels=3, num_bands=4, sample_rate=5, chunk_size=6,
                num_overlap=7, n_fft=8, hop=9, heads=10, dim_head=11, band_freqs=12, zero_dc=13,
                match_input_audio_length=14)

    def __init__(self, path: str, weight_dtype: int = 0):
        self.h = lib().orc_model_load(path.encode(), weight_dtype)
        if not self.h:
            raise RuntimeError("oracle: " + lib().orc_last_error().decode())

    def __del__(self):
        if getattr(self, "h", None):
            lib().orc_model_free(self.h)
            self.h = None

    def info(self, key: str) -> int:
        return int(lib().orc_model_info(self.h, self.INFO[key]))

    def forward(self, audio: np.ndarray) -> np.ndarray:
        audio = np.ascontiguousarray(audio, np.float32)
        B, C, L = audio.shape
        S = self.info("num_stems")
        out = np.zeros((B, S, C, L), np.float32)
        lo = np.zeros(1, np.int64)
        _check(lib().orc_forward(self.h, _fp(audio), B, L, _fp(out), _ip(lo)))
        lo = int(lo[0])
        return out.reshape(-1)[: B * S * C * lo].reshape(B, S, C, lo)

    def tap(self, audio: np.ndarray, tap: int) -> np.ndarray:
        audio = np.ascontiguousarray(audio, np.float32)
        B, C, L = audio.shape
        n = np.zeros(1, np.int64)
        _check(lib().orc_forward_tap(self.h, _fp(audio), B, L, tap, None, _ip(n)))
        buf = np.zeros(int(n[0]), np.float32)
        _check(lib().orc_forward_tap(self.h, _fp(audio), B, L, tap, _fp(buf), _ip(n)))
        return buf

    def separate(self, track: np.ndarray, overlap: float = -1.0, chunk_batch: int = 1) -> np.ndarray:
        track = np.ascontiguousarray(track, np.float32)
        C, N = track.shape
        S = self.info("num_stems")
        out = np.zeros((S, C, N), np.float32)
        _check(lib().orc_separate(self.h, _fp(track), N, overlap, chunk_batch, _fp(out)))
        return out

"""cudasep — Python binding of libmbr_b200.so (include/mbr_b200.h) over ctypes.

Mirrors the reference's C++ entry points (cudasep::app::load_model /
run_inference, MelBandRoformer::forward) for Python callers, tests and the
benchmark.  torch is used only to hold device memory and streams; every
computation runs in the library's CUDA kernels.  There is no fallback: if the
shared library is missing or a call fails, an exception is raised.
"""
from __future__ import annotations

import ctypes
import os

import numpy as np

HERE = os.path.dirname(os.path.abspath(__file__))
LIB_PATH = os.path.join(HERE, "libmbr_b200.so")

FP32, FP16, BF16 = 0, 1, 3
DTYPES = {"fp32": FP32, "float32": FP32, "fp16": FP16, "float16": FP16, "bf16": BF16, "bfloat16": BF16}
BACKEND_SIMT, BACKEND_TC, BACKEND_TC_DIRECT = 0, 1, 2

INFO = dict(dim=0, depth=1, num_stems=2, channels=3, num_bands=4, sample_rate=5, chunk_size=6, num_overlap=7,
            heads=8, dim_head=9, band_freqs=10, dtype=11, device=12, hop=13)

# Every symbol include/mbr_b200.h declares (checked by the ABI test).
EXPORTS = [
    "mbr_last_error", "mbr_version", "mbr_create", "mbr_destroy", "mbr_get_info", "mbr_output_length",
    "mbr_forward_chunk", "mbr_forward_tap", "mbr_separate_device", "mbr_separate", "mbr_shard_info",
    "mbr_shard_run", "mbr_shard_window", "mbr_plan_shard_window", "mbr_shard_run_window", "mbr_shard_add_boundary", "mbr_shard_finalize", "mbr_set_graphs", "mbr_set_backend", "mbr_last_launches",
    "mbr_sync_check", "mbr_profile_enable", "mbr_profile_read",
    "mbr_op_rms_norm", "mbr_op_add", "mbr_op_gelu", "mbr_op_sigmoid_gate", "mbr_op_rope", "mbr_op_attention", "mbr_op_linear", "mbr_op_ffn",
    "mbr_rope_tables",
    "mbr_op_band_gather", "mbr_op_mask_scatter", "mbr_op_stft", "mbr_op_istft", "mbr_op_istft_noalloc",
    "mbr_plan_shard", "mbr_wav_info", "mbr_wav_read", "mbr_wav_write",
    "mbr_pcm_to_planar", "mbr_wav_read_device", "mbr_wav_write_device",
]

# Kernel classes of mbr_profile_read.
PROFILE_KINDS = ["stft", "band_gather", "gemm_bandsplit", "norm", "gemm_qkv", "rope", "attn_time", "attn_freq",
                 "gemm_out", "gemm_ffn1", "gemm_ffn2", "gemm_mask_hidden", "gemm_mask_out", "mask_scatter", "istft",
                 "ffn"]

_lib = None


class MBRError(RuntimeError):
    def __init__(self, code: int, msg: str):
        super().__init__(f"[{code}] {msg}")
        self.code = code


def lib():
    """Load libmbr_b200.so (raises if it has not been built)."""
    global _lib
    if _lib is None:
        if not os.path.exists(LIB_PATH):
            raise ImportError(f"{LIB_PATH} is missing: build it with `make -C {HERE}` (or __graft_entry__.build())")
        L = ctypes.CDLL(LIB_PATH)
        vp, i64, i64p, fp = ctypes.c_void_p, ctypes.c_int64, ctypes.POINTER(ctypes.c_int64), ctypes.c_void_p
        c_int, c_float = ctypes.c_int, ctypes.c_float
        L.mbr_last_error.restype = ctypes.c_char_p
        L.mbr_version.restype = c_int
        L.mbr_create.argtypes = [ctypes.c_char_p, c_int, c_int, ctypes.POINTER(vp)]
        L.mbr_destroy.argtypes = [vp]
        L.mbr_destroy.restype = None
        L.mbr_get_info.argtypes = [vp, c_int, i64p]
        L.mbr_output_length.argtypes = [vp, i64, i64p]
        L.mbr_forward_chunk.argtypes = [vp, fp, c_int, i64, fp, vp]
        L.mbr_forward_tap.argtypes = [vp, fp, c_int, i64, c_int, fp, i64p, vp]
        L.mbr_separate_device.argtypes = [vp, fp, i64, c_float, c_int, fp, vp]
        L.mbr_separate.argtypes = [vp, fp, i64, c_float, c_int, c_int, fp]
        L.mbr_shard_info.argtypes = [vp, i64, c_float, c_int, c_int, i64p]
        L.mbr_shard_run.argtypes = [vp, fp, i64, c_float, c_int, c_int, c_int, fp, fp, vp]
        L.mbr_shard_window.argtypes = [vp, i64, c_float, c_int, c_int, ctypes.POINTER(i64), ctypes.POINTER(i64)]
        L.mbr_plan_shard_window.argtypes = [i64, c_int, c_float, c_int, c_int, c_int, ctypes.POINTER(i64),
                                            ctypes.POINTER(i64)]
        L.mbr_shard_run_window.argtypes = [vp, fp, i64, i64, i64, c_float, c_int, c_int, c_int, fp, fp, vp]
        L.mbr_shard_add_boundary.argtypes = [vp, i64, c_float, c_int, c_int, fp, fp, fp, fp, i64, vp]
        L.mbr_shard_finalize.argtypes = [vp, i64, c_float, c_int, c_int, fp, fp, fp, i64, vp]
        L.mbr_set_backend.argtypes = [vp, c_int, c_int]
        L.mbr_set_graphs.argtypes = [vp, c_int]
        L.mbr_last_launches.argtypes = [vp, i64p]
        L.mbr_sync_check.argtypes = [vp]
        L.mbr_profile_enable.argtypes = [vp, c_int]
        L.mbr_profile_read.argtypes = [vp, c_int, ctypes.POINTER(ctypes.c_double), i64p]
        L.mbr_op_rms_norm.argtypes = [fp, fp, fp, i64, c_int, c_float, c_int, vp]
        L.mbr_op_add.argtypes = [fp, fp, fp, i64, c_int, vp]
        L.mbr_op_gelu.argtypes = [fp, fp, i64, c_int, vp]
        L.mbr_op_sigmoid_gate.argtypes = [fp, fp, fp, i64, c_int, c_int, c_int, vp]
        L.mbr_op_rope.argtypes = [fp, fp, fp, fp, i64, c_int, c_int, c_int, vp]
        L.mbr_op_linear.argtypes = [fp, fp, fp, fp, i64, c_int, c_int, c_int, c_int, vp]
        L.mbr_op_attention.argtypes = [fp, fp, fp, i64, c_int, c_int, c_int, c_float, fp, fp, c_int, vp]
        L.mbr_op_ffn.argtypes = [fp, fp, fp, fp, fp, fp, i64, c_int, c_int, c_int, vp]
        L.mbr_rope_tables.argtypes = [c_int, c_int, fp, fp]
        L.mbr_op_band_gather.argtypes = [vp, fp, c_int, c_int, fp, c_int, vp]
        L.mbr_op_mask_scatter.argtypes = [vp, fp, fp, c_int, c_int, c_int, fp, c_int, vp]
        L.mbr_op_stft.argtypes = [fp, i64, i64, c_int, fp, vp]
        L.mbr_op_istft.argtypes = [fp, i64, c_int, c_int, i64, fp, vp]
        L.mbr_op_istft_noalloc.argtypes = [fp, i64, c_int, c_int, i64, fp, vp]
        L.mbr_plan_shard.argtypes = [i64, c_int, c_float, c_int, c_int, c_int, i64p]
        L.mbr_wav_info.argtypes = [ctypes.c_char_p, ctypes.POINTER(c_int), ctypes.POINTER(c_int), i64p]
        L.mbr_wav_read.argtypes = [ctypes.c_char_p, fp, i64]
        L.mbr_wav_write.argtypes = [ctypes.c_char_p, fp, c_int, i64, c_int]
        L.mbr_pcm_to_planar.argtypes = [vp, i64, c_int, c_int, c_int, fp, vp]
        L.mbr_wav_read_device.argtypes = [ctypes.c_char_p, fp, i64, ctypes.POINTER(c_int), ctypes.POINTER(c_int),
                                          i64p, vp]
        L.mbr_wav_write_device.argtypes = [ctypes.c_char_p, fp, c_int, i64, c_int, vp]
        _lib = L
    return _lib


def _check(rc: int):
    if rc != 0:
        raise MBRError(rc, lib().mbr_last_error().decode())


def _ptr(t) -> int:
    """Device/host address of a torch tensor or numpy array."""
    if isinstance(t, np.ndarray):
        return t.ctypes.data
    return t.data_ptr()


def _stream(stream):
    if stream is None:
        import torch
        return ctypes.c_void_p(torch.cuda.current_stream().cuda_stream)
    return ctypes.c_void_p(stream if isinstance(stream, int) else stream.cuda_stream)


def _dt(t) -> int:
    """C-ABI dtype code of a torch tensor."""
    import torch

    return {torch.float32: FP32, torch.float16: FP16, torch.bfloat16: BF16}[t.dtype]


# ---- stand-alone ops (device tensors; reference op-library layouts) ----
def op_rms_norm(x, gamma, scale, y=None, stream=None):
    import torch

    y = torch.empty_like(x) if y is None else y
    rows, dim = x.shape[0], x.shape[-1]
    rows = x.numel() // dim
    _check(lib().mbr_op_rms_norm(_ptr(x), _ptr(gamma), _ptr(y), rows, dim, float(scale), _dt(x), _stream(stream)))
    return y


def op_add(a, b, y=None, stream=None):
    import torch

    y = torch.empty_like(a) if y is None else y
    _check(lib().mbr_op_add(_ptr(a), _ptr(b), _ptr(y), a.numel(), _dt(a), _stream(stream)))
    return y


def op_gelu(x, y=None, stream=None):
    import torch

    y = torch.empty_like(x) if y is None else y
    _check(lib().mbr_op_gelu(_ptr(x), _ptr(y), x.numel(), _dt(x), _stream(stream)))
    return y


def op_sigmoid_gate(x, gate, heads, y=None, stream=None):
    """x [rows, heads*dh], gate [rows, heads] -> x * gate (broadcast over dh)."""
    import torch

    y = torch.empty_like(x) if y is None else y
    rows = gate.numel() // heads
    dh = x.numel() // (rows * heads)
    _check(lib().mbr_op_sigmoid_gate(_ptr(x), _ptr(gate), _ptr(y), rows, heads, dh, _dt(x), _stream(stream)))
    return y


def rope_tables(L: int, dim_head: int = 64):
    c = np.empty((L, dim_head // 2), np.float32)
    s = np.empty((L, dim_head // 2), np.float32)
    _check(lib().mbr_rope_tables(L, dim_head, _ptr(c), _ptr(s)))
    return c, s


def op_rope(x, cos_t, sin_t, y=None, stream=None):
    """x [seqs, L, heads, 64] rotated by position."""
    import torch

    y = torch.empty_like(x) if y is None else y
    seqs, L, heads = x.shape[0], x.shape[1], x.shape[2]
    _check(lib().mbr_op_rope(_ptr(x), _ptr(cos_t), _ptr(sin_t), _ptr(y), seqs, L, heads, _dt(x), _stream(stream)))
    return y


ACT_NONE, ACT_GELU, ACT_TANH = 0, 1, 2


def op_linear(x, w, bias=None, act=ACT_NONE, out=None, stream=None):
    """x [rows, in] . w[out, in]^T + bias, then act; same dtype as x."""
    import torch

    rows, fin = x.shape
    fout = w.shape[0]
    out = torch.empty((rows, fout), dtype=x.dtype, device=x.device) if out is None else out
    b = _ptr(bias) if bias is not None else None
    _check(lib().mbr_op_linear(_ptr(x), _ptr(w), b, _ptr(out), rows, fin, fout, int(act), _dt(x), _stream(stream)))
    return out


def op_ffn(x, w1, b1, w2, b2, resid, stream=None):
    """resid [rows, dim] fp32 += GELU(x . w1^T + b1) . w2^T + b2 (x, w1 [hidden, dim], w2 [dim, hidden]
    fp16 / bf16; b1, b2 fp32), in place; returns resid."""
    rows, dim = x.shape
    hidden = w1.shape[0]
    assert w1.shape == (hidden, dim) and w2.shape == (dim, hidden) and resid.shape == (rows, dim)
    _check(lib().mbr_op_ffn(_ptr(x), _ptr(w1), _ptr(b1), _ptr(w2), _ptr(b2), _ptr(resid), rows, dim, hidden, _dt(x),
                            _stream(stream)))
    return resid


def op_attention(q, k, v, scale=0.0, gates=None, out=None, stream=None):
    """q, k, v [B, heads, N, dim_head] -> [B, N, heads * dim_head], times gates [B, N, heads] if given."""
    import torch

    B, H, N, D = q.shape
    out = torch.empty((B, N, H * D), dtype=q.dtype, device=q.device) if out is None else out
    g = _ptr(gates) if gates is not None else None
    _check(lib().mbr_op_attention(_ptr(q), _ptr(k), _ptr(v), B, H, N, D, float(scale), g, _ptr(out), _dt(q),
                                  _stream(stream)))
    return out


def op_stft(sig, hop=441, stream=None):
    """sig [n, L] float32 CUDA -> [n, 1025, T, 2]."""
    import torch

    n, L = sig.shape
    T = L // hop + 1
    out = torch.empty((n, 1025, T, 2), dtype=torch.float32, device=sig.device)
    _check(lib().mbr_op_stft(_ptr(sig), n, L, hop, _ptr(out), _stream(stream)))
    return out


def op_istft(spec, hop=441, length=-1, stream=None):
    """spec [n, 1025, T, 2] float32 CUDA -> [n, lout]."""
    import torch

    n, _, T, _ = spec.shape
    lout = length if length > 0 else (T - 1) * hop
    out = torch.empty((n, lout), dtype=torch.float32, device=spec.device)
    _check(lib().mbr_op_istft(_ptr(spec), n, T, hop, length, _ptr(out), _stream(stream)))
    return out


def plan_shard_window(N: int, chunk_size: int, overlap: float, default_overlap: int, rank: int, world: int):
    """Host-only: track samples (lo, hi) the shard of `rank` reads."""
    lo, hi = ctypes.c_int64(), ctypes.c_int64()
    _check(lib().mbr_plan_shard_window(int(N), int(chunk_size), float(overlap), int(default_overlap), rank, world,
                                       ctypes.byref(lo), ctypes.byref(hi)))
    return lo.value, hi.value


def wav_read_device(path: str, stream=None):
    """WAV file -> (planar float32 CUDA tensor [channels, frames], sample_rate),
    the samples converted on the GPU."""
    import torch

    sr, ch, n = ctypes.c_int(), ctypes.c_int(), ctypes.c_int64()
    _check(lib().mbr_wav_read_device(path.encode(), None, 0, ctypes.byref(sr), ctypes.byref(ch), ctypes.byref(n),
                                     _stream(stream)))
    out = torch.empty((ch.value, n.value), dtype=torch.float32, device="cuda")
    _check(lib().mbr_wav_read_device(path.encode(), _ptr(out), out.numel(), ctypes.byref(sr), ctypes.byref(ch),
                                     ctypes.byref(n), _stream(stream)))
    return out, sr.value


def wav_write_device(path: str, planar, sample_rate: int, stream=None) -> None:
    """planar float32 CUDA tensor [channels, frames] -> float32 WAV file."""
    ch, n = planar.shape
    _check(lib().mbr_wav_write_device(path.encode(), _ptr(planar.contiguous()), ch, n, int(sample_rate),
                                      _stream(stream)))


def pcm_to_planar(d_pcm, frames: int, channels: int, bits: int, is_float: bool, out, stream=None):
    """Interleaved PCM bytes on the device (uint8 CUDA tensor) -> out [channels, frames] float32."""
    _check(lib().mbr_pcm_to_planar(_ptr(d_pcm), int(frames), int(channels), int(bits), int(is_float), _ptr(out),
                                   _stream(stream)))
    return out


SHARD_KEYS = ["c0", "c1", "lo", "hi", "send_lo", "out_lo", "out_hi", "n_chunks", "step", "border", "total"]


def plan_shard(N: int, chunk_size: int, overlap: float, default_overlap: int, rank: int, world: int) -> dict:
    """Host-only shard plan (no GPU): chunk range and sample windows of `rank`."""
    info = (ctypes.c_int64 * 11)()
    _check(lib().mbr_plan_shard(int(N), int(chunk_size), float(overlap), int(default_overlap), rank, world, info))
    return dict(zip(SHARD_KEYS, list(info)))


def op_istft_noalloc(spec, out, hop=441, length=-1, stream=None):
    """Allocation-free iSTFT for callers that must not allocate device memory:
    spec [n, 1025, T, 2] and the caller's out [n, lout] (float32, CUDA).  Its
    frame scratch is a fixed 16 MiB array inside the library (n * T <= 2048);
    calls that overlap on the GPU share that array and race.  The first call
    on a device may load the library's module and reserve the array, so make
    it during set-up."""
    import torch

    if spec.dim() != 4 or spec.shape[1] != 1025 or spec.shape[3] != 2:
        raise ValueError(f"spec must be [n, 1025, T, 2], got {tuple(spec.shape)}")
    n, _, T, _ = spec.shape
    lout = length if length > 0 else (T - 1) * hop
    for name, t in (("spec", spec), ("out", out)):
        if t.dtype != torch.float32 or not t.is_contiguous() or not t.is_cuda:
            raise ValueError(f"{name} must be a contiguous float32 CUDA tensor")
    if out.device != spec.device:
        raise ValueError("spec and out must be on the same device")
    if tuple(out.shape) != (n, lout):
        raise ValueError(f"out must have shape {(n, lout)}, got {tuple(out.shape)}")
    with torch.cuda.device(spec.device):
        _check(lib().mbr_op_istft_noalloc(_ptr(spec), n, T, hop, length, _ptr(out), _stream(stream)))
    return out


class Model:
    """A loaded MelBandRoformer (`.csm`) on one GPU.

    dtype: "fp32" | "fp16" | "bf16" (the reference's --bf16/--fp16 switch; fp32
    keeps every weight in fp32).
    """

    def __init__(self, csm_path: str, device: int = 0, dtype="fp16"):
        self.h = ctypes.c_void_p()
        d = DTYPES[dtype] if isinstance(dtype, str) else int(dtype)
        _check(lib().mbr_create(csm_path.encode(), int(device), d, ctypes.byref(self.h)))
        self.device = int(device)
        self.path = csm_path

    def close(self):
        if self.h:
            lib().mbr_destroy(self.h)
            self.h = ctypes.c_void_p()

    def __del__(self):
        try:
            self.close()
        except Exception:
            pass

    def info(self, key: str) -> int:
        v = ctypes.c_int64()
        _check(lib().mbr_get_info(self.h, INFO[key], ctypes.byref(v)))
        return v.value

    def output_length(self, L: int) -> int:
        v = ctypes.c_int64()
        _check(lib().mbr_output_length(self.h, int(L), ctypes.byref(v)))
        return v.value

    def set_graphs(self, enable: bool = True):
        """CUDA-graph replay of the chunk forward (on by default)."""
        _check(lib().mbr_set_graphs(self.h, int(bool(enable))))

    def set_backend(self, gemm: int = BACKEND_TC, attention: int = BACKEND_TC):
        _check(lib().mbr_set_backend(self.h, int(gemm), int(attention)))

    def last_launches(self) -> int:
        v = ctypes.c_int64()
        _check(lib().mbr_last_launches(self.h, ctypes.byref(v)))
        return v.value

    def sync_check(self):
        """Synchronise the device and raise if a kernel reported a timed-out wait."""
        _check(lib().mbr_sync_check(self.h))

    def profile(self, on: bool = True):
        _check(lib().mbr_profile_enable(self.h, int(bool(on))))

    def profile_read(self) -> dict:
        """{kind: (milliseconds, launches)} accumulated since profile(True)."""
        out = {}
        for i, k in enumerate(PROFILE_KINDS):
            ms, n = ctypes.c_double(), ctypes.c_int64()
            _check(lib().mbr_profile_read(self.h, i, ctypes.byref(ms), ctypes.byref(n)))
            out[k] = (ms.value, n.value)
        return out

    # ---- device entry points (torch CUDA tensors) ----
    def forward(self, audio, out=None, stream=None):
        """audio: float32 CUDA tensor [B, C, L] -> [B, S, C, Lout]."""
        import torch
        assert audio.is_cuda and audio.dtype == torch.float32 and audio.is_contiguous()
        B, C, L = audio.shape
        S = self.info("num_stems")
        lo = self.output_length(L)
        if out is None:
            out = torch.empty((B, S, C, lo), dtype=torch.float32, device=audio.device)
        _check(lib().mbr_forward_chunk(self.h, _ptr(audio), B, L, _ptr(out), _stream(stream)))
        return out

    def tap(self, audio, tap: int, stream=None):
        import torch
        B, C, L = audio.shape
        n = ctypes.c_int64()
        _check(lib().mbr_forward_tap(self.h, _ptr(audio), B, L, tap, None, ctypes.byref(n), _stream(stream)))
        buf = torch.empty(n.value, dtype=torch.float32, device=audio.device)
        _check(lib().mbr_forward_tap(self.h, _ptr(audio), B, L, tap, _ptr(buf), ctypes.byref(n), _stream(stream)))
        return buf

    def separate_device(self, track, overlap: float = -1.0, chunk_batch: int = 1, out=None, stream=None):
        """track: float32 CUDA tensor [C, N] -> [S, C, N]."""
        import torch
        C, N = track.shape
        S = self.info("num_stems")
        if out is None:
            out = torch.empty((S, C, N), dtype=torch.float32, device=track.device)
        _check(lib().mbr_separate_device(self.h, _ptr(track), N, float(overlap), int(chunk_batch), _ptr(out),
                                         _stream(stream)))
        return out

    # ---- host entry point ----
    def separate(self, track: np.ndarray, overlap: float = -1.0, chunk_batch: int = 1, n_gpus: int = 1,
                 out: np.ndarray | None = None) -> np.ndarray:
        """track: float32 host array [C, N] -> [S, C, N] (host); synchronous."""
        track = np.ascontiguousarray(track, dtype=np.float32)
        C, N = track.shape
        S = self.info("num_stems")
        if out is None:
            out = np.empty((S, C, N), dtype=np.float32)
        _check(lib().mbr_separate(self.h, _ptr(track), N, float(overlap), int(chunk_batch), int(n_gpus), _ptr(out)))
        return out

    # ---- band ops with this checkpoint's band map ----
    def op_band_gather(self, spec, out_dtype=None, stream=None):
        """spec [B, C, 1025, T, 2] float32 -> [B, T, 2J]."""
        import torch

        B, C, F, T, _ = spec.shape
        J = self.info("band_freqs")
        out = torch.empty((B, T, 2 * J), dtype=out_dtype or torch.float32, device=spec.device)
        _check(lib().mbr_op_band_gather(self.h, _ptr(spec), B, T, _ptr(out), _dt(out), _stream(stream)))
        return out

    def op_mask_scatter(self, spec, masks, stream=None):
        """spec [B, C, 1025, T, 2] float32, masks [S, B*T, 2J] -> [B, S, C, 1025, T, 2]."""
        import torch

        B, C, F, T, _ = spec.shape
        S = masks.shape[0]
        out = torch.empty((B, S, C, F, T, 2), dtype=torch.float32, device=spec.device)
        _check(lib().mbr_op_mask_scatter(self.h, _ptr(spec), _ptr(masks), B, S, T, _ptr(out), _dt(masks),
                                         _stream(stream)))
        return out

    # ---- sharded (one process per GPU) ----
    def shard_info(self, N: int, overlap: float, rank: int, world: int) -> dict:
        info = (ctypes.c_int64 * 8)()
        _check(lib().mbr_shard_info(self.h, int(N), float(overlap), rank, world, info))
        keys = ["c0", "c1", "lo", "hi", "send_lo", "out_lo", "out_hi", "n_chunks"]
        return dict(zip(keys, list(info)))

    def shard_run(self, track, N, overlap, chunk_batch, rank, world, acc, wsum, stream=None):
        _check(lib().mbr_shard_run(self.h, _ptr(track), int(N), float(overlap), int(chunk_batch), rank, world,
                                   _ptr(acc), _ptr(wsum), _stream(stream)))

    def shard_window(self, N: int, overlap: float, rank: int, world: int):
        """Track samples (lo, hi) the shard of `rank` reads."""
        lo, hi = ctypes.c_int64(), ctypes.c_int64()
        _check(lib().mbr_shard_window(self.h, int(N), float(overlap), rank, world, ctypes.byref(lo), ctypes.byref(hi)))
        return lo.value, hi.value

    def shard_run_window(self, window, win_lo, N, overlap, chunk_batch, rank, world, acc, wsum, stream=None):
        """shard_run over window [C, win_len] = track samples [win_lo, win_lo + win_len)."""
        _check(lib().mbr_shard_run_window(self.h, _ptr(window), int(win_lo), int(window.shape[-1]), int(N),
                                          float(overlap), int(chunk_batch), rank, world, _ptr(acc), _ptr(wsum),
                                          _stream(stream)))

    def shard_add_boundary(self, N, overlap, rank, world, acc, wsum, racc, rwsum, rlen, stream=None):
        _check(lib().mbr_shard_add_boundary(self.h, int(N), float(overlap), rank, world, _ptr(acc), _ptr(wsum),
                                            _ptr(racc), _ptr(rwsum), int(rlen), _stream(stream)))

    def shard_finalize(self, N, overlap, rank, world, acc, wsum, out, out_stride, stream=None, out_col0=0):
        """Writes the shard's own track columns [out_lo, out_hi) into `out`
        ([S*C][out_stride]); with out_col0 = out_lo, `out` holds only those
        columns (column t at t - out_col0)."""
        _check(lib().mbr_shard_finalize(self.h, int(N), float(overlap), rank, world, _ptr(acc), _ptr(wsum),
                                        _ptr(out) - 4 * int(out_col0), int(out_stride), _stream(stream)))

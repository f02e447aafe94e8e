"""csm_tool — `.csm` v1 writer/reader, mel band-map generator and seeded
random-init MelBandRoformer checkpoints.

The reference loads MelBandRoformer weights from `.csm` files
(src/weights.h:82-96, src/weights.cu:412-509) whose band maps are precomputed
tensors (`__precomputed__.*`, src/model_mel_band_roformer.cu:79-150).  The
converter that writes them is not part of the reference, so this module is the
writer: it builds the band map with the published MelBandRoformer construction
(slaney mel filterbank, see `mel_band_map`) and writes configs and weights with
the tensor names MelBandRoformer::load expects (src/model_mel_band_roformer.cu:159-253).

Command line:
    python csm_tool.py random --preset std --seed 0 --out model.csm
    python csm_tool.py info model.csm
"""
from __future__ import annotations

import argparse
import json
import struct
import sys

import numpy as np

DTYPE_F32, DTYPE_F16, DTYPE_I64, DTYPE_BF16 = 0, 1, 2, 3

# Model presets.  The first five are the benchmark configurations; "tiny*" are
# small shapes for fast parity tests.
PRESETS = {
    # fp32 parity config: dim 192, depth 1, 8x32, 1 stem, one 8 s chunk.
    "pr1": dict(dim=192, depth=1, heads=8, dim_head=32, num_stems=1, chunk_size=352800, num_overlap=1),
    # dim 384, depth 6, 8x64, 1 stem, 8 s chunks, overlap 4.
    "std": dict(dim=384, depth=6, heads=8, dim_head=64, num_stems=1, chunk_size=352800, num_overlap=4),
    # dim 384, depth 12, 2 stems, 8 s chunks, overlap 4.
    "two_stem": dict(dim=384, depth=12, heads=8, dim_head=64, num_stems=2, chunk_size=352800, num_overlap=4),
    # dim 512, depth 12, 16x64, 2 stems, 11 s chunks, overlap 2.
    "large": dict(dim=512, depth=12, heads=16, dim_head=64, num_stems=2, chunk_size=485100, num_overlap=2),
    # the reference's own shape: dim 256, depth 12, 8x64, 2 stems, T=1301.
    "r0": dict(dim=256, depth=12, heads=8, dim_head=64, num_stems=2, chunk_size=573300, num_overlap=2),
    # small shapes for tests
    "tiny": dict(dim=64, depth=1, heads=2, dim_head=64, num_stems=1, chunk_size=44100, num_overlap=2),
    "tiny2": dict(dim=128, depth=2, heads=2, dim_head=64, num_stems=2, chunk_size=88200, num_overlap=4,
                  time_transformer_depth=2),
    # the std layer shapes (dim 384, 8x64) at depth 1 with 1 s chunks
    "mid": dict(dim=384, depth=1, heads=8, dim_head=64, num_stems=1, chunk_size=44100, num_overlap=2),
}


def base_config(**kw) -> dict:
    """Config keys read by MBRConfig::from_json (src/model_mel_band_roformer.cu:46-69)
    and by the app layer (src/inference_app.cpp:42-44, :298)."""
    cfg = dict(
        model_type="mel_band_roformer",
        dim=384, depth=6, stereo=True, num_stems=1,
        time_transformer_depth=1, freq_transformer_depth=1,
        num_bands=60, dim_head=64, heads=8, mask_estimator_depth=2,
        mlp_expansion_factor=4, zero_dc=True, sample_rate=44100,
        stft_n_fft=2048, stft_hop_length=441, stft_win_length=2048,
        stft_normalized=False, match_input_audio_length=False,
        dim_freqs_in=1025, skip_connection=False,
        chunk_size=352800, num_overlap=4,
    )
    cfg.update(kw)
    n = cfg["num_stems"]
    cfg.setdefault("instruments", ["vocals", "instrumental", "drums", "bass"][:n] if n <= 4
                   else [f"stem_{i}" for i in range(n)])
    return cfg


# ---------------------------------------------------------------------------
# Mel band map
# ---------------------------------------------------------------------------
def _hz_to_mel(f):
    f = np.asanyarray(f, dtype=np.float64)
    f_sp = 200.0 / 3
    mels = (f - 0.0) / f_sp
    min_log_hz = 1000.0
    min_log_mel = (min_log_hz - 0.0) / f_sp
    logstep = np.log(6.4) / 27.0
    if f.ndim:
        log_t = f >= min_log_hz
        mels[log_t] = min_log_mel + np.log(f[log_t] / min_log_hz) / logstep
    elif f >= min_log_hz:
        mels = min_log_mel + np.log(f / min_log_hz) / logstep
    return mels


def _mel_to_hz(m):
    m = np.asanyarray(m, dtype=np.float64)
    f_sp = 200.0 / 3
    freqs = 0.0 + f_sp * m
    min_log_hz = 1000.0
    min_log_mel = (min_log_hz - 0.0) / f_sp
    logstep = np.log(6.4) / 27.0
    log_t = m >= min_log_mel
    freqs[log_t] = min_log_hz * np.exp(logstep * (m[log_t] - min_log_mel))
    return freqs


def mel_band_map(sample_rate=44100, n_fft=2048, num_bands=60, stereo=True):
    """Band map of the published MelBandRoformer (lucidrains BS-RoFormer,
    `MelBandRoformer.__init__`) over librosa.filters.mel (slaney scale,
    htk=False, fmin=0, fmax=sr/2): bin j belongs to band i where the
    triangular weight is > 0, i.e. mel_f[i] < fft_f[j] < mel_f[i+2]; bin 0 is
    forced into band 0 and the Nyquist bin into the last band.  Stereo
    interleaves the two channels as 2*f + s.

    Returns (freq_indices [sum], num_freqs_per_band [num_bands],
    num_bands_per_freq [n_fft//2+1]) as int64 arrays.
    """
    nf = n_fft // 2 + 1
    fft_f = np.arange(0, nf) * (1.0 / (n_fft * (1.0 / sample_rate)))
    mn, mx = _hz_to_mel(0.0), _hz_to_mel(sample_rate / 2.0)
    mels = np.linspace(mn, mx, num_bands + 2)
    mel_f = _mel_to_hz(mels)
    fdiff = np.diff(mel_f)
    ramps = np.subtract.outer(mel_f, fft_f)
    member = np.zeros((num_bands, nf), dtype=bool)
    for i in range(num_bands):
        lower = -ramps[i] / fdiff[i]
        upper = ramps[i + 2] / fdiff[i + 1]
        member[i] = np.maximum(0, np.minimum(lower, upper)) > 0
    member[0, 0] = True
    member[-1, -1] = True
    if not member.any(axis=0).all():
        raise ValueError("band map leaves a frequency bin uncovered")
    idx = np.broadcast_to(np.arange(nf), (num_bands, nf))[member]
    if stereo:
        idx = (idx[:, None] * 2 + np.arange(2)[None, :]).reshape(-1)
    return (idx.astype(np.int64), member.sum(axis=1).astype(np.int64),
            member.sum(axis=0).astype(np.int64))


# ---------------------------------------------------------------------------
# .csm v1 I/O
# ---------------------------------------------------------------------------
def write_csm(path: str, config: dict, tensors: dict) -> None:
    """Write the .csm v1 layout of src/weights.h:82-96: magic CSM\\0, u32
    version=1, u32 json_len, json, u32 n_tensors, then per tensor u32
    name_len, name, u32 ndim, i64[ndim] shape, u32 dtype, raw data."""
    js = json.dumps(config).encode()
    with open(path, "wb") as f:
        f.write(b"CSM\x00")
        f.write(struct.pack("<II", 1, len(js)))
        f.write(js)
        f.write(struct.pack("<I", len(tensors)))
        for name, arr in tensors.items():
            arr = np.ascontiguousarray(arr)
            if arr.dtype == np.float32:
                dt = DTYPE_F32
            elif arr.dtype == np.float16:
                dt = DTYPE_F16
            elif arr.dtype == np.int64:
                dt = DTYPE_I64
            elif arr.dtype == np.uint16:  # raw bf16 bits
                dt = DTYPE_BF16
            else:
                raise TypeError(f"unsupported dtype {arr.dtype} for {name}")
            nb = name.encode()
            f.write(struct.pack("<I", len(nb)))
            f.write(nb)
            f.write(struct.pack("<I", arr.ndim))
            f.write(struct.pack(f"<{arr.ndim}q", *arr.shape))
            f.write(struct.pack("<I", dt))
            f.write(arr.tobytes())


def read_csm(path: str):
    """Read a .csm v1 file -> (config dict, {name: ndarray}); bf16 tensors come
    back as uint16 bit patterns."""
    with open(path, "rb") as f:
        data = f.read()
    if data[:4] != b"CSM\x00":
        raise ValueError("invalid magic (expected CSM\\0)")
    ver, jl = struct.unpack_from("<II", data, 4)
    if ver != 1:
        raise ValueError(f"unsupported version {ver}")
    p = 12
    cfg = json.loads(data[p:p + jl].decode())
    p += jl
    (nt,) = struct.unpack_from("<I", data, p)
    p += 4
    out = {}
    np_dt = {DTYPE_F32: np.float32, DTYPE_F16: np.float16, DTYPE_I64: np.int64, DTYPE_BF16: np.uint16}
    for _ in range(nt):
        (nl,) = struct.unpack_from("<I", data, p)
        p += 4
        name = data[p:p + nl].decode()
        p += nl
        (nd,) = struct.unpack_from("<I", data, p)
        p += 4
        shape = struct.unpack_from(f"<{nd}q", data, p)
        p += 8 * nd
        (dt,) = struct.unpack_from("<I", data, p)
        p += 4
        t = np.dtype(np_dt[dt])
        n = int(np.prod(shape)) if nd else 1
        out[name] = np.frombuffer(data, dtype=t, count=n, offset=p).reshape(shape).copy()
        p += n * t.itemsize
    return cfg, out


# ---------------------------------------------------------------------------
# Random-init weights
# ---------------------------------------------------------------------------
def random_weights(cfg: dict, seed: int = 0, std: float = 0.02) -> dict:
    """Seeded random-init MelBandRoformer weights: every Linear weight and
    bias ~ N(0, std), every RMSNorm gamma = 1, plus the precomputed band map.
    Names follow MelBandRoformer::load (src/model_mel_band_roformer.cu:159-253)."""
    rng = np.random.default_rng(seed)
    C = 2 if cfg["stereo"] else 1
    fi, nfpb, nbpf = mel_band_map(cfg["sample_rate"], cfg["stft_n_fft"], cfg["num_bands"], cfg["stereo"])
    D, H, dh = cfg["dim"], cfg["heads"], cfg["dim_head"]
    DI = H * dh
    hid = D * cfg["mlp_expansion_factor"]
    t = {}

    def lin(name, out_f, in_f, bias=True):
        t[name + ".weight"] = rng.normal(0.0, std, (out_f, in_f)).astype(np.float32)
        if bias:
            t[name + ".bias"] = rng.normal(0.0, std, (out_f,)).astype(np.float32)

    bd = [2 * int(n) * C for n in nfpb]
    for b in range(cfg["num_bands"]):
        p = f"band_split.to_features.{b}"
        t[p + ".0.gamma"] = np.ones(bd[b], np.float32)
        lin(p + ".1", D, bd[b])
    for d in range(cfg["depth"]):
        for kind, depth in ((0, cfg["time_transformer_depth"]), (1, cfg["freq_transformer_depth"])):
            tp = f"layers.{d}.{kind}"
            for l in range(depth):
                lp = f"{tp}.layers.{l}"
                t[lp + ".0.norm.gamma"] = np.ones(D, np.float32)
                lin(lp + ".0.to_qkv", 3 * DI, D, bias=False)
                lin(lp + ".0.to_gates", H, D)
                lin(lp + ".0.to_out.0", D, DI, bias=False)
                t[lp + ".1.net.0.gamma"] = np.ones(D, np.float32)
                lin(lp + ".1.net.1", hid, D)
                lin(lp + ".1.net.4", D, hid)
            t[tp + ".norm.gamma"] = np.ones(D, np.float32)
    md = cfg["mask_estimator_depth"]
    for s in range(cfg["num_stems"]):
        for b in range(cfg["num_bands"]):
            dims = [D] + [hid] * md + [2 * bd[b]]
            for i in range(md + 1):
                lin(f"mask_estimators.{s}.to_freqs.{b}.0.{2 * i}", dims[i + 1], dims[i])
    t["__precomputed__.freq_indices"] = fi
    t["__precomputed__.num_freqs_per_band"] = nfpb
    t["__precomputed__.num_bands_per_freq"] = nbpf
    return t


# ---------------------------------------------------------------------------
# Seeded synthetic tracks (the reference's own test WAVs are private; these
# stand in for them in benchmarks and parity fixtures)
# ---------------------------------------------------------------------------
def pink_noise(seconds: float, seed: int, channels: int = 2, sample_rate: int = 44100) -> np.ndarray:
    """Seeded 1/f noise, RMS -18 dBFS, quantised to 16-bit levels (k / 32768):
    [channels, round(seconds * sample_rate)] float32."""
    n = int(round(seconds * sample_rate))
    rng = np.random.default_rng(seed)
    out = np.empty((channels, n), np.float32)
    for c in range(channels):
        w = rng.standard_normal(n)
        X = np.fft.rfft(w)
        f = np.arange(X.shape[0], dtype=np.float64)
        f[0] = 1.0
        X /= np.sqrt(f)
        x = np.fft.irfft(X, n)
        x *= (10 ** (-18 / 20)) / np.sqrt(np.mean(x ** 2))
        out[c] = np.clip(np.round(x * 32768.0), -32768, 32767) / 32768.0
    return out


def uniform_noise16(n: int, seed: int, channels: int = 2, amp: float = 0.5) -> np.ndarray:
    """Seeded uniform noise in [-amp, amp] quantised to 16-bit levels (a clip
    stored as a 16-bit WAV and read back): [channels, n] float32."""
    x = np.random.default_rng(seed).uniform(-amp, amp, (channels, n))
    return (np.clip(np.round(x * 32768.0), -32768, 32767) / 32768.0).astype(np.float32)


def make_random_csm(path: str, preset: str = "std", seed: int = 0, **overrides) -> dict:
    cfg = base_config(**{**PRESETS[preset], **overrides})
    write_csm(path, cfg, random_weights(cfg, seed))
    return cfg


def main(argv=None):
    ap = argparse.ArgumentParser(description=__doc__, formatter_class=argparse.RawDescriptionHelpFormatter)
    sub = ap.add_subparsers(dest="cmd", required=True)
    r = sub.add_parser("random", help="write a seeded random-init checkpoint")
    r.add_argument("--preset", default="std", choices=sorted(PRESETS))
    r.add_argument("--seed", type=int, default=0)
    r.add_argument("--out", required=True)
    r.add_argument("--set", action="append", default=[], help="config override key=json_value")
    i = sub.add_parser("info", help="print config and tensor count")
    i.add_argument("path")
    a = ap.parse_args(argv)
    if a.cmd == "random":
        ov = {}
        for kv in a.set:
            k, v = kv.split("=", 1)
            ov[k] = json.loads(v)
        cfg = make_random_csm(a.out, a.preset, a.seed, **ov)
        print(json.dumps(cfg))
    else:
        cfg, t = read_csm(a.path)
        print(json.dumps(cfg, indent=1))
        print(f"{len(t)} tensors")
    return 0


if __name__ == "__main__":
    sys.exit(main())

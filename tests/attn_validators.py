"""Restatement of the reference's own attention validators, the only known
answers its test code holds for this path (test infrastructure).

* Inputs: q = k = v of one (sequence, head) slice filled by the reference's
  deterministic generator, value(idx) = bf16(0.125 + ((17 idx) & 1023) * 2^-12)
  over the flat [L][64] slice (fill_bf16_kernel,
  bench/bf16_time_attention_cutile.cu:320-329; bench/bf16_freq_attention_cutile.cu:166-173).
* Time axis, L = 1301 (validate_rows, bench/bf16_time_attention_cutile.cu:3920-3984):
  fp32 online softmax over 64-key tiles, scale 1/8, probabilities rounded to
  bf16 before P.V and summed as rounded, the output rounded to bf16; rows
  0, 37 and L-1.
* Band axis, L = 60 (validate_q16, bench/bf16_freq_attention_cutile.cu:1496-1546):
  full-row fp32 softmax, bf16 probabilities, bf16 output; every row.
"""
import numpy as np

D = 64


def bf16(x):
    """Round fp32 values to bf16 (nearest even) and back."""
    x = np.ascontiguousarray(x, np.float32)
    u = x.view(np.uint32).astype(np.uint64)
    u = (u + 0x7FFF + ((u >> 16) & 1)) & 0xFFFF0000
    return u.astype(np.uint32).view(np.float32)


def inputs(L):
    idx = np.arange(L * D, dtype=np.int64)
    v = np.float32(0.125) + ((idx * 17) & 1023).astype(np.float32) * np.float32(0.000244140625)
    return bf16(v).reshape(L, D)


def time_rows(x, rows=(0, 37), ktile=64, scale=0.125):
    """validate_rows: online softmax in fp32 over key tiles of `ktile`."""
    L = x.shape[0]
    rows = list(rows) + [L - 1]
    out = {}
    f32 = np.float32
    for r in rows:
        acc = np.zeros(D, f32)
        row_m, row_l = f32(-3.402823466e38), f32(0)
        for kt in range(0, -(-L // ktile) * ktile, ktile):
            cols = np.arange(kt, min(kt + ktile, L))
            sc = (x[cols].astype(f32) @ x[r].astype(f32)).astype(f32) * f32(scale)
            new_m = max(row_m, f32(sc.max()))
            alpha = f32(np.exp(f32(row_m - new_m)))
            acc = (acc * alpha).astype(f32)
            p = bf16(np.exp((sc - new_m).astype(f32)).astype(f32))
            acc = (acc + (p[:, None] * x[cols]).sum(0, dtype=f32)).astype(f32)
            row_l = f32(row_l * alpha + p.sum(dtype=f32))
            row_m = new_m
        out[r] = bf16(acc / row_l)
    return out


def band_rows(x, scale=0.125):
    """validate_q16: full-row softmax in fp32."""
    f32 = np.float32
    sc = (x @ x.T).astype(f32) * f32(scale)
    p = bf16(np.exp(sc - sc.max(1, keepdims=True)).astype(f32))
    return bf16((p @ x).astype(f32) / p.sum(1, keepdims=True, dtype=f32))


def err_ulps(got, ref):
    """max |got - ref| in units of the bf16 ulp at |ref| (the validators' own
    output rounding is half of one)."""
    ref = np.asarray(ref, np.float64)
    ulp = 2.0 ** (np.floor(np.log2(np.abs(ref))) - 7)
    return float((np.abs(np.asarray(got, np.float64) - ref) / ulp).max())

"""Error metrics used by the parity tests."""
import numpy as np


def gelu_ref(x):
    """The reference's GELU, 0.5 x (1 + erf(x)) (erf of x itself, not of x/sqrt2:
    add_bias_gelu_kernel, src/mbr_cuda_tile.cu:5536-5558), in float64."""
    from scipy.special import erf

    x = np.asarray(x, np.float64)
    return 0.5 * x * (1.0 + erf(x))


def rel_max_err(ref: np.ndarray, got: np.ndarray) -> float:
    """max |got - ref| / max |ref| (the fp32 parity measure; bar 1e-4)."""
    ref = np.asarray(ref, np.float64)
    got = np.asarray(got, np.float64)
    den = np.abs(ref).max()
    return float(np.abs(got - ref).max() / (den if den > 0 else 1.0))


def snr_db(ref: np.ndarray, got: np.ndarray) -> float:
    """Signal-to-error ratio of got against ref in dB (the fp16/bf16 measure; bar 60 dB)."""
    ref = np.asarray(ref, np.float64)
    got = np.asarray(got, np.float64)
    err = np.sum((got - ref) ** 2)
    sig = np.sum(ref ** 2)
    if err == 0:
        return float("inf")
    return float(10.0 * np.log10(sig / err))

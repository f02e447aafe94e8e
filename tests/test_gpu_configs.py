"""GPU parity at the benchmark configurations: full depth, full chunks, the real
shapes (T = 801 / 1101 frames, dim 384 / 512, 8 / 16 heads, 1 / 2 stems).

* PR1 (fp32, dim 192, depth 1, 8x32, one 8 s chunk of 16-bit uniform noise,
  the single-chunk path of run_inference): against the live CPU oracle,
  max |err| / max |ref| <= 1e-4.
* Std (fp16, dim 384, depth 6, one 8 s chunk) and Large (fp16, dim 512,
  depth 12, 16x64, 2 stems, one 11 s chunk): stem SNR >= 60 dB against the
  oracle output in tests/golden/config_<case>.npz (made by
  tests/golden/make_config_golden.py; the oracle needs minutes per chunk at
  these sizes).
* Two-stem (bf16, dim 384, depth 12, 2 stems, chunk-batch 4): against both the
  exact oracle (bf16 weights, fp32 storage, fp64 sums) and the oracle's
  reference-bf16 mode (activations rounded where the reference's --bf16 path
  stores them).  The reference's own bf16 rounding puts it 37.5 dB from the
  exact forward at this depth, so no bf16 implementation with another
  summation order can be 60 dB from it; the bar is instead that this bf16
  forward is at least as close to the exact forward as the reference's bf16
  scheme is, and as close to the reference-bf16 output as the exact forward
  is, within 1.5 dB.

Inputs (weights and audio) are rebuilt from seeds and checked against the
fixture's SHA-256 digests; on a mismatch the oracle runs live instead.
"""
import os

import numpy as np
import pytest

from metrics import rel_max_err, snr_db

pytestmark = pytest.mark.gpu

HERE = os.path.dirname(os.path.abspath(__file__))
FP32_TOL = 1e-4
FP16_SNR_DB = 60.0
BF16_REF_MARGIN_DB = 1.5


@pytest.fixture(scope="module")
def torch_cuda():
    import torch

    if not torch.cuda.is_available():
        pytest.skip("no CUDA device")
    return torch


def _golden():
    import sys

    sys.path.insert(0, os.path.join(HERE, "golden"))
    import make_config_golden

    return make_config_golden


def _reference(name, path, x):
    """Oracle output subsample for case `name`: the committed fixture when the
    rebuilt inputs match it, else a live oracle run."""
    g = _golden()
    case = g.CASES[name]
    fx = np.load(g.fixture_path(name))
    if str(fx["csm_sha"]) == g.sha256_file(path) and str(fx["input_sha"]) == g.sha256_array(x):
        out = {"ref": fx["ref"], "stride": int(fx["stride"]), "shape": tuple(fx["shape"])}
        if "ref_bf16" in fx:
            out["ref_bf16"] = fx["ref_bf16"]
        return out
    import oracle

    print(f"{name}: rebuilt inputs differ from the fixture's; running the oracle live")
    ref = oracle.Model(path, case["wdt"]).forward(x)
    stride = max(1, ref.size // g.TARGET_SAMPLES)
    out = {"ref": g.subsample(ref, stride), "stride": stride, "shape": ref.shape}
    if "ref_bf16_wdt" in case:
        out["ref_bf16"] = g.subsample(oracle.Model(path, case["ref_bf16_wdt"]).forward(x), stride)
    return out


def _run_case(torch, make_csm, name):
    import cudasep

    g = _golden()
    case = g.CASES[name]
    path = make_csm(case["preset"], seed=case["seed"])
    x = g.case_audio(case)
    ref = _reference(name, path, x)
    m = cudasep.Model(path, 0, case["dtype"])
    got = m.forward(torch.from_numpy(x).cuda()).cpu().numpy()
    m.sync_check()
    assert got.shape == ref["shape"], (got.shape, ref["shape"])
    return ref, g.subsample(got, ref["stride"]), got


def test_pr1_fp32_matches_oracle(torch_cuda, make_csm):
    """PR1: one 8 s chunk through mbr_separate (the single-chunk path) and the
    chunk forward, fp32 compute, against the live oracle."""
    import csm_tool
    import cudasep
    import oracle

    path = make_csm("pr1", seed=107)
    x = csm_tool.uniform_noise16(352800, 307)
    orc = oracle.Model(path, 0)
    ref = orc.separate(x)
    m = cudasep.Model(path, 0, "fp32")
    got = m.separate(x)
    err = rel_max_err(ref, got)
    print(f"pr1 fp32 separate: max rel err {err:.3e}")
    assert got.shape == ref.shape and err <= FP32_TOL
    fwd = m.forward(torch_cuda.from_numpy(x[None].copy()).cuda()).cpu().numpy()
    m.sync_check()
    err_f = rel_max_err(orc.forward(x[None]), fwd)
    print(f"pr1 fp32 forward: max rel err {err_f:.3e}")
    assert err_f <= FP32_TOL


@pytest.mark.parametrize("name", ["std", "large"])
def test_fp16_config_chunk_snr(torch_cuda, make_csm, name):
    ref, sub, _ = _run_case(torch_cuda, make_csm, name)
    s = snr_db(ref["ref"], sub)
    print(f"{name} fp16 chunk forward {ref['shape']}: SNR vs oracle {s:.2f} dB")
    assert s >= FP16_SNR_DB


def test_two_stem_bf16_chunk_batch4(torch_cuda, make_csm):
    ref, sub, got = _run_case(torch_cuda, make_csm, "two_stem")
    s_exact = snr_db(ref["ref"], sub)
    s_refbf16 = snr_db(ref["ref_bf16"], sub)
    s_ref_scheme = snr_db(ref["ref"], ref["ref_bf16"])
    print(f"two_stem bf16 chunk-batch 4 {ref['shape']}: SNR vs exact oracle {s_exact:.2f} dB, "
          f"vs reference-bf16 oracle {s_refbf16:.2f} dB; reference-bf16 vs exact {s_ref_scheme:.2f} dB")
    assert np.isfinite(got).all()
    assert s_exact >= s_ref_scheme, "bf16 forward less accurate than the reference's bf16 scheme"
    assert s_refbf16 >= s_ref_scheme - BF16_REF_MARGIN_DB

"""The allocation-free iSTFT entry point (mbr_op_istft_noalloc).

It exists for callers that may not allocate device memory while they run (for
example a real-time audio host whose processing thread must not block in an
allocator).  It must give the same output as mbr_op_istft, which takes its
scratch from the stream-ordered allocator, on two calls in a row (the second
call reuses the library's fixed scratch array left over from the first), and
reject inputs larger than that array.  This file is collected last.
"""
import ctypes

import numpy as np
import pytest

pytestmark = pytest.mark.gpu

TOL = 1e-6  # both entry points run the same kernels in fp32


@pytest.fixture(scope="module")
def torch_cuda():
    import torch

    if not torch.cuda.is_available():
        pytest.skip("no CUDA device")
    return torch


def _spec(torch, n, T, seed):
    rng = np.random.default_rng(seed)
    s = rng.standard_normal((n, 1025, T, 2)).astype(np.float32)
    return torch.from_numpy(s).cuda()


def test_noalloc_istft_matches_allocating_entry_point_twice(torch_cuda):
    torch = torch_cuda
    import cudasep

    for call, (n, T, length) in enumerate([(2, 801, -1), (3, 101, 44100 + 7)]):
        spec = _spec(torch, n, T, seed=call)
        ref = cudasep.op_istft(spec, length=length)
        out = torch.full_like(ref, float("nan"))
        cudasep.op_istft_noalloc(spec, out, length=length)
        torch.cuda.synchronize()
        err = (out - ref).abs().max().item()
        assert err <= TOL * max(1.0, ref.abs().max().item()), f"call {call}: max err {err:.3e}"


def test_noalloc_istft_rejects_oversized_input(torch_cuda):
    torch = torch_cuda
    import cudasep

    spec = torch.zeros((3, 1025, 700, 2), dtype=torch.float32, device="cuda")  # 2100 frames > 2048
    out = torch.zeros((3, 699 * 441), dtype=torch.float32, device="cuda")
    with pytest.raises(cudasep.MBRError) as e:
        cudasep.op_istft_noalloc(spec, out)
    assert e.value.code == 1 and b"static scratch" in cudasep.lib().mbr_last_error()

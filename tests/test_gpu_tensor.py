"""GPU check of the Tensor API (reference src/tensor.h interface) and its
caching allocator: runs the native self-test, which compares every Tensor
method with a host computation."""
import os
import subprocess

import pytest

pytestmark = pytest.mark.gpu

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
EXE = os.path.join(ROOT, "tests", "native", "_build", "tensor_selftest")


def test_tensor_api_selftest():
    import torch

    if not torch.cuda.is_available():
        pytest.skip("no CUDA device")
    assert os.path.exists(EXE), "build it with make -C mbr-cuda-tile_b200"
    r = subprocess.run([EXE], capture_output=True, text=True, timeout=300)
    print(r.stdout)
    assert r.returncode == 0 and "tensor_selftest: OK" in r.stdout, r.stdout + r.stderr

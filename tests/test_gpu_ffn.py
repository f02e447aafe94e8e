"""GPU tests of the fused feed-forward block (mbr_op_ffn: FFN1 + GELU + FFN2 and
the residual add in one tcgen05 kernel, the reference's
try_feedforward_fused_residual, src/mbr_cuda_tile.cu:6840) against fp64 math on
the same rounded operands.

The kernel rounds the hidden activations GELU(x w1^T + b1) to the compute dtype
(they feed the second contraction as 16-bit operands, as the reference's
kernels do); the reference here rounds them the same way, so what remains is
fp32 accumulation and the rare hidden value whose rounding falls on the other
side of a 16-bit boundary.  Bar: max |got - ref| / max |update| below TOL.

The shapes cover one row (a single tile whose 24 hidden chunks are spread over
24 CTAs, each reduce-adding its part), ragged last tiles, tiles split between
two CTAs, dim 256 (one 256-wide O MMA) and 384 (two 192-wide), a single hidden
chunk, and the std activation shape (801 frames x 60 bands).
"""
import numpy as np
import pytest

from metrics import gelu_ref

pytestmark = pytest.mark.gpu

TOL = {"fp16": 2e-3, "bf16": 1e-2}


@pytest.fixture(scope="module")
def torch_cuda():
    import torch

    if not torch.cuda.is_available():
        pytest.skip("no CUDA device")
    return torch


@pytest.mark.parametrize(
    "dtype,dim,hidden,rows",
    [
        ("fp16", 384, 1536, 1),
        ("fp16", 384, 1536, 1000),
        ("bf16", 384, 1536, 4097),
        ("fp16", 256, 1024, 3000),
        ("bf16", 256, 64, 130),
        ("fp16", 384, 1536, 48060),
    ],
)
def test_ffn_op(torch_cuda, dtype, dim, hidden, rows):
    torch = torch_cuda
    import cudasep

    tdt = torch.float16 if dtype == "fp16" else torch.bfloat16
    g = torch.Generator().manual_seed(rows * 7 + dim + hidden)
    x = torch.randn(rows, dim, generator=g).to(tdt)
    w1 = (torch.randn(hidden, dim, generator=g) / np.sqrt(dim)).to(tdt)
    b1 = torch.randn(hidden, generator=g) * 0.1
    w2 = (torch.randn(dim, hidden, generator=g) / np.sqrt(hidden)).to(tdt)
    b2 = torch.randn(dim, generator=g) * 0.1
    r0 = torch.randn(rows, dim, generator=g)
    r = r0.cuda()
    cudasep.op_ffn(x.cuda(), w1.cuda(), b1.cuda(), w2.cuda(), b2.cuda(), r)
    got = r.double().cpu().numpy()

    pre = x.double().numpy() @ w1.double().numpy().T + b1.double().numpy()
    h = torch.from_numpy(gelu_ref(pre)).to(tdt).double().numpy()  # the kernel's 16-bit hidden values
    upd = h @ w2.double().numpy().T + b2.double().numpy()
    ref = r0.double().numpy() + upd
    err = np.abs(got - ref).max() / np.abs(upd).max()
    print(f"ffn {dtype} rows {rows} dim {dim} hidden {hidden}: max err / max |update| {err:.2e}")
    assert np.isfinite(got).all()
    assert err <= TOL[dtype]


def test_ffn_op_rejects_unsupported(torch_cuda):
    """dim 512 does not fit TMEM beside two hidden chunks: the op refuses it
    (the model keeps the two-GEMM path there)."""
    torch = torch_cuda
    import cudasep

    x = torch.zeros(8, 512, dtype=torch.float16, device="cuda")
    w1 = torch.zeros(2048, 512, dtype=torch.float16, device="cuda")
    w2 = torch.zeros(512, 2048, dtype=torch.float16, device="cuda")
    b1 = torch.zeros(2048, device="cuda")
    b2 = torch.zeros(512, device="cuda")
    r = torch.zeros(8, 512, device="cuda")
    with pytest.raises(cudasep.MBRError):
        cudasep.op_ffn(x, w1, b1, w2, b2, r)

"""GPU parity of the stand-alone op entry points (the reference op library's
ops, at the op-sweep benchmark shapes) against CPU references.

Inputs are seeded N(0, 1) activations of shape [B*801*60, D].  The CPU
reference evaluates in fp64 from the same (already rounded) inputs; tolerances:
fp32 max abs err <= 1e-5 * max|ref| (+1e-6), fp16 <= 2^-10 relative to the
output magnitude, bf16 <= 2^-7 (one rounding of the output).  STFT / iSTFT are
checked against the CPU oracle; band gather / mask scatter bit-exact (gather)
and 1e-6 relative (scatter) against numpy on the checkpoint's band map.
"""
import numpy as np
import pytest

from metrics import gelu_ref

pytestmark = pytest.mark.gpu

T = 801
NB = 60
TOL = {"fp32": 1e-5, "fp16": 2.0 ** -10, "bf16": 2.0 ** -7}


@pytest.fixture(scope="module")
def torch_cuda():
    import torch

    if not torch.cuda.is_available():
        pytest.skip("no CUDA device")
    return torch


def _tdt(torch, name):
    return {"fp32": torch.float32, "fp16": torch.float16, "bf16": torch.bfloat16}[name]


def _inputs(torch, rows, D, dtype, seed=0, n=1):
    g = torch.Generator().manual_seed(seed)
    return [torch.randn(rows, D, generator=g).to(_tdt(torch, dtype)) for _ in range(n)]


def _close(got, ref, dtype, what):
    got = got.double().cpu().numpy() if hasattr(got, "cpu") else np.asarray(got, np.float64)
    ref = np.asarray(ref, np.float64)
    tol = TOL[dtype]
    err = np.abs(got - ref)
    bound = tol * np.maximum(np.abs(ref), 1.0) * 1.01 + (1e-6 if dtype == "fp32" else 0)
    assert np.all(err <= bound), f"{what}/{dtype}: max err {err.max():.3e}"


@pytest.mark.parametrize("dtype", ["fp32", "fp16", "bf16"])
@pytest.mark.parametrize("D", [192, 384, 512])
def test_rms_norm_add_gelu(torch_cuda, dtype, D):
    torch = torch_cuda
    import cudasep

    rows = 1 * T * NB
    x, y = _inputs(torch, rows, D, dtype, seed=D, n=2)
    gamma = torch.linspace(0.5, 1.5, D)
    scale = float(np.sqrt(np.float32(D)))
    xd, yd, gd = x.cuda(), y.cuda(), gamma.cuda()
    xr = x.double().numpy()
    ref = xr / np.sqrt((xr ** 2).sum(-1, keepdims=True) + 1e-12) * gamma.double().numpy() * scale
    _close(cudasep.op_rms_norm(xd, gd, scale), ref, dtype, "rms_norm")
    _close(cudasep.op_add(xd, yd), xr + y.double().numpy(), dtype, "add")

    _close(cudasep.op_gelu(xd), gelu_ref(xr), dtype, "gelu")


@pytest.mark.parametrize("dtype", ["fp32", "fp16", "bf16"])
@pytest.mark.parametrize("rows,D", [(1001, 64), (1003, 128), (999, 192), (1001, 200), (7, 384), (5, 1024), (1, 512)])
def test_ragged_rows(torch_cuda, dtype, rows, D):
    """Row counts that leave a partial row group (RMSNorm) and element counts
    that leave a partial unrolled step (add, GELU)."""
    torch = torch_cuda
    import cudasep

    x, y = _inputs(torch, rows, D, dtype, seed=rows + D, n=2)
    gamma = torch.linspace(0.25, 2.0, D)
    xd, yd, gd = x.cuda(), y.cuda(), gamma.cuda()
    xr = x.double().numpy()
    ref = xr / np.sqrt((xr ** 2).sum(-1, keepdims=True) + 1e-12) * gamma.double().numpy() * 3.0
    _close(cudasep.op_rms_norm(xd, gd, 3.0), ref, dtype, "rms_norm")
    _close(cudasep.op_add(xd, yd), xr + y.double().numpy(), dtype, "add")

    _close(cudasep.op_gelu(xd), gelu_ref(xr), dtype, "gelu")


@pytest.mark.parametrize("dtype", ["fp32", "fp16", "bf16"])
def test_sigmoid_gate_and_rope(torch_cuda, dtype):
    torch = torch_cuda
    import cudasep

    H = 8
    rows = T * NB
    (x,) = _inputs(torch, rows, H * 64, dtype, seed=5)
    g = torch.sigmoid(torch.randn(rows, H, generator=torch.Generator().manual_seed(6))).to(x.dtype)
    ref = x.double().numpy().reshape(rows, H, 64) * g.double().numpy()[:, :, None]
    _close(cudasep.op_sigmoid_gate(x.cuda(), g.cuda(), H), ref.reshape(rows, -1), dtype, "gate")
    # RoPE over T: x viewed as [60 sequences][T][H][64]
    c, s = cudasep.rope_tables(T, 64)
    xs = x.reshape(NB, T, H, 64)
    got = cudasep.op_rope(xs.cuda(), torch.from_numpy(c).cuda(), torch.from_numpy(s).cuda())
    xr = xs.double().numpy()
    x0, x1 = xr[..., 0::2], xr[..., 1::2]
    cc, ss = c.astype(np.float64)[None, :, None, :], s.astype(np.float64)[None, :, None, :]
    ref = np.empty_like(xr)
    ref[..., 0::2] = x0 * cc - x1 * ss
    ref[..., 1::2] = x0 * ss + x1 * cc
    _close(got, ref, dtype, "rope")


def test_rope_tables_match_reference_formula():
    import cudasep

    c, s = cudasep.rope_tables(801, 64)
    # compute_rotary_cos_sin: angle = n / 10000^(2i/dim), evaluated in fp32 on the
    # host (so the angle carries up to ~n * 2^-24 rad of rounding: <= 1e-4 at n = 800)
    i = np.arange(32, dtype=np.float64)
    ang = np.arange(801, dtype=np.float64)[:, None] / np.power(10000.0, 2 * i / 64)[None, :]
    assert np.abs(c - np.cos(ang)).max() < 2e-4
    assert np.abs(s - np.sin(ang)).max() < 2e-4
    assert np.abs(c[:16] - np.cos(ang[:16])).max() < 1e-6


def test_stft_istft_match_oracle(torch_cuda):
    torch = torch_cuda
    import cudasep
    import oracle

    rng = np.random.default_rng(3)
    x = rng.uniform(-0.5, 0.5, (3, 44100 + 123)).astype(np.float32)
    S = cudasep.op_stft(torch.from_numpy(x).cuda()).cpu().numpy()
    ref = oracle.stft(x)
    assert S.shape == ref.shape
    assert np.abs(S - ref).max() <= 1e-5 * np.abs(ref).max()
    y = cudasep.op_istft(torch.from_numpy(ref).cuda()).cpu().numpy()
    yr = oracle.istft(ref)
    assert y.shape == yr.shape
    assert np.abs(y - yr).max() <= 1e-5
    y2 = cudasep.op_istft(torch.from_numpy(ref).cuda(), length=x.shape[1]).cpu().numpy()
    assert y2.shape == x.shape and np.abs(y2[:, : yr.shape[1]] - yr).max() <= 1e-5


@pytest.mark.parametrize("B,dtype", [(1, "fp32"), (2, "fp16"), (1, "bf16")])
def test_band_gather_and_mask_scatter(torch_cuda, make_csm, B, dtype):
    torch = torch_cuda
    import csm_tool
    import cudasep

    path = make_csm("tiny", seed=31)
    _, t = csm_tool.read_csm(path)
    fi = t["__precomputed__.freq_indices"]
    nbpf = t["__precomputed__.num_bands_per_freq"]
    J = fi.shape[0]
    m = cudasep.Model(path, 0, "fp32")
    rng = np.random.default_rng(B)
    spec = rng.standard_normal((B, 2, 1025, T, 2)).astype(np.float32)
    xd = m.op_band_gather(torch.from_numpy(spec).cuda(), out_dtype=_tdt(torch, dtype))
    ch, f = fi % 2, fi // 2
    ref = spec[:, ch, f, :, :].transpose(0, 2, 1, 3).reshape(B, T, 2 * J)
    assert np.array_equal(xd.float().cpu().numpy(), torch.from_numpy(ref).to(_tdt(torch, dtype)).float().numpy())
    # mask scatter-average, S = 2
    S = 2
    masks = torch.from_numpy(rng.standard_normal((S, B * T, 2 * J)).astype(np.float32)).to(_tdt(torch, dtype))
    got = m.op_mask_scatter(torch.from_numpy(spec).cuda(), masks.cuda()).cpu().numpy()
    mk = masks.double().numpy().reshape(S, B, T, J, 2)
    sc = spec.astype(np.float64)[..., 0] + 1j * spec.astype(np.float64)[..., 1]  # [B, 2, F, T]
    mc = mk[..., 0] + 1j * mk[..., 1]  # [S, B, T, J]
    out = np.zeros((B, S, 2, 1025, T), np.complex128)
    for j in range(J):
        c, fr = fi[j] % 2, fi[j] // 2
        out[:, :, c, fr, :] += (sc[:, None, c, fr, :] * mc[:, :, :, j].transpose(1, 0, 2)) / nbpf[fr]
    ref = np.stack([out.real, out.imag], -1)
    assert np.abs(got - ref).max() <= 1e-5 * np.abs(ref).max()


@pytest.mark.parametrize("dtype", ["fp16", "bf16"])
def test_full_size_sweep_properties(torch_cuda, dtype):
    """The op sweep's largest shape (B = 8, D = 512): add then subtract returns
    the input (to one rounding), RMSNorm rows have RMS == gamma-weighted scale."""
    torch = torch_cuda
    import cudasep

    rows, D = 8 * T * NB, 512
    g = torch.Generator(device="cuda").manual_seed(11)
    x = torch.randn(rows, D, generator=g, device="cuda").to(_tdt(torch, dtype))
    y = torch.randn(rows, D, generator=g, device="cuda").to(_tdt(torch, dtype))
    s = cudasep.op_add(x, y)
    assert torch.isfinite(s.float()).all()
    back = cudasep.op_add(s, (-y).contiguous())
    tol = TOL[dtype] * 4
    assert ((back.float() - x.float()).abs() <= tol * (x.float().abs() + y.float().abs() + 1)).all()
    gamma = torch.ones(D, device="cuda")
    n = cudasep.op_rms_norm(x, gamma, 1.0)
    nrm = n.float().pow(2).sum(-1).sqrt()
    assert ((nrm - 1).abs() < 8 * TOL[dtype]).all()


def _attention_ref(q, k, v, scale, gates):
    """fp64 softmax attention + head merge, and sum_i p_i |v_i| / l (error scale)."""
    qd, kd, vd = (t.double().cpu().numpy() for t in (q, k, v))
    s = np.einsum("bhnd,bhmd->bhnm", qd, kd) * scale
    s -= s.max(-1, keepdims=True)
    p = np.exp(s)
    p /= p.sum(-1, keepdims=True)
    o = np.einsum("bhnm,bhmd->bhnd", p, vd)
    a = np.einsum("bhnm,bhmd->bhnd", p, np.abs(vd))
    if gates is not None:
        g = gates.double().cpu().numpy().transpose(0, 2, 1)[..., None]  # [B, H, N, 1]
        o, a = o * g, a * np.abs(g)
    B, H, N, D = o.shape
    merge = lambda t: t.transpose(0, 2, 1, 3).reshape(B, N, H * D)
    return merge(o), merge(a)


@pytest.mark.parametrize(
    "dtype,B,H,N,D,ramp,gated",
    [
        ("fp16", 2, 4, 1301, 64, 12.0, False),  # time path, 21 key blocks, 21-key tail, rescales
        ("fp16", 1, 2, 801, 64, 1e3 + 40.0, False),  # score step of ~2^288 mid-sequence (exp overflow, recompute)
        ("bf16", 1, 3, 801, 64, 12.0, True),  # the std chunk length
        ("fp16", 1, 2, 801, 64, -12.0, False),  # max in the first block (no rescale)
        ("fp16", 3, 3, 60, 64, 0.0, True),  # band axis: two sequences per tile, odd count
        ("bf16", 2, 2, 64, 64, 4.0, False),  # largest packed length
        ("fp16", 2, 2, 65, 64, 4.0, False),  # smallest blocked length
        ("fp16", 2, 2, 128, 64, 0.0, True),  # one full key block
        ("bf16", 1, 2, 1, 64, 0.0, False),  # a single token
        ("fp32", 1, 2, 300, 64, 6.0, True),  # CUDA-core path
        ("fp16", 1, 2, 300, 32, 6.0, False),  # head dim 32: CUDA-core path in 16 bits
    ],
)
def test_attention_op(torch_cuda, dtype, B, H, N, D, ramp, gated):
    """mbr_op_attention (scaled_dot_product_attention + apply_gates_and_merge_heads)
    against fp64 softmax attention of the same rounded inputs.  The key ramp
    makes the row max grow (or, negative, shrink) block by block so the
    tensor-core kernel's deferred rescaling of O runs.  Error bound per output:
    2u (sum p|v| / l + |ref|), u the unit roundoff of the 16-bit probabilities
    and outputs (one rounding each); fp32: 1e-5 of max |ref|."""
    torch = torch_cuda
    import cudasep

    g = torch.Generator().manual_seed(N * 7 + H)
    u = torch.randn(D, generator=g)
    u /= u.norm()
    q = torch.randn(B, H, N, D, generator=g) + min(abs(ramp), 1e3) * u
    pos = torch.linspace(0.0, 1.0, N)[:, None]
    if abs(ramp) > 1e3:  # step: the second half of the keys jumps by |ramp| - 1000 along u
        step = abs(ramp) - 1e3
        q = torch.randn(B, H, N, D, generator=g) + step * u
        k = torch.randn(B, H, N, D, generator=g) + step * (pos >= 0.5).float() * u
    else:
        k = torch.randn(B, H, N, D, generator=g) + np.sign(ramp) * abs(ramp) * pos * u
    v = torch.randn(B, H, N, D, generator=g)
    gates = torch.rand(B, N, H, generator=g) if gated else None
    tq, tk, tv = (t.to(_tdt(torch, dtype)) for t in (q, k, v))
    ref, amag = _attention_ref(tq, tk, tv, 1.0 / np.sqrt(D), gates)
    got = cudasep.op_attention(tq.cuda(), tk.cuda(), tv.cuda(), 0.0,
                               gates.cuda() if gated else None).double().cpu().numpy()
    assert got.shape == (B, N, H * D)
    err = np.abs(got - ref)
    if dtype == "fp32":
        assert err.max() <= 1e-5 * np.abs(ref).max(), f"max err {err.max():.3e}"
    else:
        u16 = {"fp16": 2.0 ** -11, "bf16": 2.0 ** -8}[dtype]
        bound = 2 * u16 * (amag + np.abs(ref)) + 1e-7
        worst = (err / bound).max()
        print(f"attention {dtype} B{B} H{H} N{N} D{D} ramp {ramp}: worst err/bound {worst:.3f}")
        assert worst <= 1.0


@pytest.mark.parametrize(
    "dtype,rows,fin,fout,act",
    [
        ("fp16", 48060, 384, 1536, 1),  # FFN1 of the std chunk (GELU)
        ("bf16", 3001, 1536, 384, 0),  # FFN2 shape, ragged rows
        ("fp16", 801, 384, 1536, 2),  # mask-estimator hidden layer (tanh)
        ("bf16", 1000, 384, 1536, 0),
        ("fp16", 130, 64, 200, 1),  # one K block, ragged N (200 = 192 + 8)
        ("fp16", 77, 100, 60, 0),  # K not a multiple of 16: CUDA-core path
        ("fp32", 500, 384, 96, 1),  # fp32: CUDA-core path
    ],
)
def test_linear_op(torch_cuda, dtype, rows, fin, fout, act):
    """mbr_op_linear (linear / linear_gelu / tanh) against fp64 math on the same
    rounded operands: one rounding of the output (TOL) plus the fp32
    accumulation (K * 2^-23 of sum |x w|)."""
    torch = torch_cuda
    import cudasep

    g = torch.Generator().manual_seed(rows + fin + fout)
    x = torch.randn(rows, fin, generator=g).to(_tdt(torch, dtype))
    w = (torch.randn(fout, fin, generator=g) * (1.0 / np.sqrt(fin))).to(_tdt(torch, dtype))
    b = torch.randn(fout, generator=g) * 0.1
    got = cudasep.op_linear(x.cuda(), w.cuda(), b.cuda(), act).double().cpu().numpy()
    xd, wd = x.double().numpy(), w.double().numpy()
    pre = xd @ wd.T + b.double().numpy()
    if act == 1:

        ref = gelu_ref(pre)
    elif act == 2:
        ref = np.tanh(pre)
    else:
        ref = pre
    acc = fin * 2.0 ** -23 * (np.abs(xd) @ np.abs(wd).T)
    bound = TOL[dtype] * np.maximum(np.abs(ref), 1e-3) * 1.01 + acc + 1e-6
    err = np.abs(got - ref)
    assert np.all(err <= bound), f"linear {dtype} {rows}x{fin}x{fout} act {act}: max err/bound {(err / bound).max():.3f}"


@pytest.mark.parametrize("dtype,L", [("bf16", 1301), ("bf16", 60), ("fp16", 1301), ("fp16", 60)])
def test_attention_matches_reference_validators(torch_cuda, dtype, L):
    """mbr_op_attention on the reference's own validator inputs (the time-axis
    tcgen05 kernel at L = 1301, the packed band-axis kernel at L = 60) against
    the restated validators: within 2 bf16 ulps (both round probabilities and
    outputs to 16 bits, in different places)."""
    torch = torch_cuda
    import attn_validators as av
    import cudasep

    x = av.inputs(L)
    t = torch.from_numpy(x).to(_tdt(torch, dtype))[None, None].cuda()
    got = cudasep.op_attention(t, t, t, 0.125).float().cpu().numpy()[0]
    if L > 64:
        ref = av.time_rows(x)
        err = max(av.err_ulps(got[r], ref[r]) for r in ref)
    else:
        err = av.err_ulps(got, av.band_rows(x))
    print(f"attention {dtype} L={L} vs the reference validator: {err:.2f} bf16 ulps")
    assert err <= 2.0, err

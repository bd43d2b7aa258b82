"""The DiT block's linear layers on the tcgen05 GEMM (fvsr_linear, fvsr_linear_qkv) against an fp32 reference.

Reference (MLX's Linear, DiT.swift:318-381): y = x·Wᵀ + b accumulated in fp32 and rounded to bf16 once; the epilogues
keep the reference's rounding points — GELU(tanh) of the rounded Linear, rounded; the gated residual
round(resid + round(gate · linear)). The GEMM's fp32 summation order differs from torch's, so an element may land
one bf16 rounding step away: the bar is |Δ| ≤ 2⁻⁷·|ref| + 1e-3·max|ref| per element (two bf16 ulps) and rel ≤ 1e-2.
Shapes cover one half tile (M = 128), a last half tile (M = 384, 17280: rows loaded as zeros past M, not written),
fewer tiles than SMs, several tiles per SM, and K = 8960 (the FFN's second layer)."""
from __future__ import annotations

import pytest

torch = pytest.importorskip("torch")
pytestmark = pytest.mark.gpu


@pytest.fixture(scope="module")
def gpu(fvsr):
    if not torch.cuda.is_available():
        pytest.skip("no CUDA device")
    return fvsr


def _data(m, n, k, seed):
    g = torch.Generator(device="cuda").manual_seed(seed)
    x = torch.randn((m, k), generator=g, device="cuda").to(torch.bfloat16)
    w = (torch.randn((n, k), generator=g, device="cuda") / k ** 0.5).to(torch.bfloat16)
    b = (0.1 * torch.randn((n,), generator=g, device="cuda")).to(torch.bfloat16)
    return x, w, b


def _lin(x, w, b):
    y = x.float() @ w.float().t()
    if b is not None:
        y = y + b.float()
    return y.to(torch.bfloat16)


def _close(got, ref):
    g, r = got.float(), ref.float()
    d = (g - r).abs()
    assert (d <= 2.0 ** -7 * r.abs() + 1e-3 * r.abs().max()).all(), float(d.max())
    assert float(d.max() / r.abs().max()) <= 1e-2


@pytest.mark.parametrize("m,n,k", [(128, 256, 64), (384, 512, 128), (1024, 1536, 1536), (2048, 4608, 1536),
                                   (256, 1536, 8960), (4096, 8960, 1536), (17280, 1536, 1536)])
def test_linear_matches_fp32_reference(gpu, m, n, k):
    x, w, b = _data(m, n, k, m + n + k)
    got = gpu.linear(x, w, b)
    torch.cuda.synchronize()
    _close(got, _lin(x, w, b))
    _close(gpu.linear(x, w, None), _lin(x, w, None))
    gpu.device_check()


def test_linear_gelu_and_gated_residual(gpu):
    """The epilogues from the kernel's own Linear output (itself checked against fp32 above): the gated residual
    round(resid + round(gate · linear)) exactly; GELU(tanh) within one bf16 step (CUDA's tanhf against torch's)."""
    m, n, k = 1024, 1536, 1536
    x, w, b = _data(m, n, k, 5)
    lin = gpu.linear(x, w, b)
    got = gpu.linear(x, w, b, epilogue=gpu.FVSR_LINEAR_GELU)
    ref = torch.nn.functional.gelu(lin.float(), approximate="tanh").to(torch.bfloat16)
    g = torch.Generator(device="cuda").manual_seed(6)
    gate = (0.5 * torch.randn((n,), generator=g, device="cuda")).to(torch.bfloat16)
    resid = torch.randn((m, n), generator=g, device="cuda").to(torch.bfloat16)
    got2 = gpu.linear(x, w, b, epilogue=gpu.FVSR_LINEAR_GATED_RESIDUAL, gate=gate, resid=resid)
    ref2 = (resid.float() + (gate.float() * lin.float()).to(torch.bfloat16).float()).to(torch.bfloat16)
    torch.cuda.synchronize()
    d = (got.float() - ref.float()).abs()
    assert (d <= 2.0 ** -8 * ref.float().abs() + 1e-6).all(), float(d.max())
    assert float((d == 0).float().mean()) > 0.99
    assert torch.equal(got2, ref2)
    _close(lin, _lin(x, w, b))
    # in place: the residual stream is both the input and the output (tok = tok + gate · f(x))
    tok = resid.clone()
    gpu.linear(x, w, b, epilogue=gpu.FVSR_LINEAR_GATED_RESIDUAL, gate=gate, resid=tok, out=tok)
    torch.cuda.synchronize()
    assert torch.equal(tok, got2)
    gpu.device_check()


def test_linear_qkv_equals_three_linears(gpu):
    m, n, k = 2048, 1536, 1536
    x, w, b = _data(m, 3 * n, k, 7)
    q, kk, v = gpu.linear_qkv(x, w, b)
    for i, got in enumerate((q, kk, v)):
        want = gpu.linear(x, w[i * n:(i + 1) * n].contiguous(), b[i * n:(i + 1) * n].contiguous())
        torch.cuda.synchronize()
        assert torch.equal(got, want), i
    gpu.device_check()

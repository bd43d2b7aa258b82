"""The DiT block's other ops against torch references with the reference's rounding points: LayerNorm (+ modulation,
+ affine), WanRMSNorm, and the cross-attention (every key of the cached context; the tcgen05 attention kernel with no
lists). Statistics are taken in float64 in the reference; the kernels' fp32 sums in another order may move an element
by one bf16 step, so the norms' bar is one bf16 step per element (and ≥ 99 % exact); the attention's is the bf16 bar
of the path, rel ≤ 1e-2 (max |Δ| / max |ref|)."""
from __future__ import annotations

import math

import pytest

torch = pytest.importorskip("torch")
pytestmark = pytest.mark.gpu


@pytest.fixture(scope="module")
def gpu(fvsr):
    if not torch.cuda.is_available():
        pytest.skip("no CUDA device")
    return fvsr


def _bf(x):
    return x.to(torch.bfloat16).double()


def _one_step(got, ref, terms=None):
    """One bf16 step of the larger value per element; `terms` (the magnitudes that cancel in an affine n·w + b) add
    the fp32 floor 2⁻²⁰·terms, since an fp32 n carries ~1e-7 of error that a cancellation to ~0 makes large."""
    g, r = got.double(), ref.double()
    d = (g - r).abs()
    floor = 1e-30 if terms is None else 2.0 ** -20 * terms
    assert (d <= 2.0 ** -7 * torch.maximum(g.abs(), r.abs()) + floor).all(), float(d.max())
    assert float((d == 0).double().mean()) > 0.99


@pytest.mark.parametrize("c", [256, 1536, 2048])
def test_layernorm_modulated_and_affine(gpu, c):
    g = torch.Generator(device="cuda").manual_seed(c)
    m, eps = 777, 1e-6
    x = (1.5 * torch.randn((m, c), generator=g, device="cuda") + 0.3).to(torch.bfloat16)
    shift, scale, w, b = ((0.3 * torch.randn((c,), generator=g, device="cuda")).to(torch.bfloat16) for _ in range(4))
    xd = x.double()
    mean = xd.mean(dim=1, keepdim=True)
    var = ((xd - mean) ** 2).mean(dim=1, keepdim=True)
    n = (xd - mean) / torch.sqrt(var + eps)
    got = gpu.layernorm(x, shift=shift, scale=scale, eps=eps)
    ref = _bf(_bf(_bf(n) * _bf(1.0 + scale.double())) + shift.double())
    got_aff = gpu.layernorm(x, weight=w, bias=b, eps=eps)
    ref_aff = _bf(n * w.double() + b.double())
    got_plain = gpu.layernorm(x, eps=eps)
    torch.cuda.synchronize()
    _one_step(got_plain, _bf(n))
    _one_step(got_aff, ref_aff, terms=(n * w.double()).abs() + b.double().abs())
    # the modulation chain re-rounds after each op: compare it from the kernel's own rounded n
    ref_from = _bf(_bf(got_plain.double() * _bf(1.0 + scale.double())) + shift.double())
    assert torch.equal(got.double(), ref_from)
    terms = (_bf(n) * _bf(1.0 + scale.double())).abs() + shift.double().abs()
    d = (got.double() - ref).abs()   # the fp64 chain: n's one step, carried through the cancellation with shift
    assert (d <= 2.0 ** -6 * torch.maximum(got.double().abs(), ref.abs()) + 2.0 ** -8 * terms).all(), float(d.max())
    gpu.device_check()


def test_rmsnorm(gpu):
    g = torch.Generator(device="cuda").manual_seed(3)
    m, c, eps = 500, 1536, 1e-6
    x = torch.randn((m, c), generator=g, device="cuda").to(torch.bfloat16)
    w = (1.0 + 0.1 * torch.randn((c,), generator=g, device="cuda")).to(torch.bfloat16)
    xd = x.double()
    inv = 1.0 / torch.sqrt((xd * xd).mean(dim=1, keepdim=True) + eps)
    ref = _bf(_bf(xd * inv) * w.double())
    got = gpu.rmsnorm(x, w, eps=eps)
    torch.cuda.synchronize()
    _one_step(got, ref)


@pytest.mark.parametrize("lq,lk", [(1024, 512), (384, 128), (17280, 512)])
def test_cross_attention_matches_sdpa(gpu, lq, lk):
    heads = 12
    g = torch.Generator(device="cuda").manual_seed(lq + lk)
    q, k, v = (torch.randn((n, heads * 128), generator=g, device="cuda").to(torch.bfloat16) for n in (lq, lk, lk))
    got = gpu.cross_attention(q, k, v, heads)
    qh, kh, vh = (t.float().view(-1, heads, 128).transpose(0, 1) for t in (q, k, v))
    ref = torch.nn.functional.scaled_dot_product_attention(qh, kh, vh, scale=1 / math.sqrt(128))
    ref = ref.transpose(0, 1).reshape(lq, heads * 128)
    torch.cuda.synchronize()
    rel = float((got.float() - ref).abs().max() / ref.abs().max())
    assert rel <= 1e-2, rel
    gpu.device_check()

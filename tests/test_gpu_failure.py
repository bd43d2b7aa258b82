"""The failure path of the device-side waits, exercised without a fault: a bounded wait that nothing completes gives
up after its limit, the kernel returns, fvsr_device_check reports FVSR_ETIMEOUT once, and the context keeps working."""
from __future__ import annotations

import time

import pytest

torch = pytest.importorskip("torch")
pytestmark = pytest.mark.gpu


def test_bounded_wait_runs_out_and_is_reported(fvsr):
    if not torch.cuda.is_available():
        pytest.skip("no CUDA device")
    fvsr.device_check()                       # clean before
    t0 = time.monotonic()
    fvsr.wait_probe(20_000)                   # 20 ms on a barrier that nothing completes
    with pytest.raises(fvsr.FVSRError) as e:
        fvsr.device_check()
    assert e.value.status == fvsr.FVSR_ETIMEOUT
    assert time.monotonic() - t0 < 10.0       # the wait gave up; nothing hung
    fvsr.device_check()                       # reported once, then cleared
    # the context is usable: a small selection + attention afterwards
    g = fvsr.Geometry(heads=2, bh=2, bw=3, q_slices=1, kv_slices=2, local_range=3, dtype=fvsr.FVSR_BF16)
    g.topk = int(round(0.5 * g.allowed_per_row()))
    gen = torch.Generator(device="cuda").manual_seed(3)
    q, k, v = (torch.randn((n * 128, g.channels), generator=gen, device="cuda").to(torch.bfloat16)
               for n in (g.nq, g.nk, g.nk))
    sel = fvsr.draft_block_mask_and_probs(q, k, g, want_probs=False, want_mask=False)
    out = fvsr.block_sparse_attention(q, k, v, sel["kidx"], sel["kcnt"], g)
    torch.cuda.synchronize()
    assert torch.isfinite(out.float()).all()
    fvsr.device_check()

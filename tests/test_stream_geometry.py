"""The streaming driver's chunk geometry (host only, no GPU): the reference's chunk schedule (Pipeline.swift:95-102),
RoPE start, topk rule (DiT.swift:482) and default top-k ratio (Pipeline.swift:68)."""
from __future__ import annotations

import pytest


@pytest.mark.parametrize("out_h,out_w", [(1152, 1920), (768, 1280), (1536, 2560), (256, 384)])
def test_chunk_geometry_follows_the_reference_schedule(fvsr, out_h, out_w):
    bh, bw = out_h // 128, out_w // 128
    s = bh * bw
    ratio = 2.0 * 768 * 1280 / float(out_h * out_w)
    for k in range(6):
        g, b, e = fvsr.chunk_geometry(k, 12, out_h, out_w)
        want_b, want_e = (0, 6) if k == 0 else (4 + 2 * k, 6 + 2 * k)   # sch.latents; t0 = its lower bound
        assert (b, e) == (want_b, want_e)
        assert g.q_slices == (e - b) // 2 and (g.bh, g.bw) == (bh, bw)
        assert g.topk == int(float(s * s) * ratio) - 1
        assert g.local_range == 11 and g.heads == 12


def test_chunk_geometry_explicit_ratio_and_range(fvsr):
    g, _, _ = fvsr.chunk_geometry(1, 2, 256, 384, topk_ratio=0.25, local_range=5)
    assert g.topk == int(36 * 0.25) - 1 and g.local_range == 5 and g.heads == 2


@pytest.mark.parametrize("args,status", [
    (dict(heads=12, out_h=1000, out_w=1920), 1),    # not a multiple of 128
    (dict(heads=17, out_h=1152, out_w=1920), 1),    # beyond the token-order path's 16 heads
    (dict(heads=12, out_h=1152, out_w=1920, local_range=0), 1),
    (dict(heads=12, out_h=1152, out_w=1920, topk_ratio=1e-9), 1),   # top-k below 0
    (dict(heads=12, out_h=1152, out_w=1920, k=600), 5),  # temporal positions past the table end
])
def test_chunk_geometry_rejects_bad_arguments(fvsr, args, status):
    kw = dict(args)
    k = kw.pop("k", 0)
    with pytest.raises(fvsr.FVSRError) as e:
        fvsr.chunk_geometry(k, **kw)
    assert e.value.status == status

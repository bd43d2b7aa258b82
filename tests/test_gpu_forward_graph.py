"""fvsr_lcsa_forward (DiT.swift:504-538) captured into a CUDA graph and replayed, against the same call made eagerly
on an identical cache: the bf16 path copies the appended slice into the cache on the cache's side stream while the
selection and the attention run (the attention reading the new blocks from k_new / v_new), so the capture has to take
the fork and the join along. Outputs, selections and the cache contents after the call must be bit-identical."""
from __future__ import annotations

import pytest

torch = pytest.importorskip("torch")
pytestmark = pytest.mark.gpu


@pytest.fixture(scope="module")
def dev(fvsr):
    if not torch.cuda.is_available():
        pytest.skip("no CUDA device")
    return "cuda"


@pytest.mark.parametrize("q_slices", [1, 2])
def test_forward_in_a_graph_equals_eager(fvsr, dev, q_slices):
    heads, bh, bw, kv_len = 2, 6, 10, 2
    g = fvsr.Geometry(heads=heads, bh=bh, bw=bw, q_slices=q_slices, kv_slices=kv_len + q_slices, local_range=11,
                      dtype=fvsr.FVSR_BF16)
    g.topk = int(round(0.5 * g.allowed_per_row()))
    gen = torch.Generator(device="cuda").manual_seed(31 + q_slices)
    srows, c = g.s * 128, heads * 128

    def rnd(rows):
        return torch.randn((rows, c), generator=gen, device="cuda").to(torch.bfloat16)

    prefill = [(rnd(srows), rnd(srows)) for _ in range(kv_len)]
    caches = []
    for _ in range(2):
        cache = fvsr.KVCache(g, kv_len=kv_len, max_new_slices=q_slices)
        for k, v in prefill:
            cache.append(k, v, 1)
        caches.append(cache)
    q, kn, vn = rnd(q_slices * srows), rnd(q_slices * srows), rnd(q_slices * srows)
    outs = [torch.empty_like(q) for _ in range(2)]
    kidx = [torch.empty((heads, g.nq, g.nk), dtype=torch.int32, device="cuda") for _ in range(2)]
    kcnt = [torch.empty((heads, g.nq), dtype=torch.int32, device="cuda") for _ in range(2)]
    ws = [fvsr.make_workspace(g) for _ in range(2)]
    torch.cuda.synchronize()

    fvsr.lcsa_forward(q, kn, vn, caches[0], g, out=outs[0], kidx=kidx[0], kcnt=kcnt[0], workspace=ws[0])
    stream = torch.cuda.Stream()
    graph = torch.cuda.CUDAGraph()
    with torch.cuda.graph(graph, stream=stream):
        fvsr.lcsa_forward(q, kn, vn, caches[1], g, out=outs[1], kidx=kidx[1], kcnt=kcnt[1], workspace=ws[1],
                          stream=torch.cuda.current_stream())
    graph.replay()
    torch.cuda.synchronize()
    assert torch.equal(kidx[0], kidx[1]) and torch.equal(kcnt[0], kcnt[1])
    assert torch.equal(outs[0], outs[1])
    assert caches[0].state() == caches[1].state()
    k0, v0 = caches[0].gather()
    k1, v1 = caches[1].gather()
    torch.cuda.synchronize()
    assert torch.equal(k0, k1) and torch.equal(v0, v1)
    # the appended slice is in the cache (the newest kv_len slices: the prefill's last ones, then the new ones)
    assert torch.equal(k0[-q_slices * srows:], kn) and torch.equal(v0[-q_slices * srows:], vn)
    graph.reset()
    del graph
    for cch in caches:
        cch.close()
    fvsr.device_check()

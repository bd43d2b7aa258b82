"""GPU parity of the token-order side of the path, through the C ABI:

- fvsr_lcsa_prepare (WanRMSNorm DiT.swift:34-47, ropeApply 100-107, windowPartition 113-118, pooled q/k 161-162)
  against the oracle's restatement (orc_prepare, orc_pool): bit-exact, both storage types, every head-count
  instantiation;
- fvsr_lcsa_forward_tokens (DiT.swift:499-539 between the linear layers) against the window-order path it fuses —
  prepare, fvsr_lcsa_forward, windowReverse — bit-exact over a streaming sequence of chunks, and its first chunk
  against the oracle (selection exact, attention within the path's tolerance)."""
from __future__ import annotations

import numpy as np
import pytest

torch = pytest.importorskip("torch")
pytestmark = pytest.mark.gpu

REL_F32 = 1e-5
REL_BF16 = 1e-2


@pytest.fixture(scope="module")
def dev(fvsr):
    if not torch.cuda.is_available():
        pytest.skip("no CUDA device")
    return "cuda"


def bits(t):
    """Tensor → numpy in the oracle's convention (fp32, or bf16 as uint16 bit patterns)."""
    t = t.contiguous().cpu()
    return t.view(torch.int16).numpy().view(np.uint16) if t.dtype == torch.bfloat16 else t.numpy()


def token_rows(bh, bw, nq):
    """Token-order row of each window-order row (window w, token r) — windowReverse's permutation."""
    w = np.arange(nq)[:, None]
    r = np.arange(128)[None, :]
    s = bh * bw
    nf, rem = w // s, w % s
    nh, nw = rem // bw, rem % bw
    wf, wh, ww = r >> 6, (r >> 3) & 7, r & 7
    return (((2 * nf + wf) * (8 * bh) + 8 * nh + wh) * (8 * bw) + 8 * nw + ww).reshape(-1)


def linear_outputs(g, dtype, seed):
    gen = torch.Generator(device="cuda").manual_seed(seed)
    t = torch.bfloat16 if dtype == "bf16" else torch.float32
    L, C = g.nq * 128, g.channels
    q, k, v = (torch.randn((L, C), generator=gen, device="cuda").mul_(2.0).to(t) for _ in range(3))
    wq, wk = ((1.0 + 0.1 * torch.randn((C,), generator=gen, device="cuda")).to(t) for _ in range(2))
    return q, k, v, wq, wk


@pytest.mark.parametrize("dtype,heads,bh,bw,q_slices,norm,rope", [
    ("bf16", 12, 3, 5, 1, True, True),
    ("f32", 3, 2, 3, 2, True, True),
    ("bf16", 5, 2, 2, 1, True, False),
    ("bf16", 16, 2, 2, 1, False, True),
    ("bf16", 2, 3, 2, 2, False, False),
    ("f32", 8, 2, 2, 1, True, True),
    ("f32", 16, 2, 2, 1, True, True),     # the 16-head fp32 instantiation
    ("bf16", 12, 2, 3, 3, True, True),    # a chunk-0 shape: three temporal slices
])
def test_prepare_matches_oracle(fvsr, orc, dev, dtype, heads, bh, bw, q_slices, norm, rope):
    g = fvsr.Geometry(heads=heads, bh=bh, bw=bw, q_slices=q_slices, kv_slices=q_slices, local_range=11,
                      dtype=fvsr.FVSR_BF16 if dtype == "bf16" else fvsr.FVSR_F32)
    f, h, w = 2 * q_slices, 8 * bh, 8 * bw
    q, k, v, wq, wk = linear_outputs(g, dtype, 100 + heads)
    tabs = fvsr.rope_tables(f, h, w, t0=4) if rope else None
    res = fvsr.lcsa_prepare(q, k, v, g, norm_q=wq if norm else None, norm_k=wk if norm else None, eps=1e-6,
                            rope=tabs)
    torch.cuda.synchronize()
    cos, sin = (bits(tabs[0]), bits(tabs[1])) if rope else (None, None)
    for name, x, wt in (("q", q, wq), ("k", k, wk)):
        want = orc.prepare(bits(x), f, h, w, heads, weight=bits(wt) if norm else None, eps=1e-6, cos=cos, sin=sin)
        got = bits(res[name])
        assert np.array_equal(got, want), f"{name}: {(got != want).sum()} of {got.size} differ"
        assert np.array_equal(bits(res["pooled_" + name]), orc.pool(want)), f"pooled {name}"
    assert np.array_equal(bits(res["v"]), orc.prepare(bits(v), f, h, w, heads))
    fvsr.device_check()


@pytest.mark.parametrize("dtype", ["bf16", "f32"])
def test_forward_tokens_equals_the_window_path(fvsr, orc, dev, dtype):
    """Three streaming chunks (2, 1, 1 slices; kvLen 2): the fused token-order layer against prepare → window-order
    forward → windowReverse, each with its own cache — outputs and selections bit-identical; chunk 0 against the
    oracle."""
    heads, bh, bw = 2, 3, 5
    dt = fvsr.FVSR_BF16 if dtype == "bf16" else fvsr.FVSR_F32
    g0 = fvsr.Geometry(heads=heads, bh=bh, bw=bw, q_slices=2, kv_slices=2, local_range=11, dtype=dt)
    cache_a = fvsr.KVCache(g0, kv_len=2, max_new_slices=2)
    cache_b = fvsr.KVCache(g0, kv_len=2, max_new_slices=2)
    s = g0.s
    for chunk, qs in enumerate((2, 1, 1)):
        kv_total = min(cache_a.slices + qs, 4)
        g = fvsr.Geometry(**{**g0.__dict__, "q_slices": qs})
        gfull = fvsr.Geometry(**{**g.__dict__, "kv_slices": kv_total})
        g.topk = gfull.topk = int(round(0.5 * gfull.allowed_per_row()))
        q, k, v, wq, wk = linear_outputs(g, dtype, 500 + chunk)
        tabs = fvsr.rope_tables(2 * qs, 8 * bh, 8 * bw, t0=4 + 2 * chunk)
        kidx_a = torch.empty((heads, gfull.nq, gfull.nk), dtype=torch.int32, device="cuda")
        kcnt_a = torch.empty((heads, gfull.nq), dtype=torch.int32, device="cuda")
        kidx_b, kcnt_b = torch.empty_like(kidx_a), torch.empty_like(kcnt_a)
        q_win = torch.empty_like(q)
        out_a = fvsr.lcsa_forward_tokens(q, k, v, cache_a, g, norm_q=wq, norm_k=wk, eps=1e-6, rope=tabs, q_win=q_win,
                                         kidx=kidx_a, kcnt=kcnt_a)
        pre = fvsr.lcsa_prepare(q, k, v, g, norm_q=wq, norm_k=wk, eps=1e-6, rope=tabs, pooled=False)
        out_b = fvsr.lcsa_forward(pre["q"], pre["k"], pre["v"], cache_b, g, kidx=kidx_b, kcnt=kcnt_b)
        torch.cuda.synchronize()
        assert torch.equal(q_win, pre["q"])
        assert torch.equal(kidx_a, kidx_b) and torch.equal(kcnt_a, kcnt_b), f"chunk {chunk}: selection differs"
        rev = torch.empty_like(out_b)
        rev[torch.from_numpy(token_rows(bh, bw, g.nq)).to("cuda")] = out_b
        assert torch.equal(out_a, rev), f"chunk {chunk}: outputs differ"
        assert cache_a.state() == cache_b.state()
        if chunk == 0:
            qw, kw, vw = (bits(pre[n]).astype(np.float32) if dtype == "f32" else
                          orc.bf16_bits_to_f32(bits(pre[n])) for n in ("q", "k", "v"))
            loc = orc.local_block_mask(bh, bw, 11)
            _, _, okidx, okcnt = orc.draft_block_mask_and_probs(qw, kw, heads, qs, s, loc, g.topk)
            assert np.array_equal(kidx_a.cpu().numpy(), okidx)
            ref = orc.window_reverse(orc.attention(qw, kw, vw, okidx, okcnt, heads), 1, 2 * qs, 8 * bh, 8 * bw)
            cmp = orc.compare(out_a.float().cpu().numpy(), ref.reshape(out_a.shape))
            assert cmp["rel"] <= (REL_BF16 if dtype == "bf16" else REL_F32), cmp
    cache_a.close()
    cache_b.close()
    fvsr.device_check()


@pytest.mark.parametrize("kv_ratio", [3.0, 1.0])
def test_stream_driver_equals_manual_layers(fvsr, dev, kv_ratio):
    """The C++ chunk driver (fvsr_stream_*) over three chunks and two blocks against the same layers called by hand:
    the reference's schedule (chunk 0: 3 slices, then 1; t0 = 0, then 4 + 2k), its RoPE tables (checked against
    rope_tables), topk and kvLen, one cache per block — outputs bit-identical."""
    heads, out_h, out_w, layers = 2, 256, 384, 2
    st = fvsr.Stream(heads, out_h, out_w, layers, kv_ratio=kv_ratio)
    st.begin()
    kv_len = int(kv_ratio)
    held = 0
    caches = [fvsr.KVCache(st.geometry(0)[0], kv_len=kv_len, max_new_slices=3) for _ in range(layers)]
    for chunk in range(3):
        g, t0, t1 = st.geometry(chunk)
        st.start_chunk(chunk)
        cos, sin = st.rope()
        ref_cos, ref_sin = fvsr.rope_tables(t1 - t0, out_h // 16, out_w // 16, t0=t0)
        assert (cos - ref_cos).abs().max().item() <= 1e-7 and (sin - ref_sin).abs().max().item() <= 1e-7
        for i in range(layers):
            q, k, v, wq, wk = linear_outputs(g, "bf16", 900 + 10 * chunk + i)
            got = st.layer(i, q, k, v, norm_q=wq, norm_k=wk, eps=1e-6)
            want = fvsr.lcsa_forward_tokens(q, k, v, caches[i], g, norm_q=wq, norm_k=wk, eps=1e-6, rope=(cos, sin))
            torch.cuda.synchronize()
            assert torch.equal(got, want), f"chunk {chunk} layer {i}"
        # DiT.swift:532-538: after a chunk, drop the oldest slice once if more than kvLen are held
        held = (0 if chunk == 0 else held) + g.q_slices
        held -= 1 if held > kv_len else 0
        assert all(c.slices == held for c in caches)
    for c in caches:
        c.close()
    st.close()
    fvsr.device_check()

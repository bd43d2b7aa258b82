"""GPU parity of the sm_100a LCSA path against the CPU oracle, through the C ABI (ctypes → libfvsr_lcsa.so).

Bars (from the path's specification): selection — block mask, block probabilities, kidx and kcnt bit-exact against the
oracle's fixed-order fp32 restatement of DiT.swift:158-174; attention — relative error (max |Δ| / max |ref|, the
measure of Sources/Smoke/Gates.swift:19-29) ≤ 1e-5 for fp32 and ≤ 1e-2 for bf16 against the reference computed in
fp32 (the oracle, itself pinned to the reference's own oracle/block_sparse_attn.py by tests/golden)."""
from __future__ import annotations

import importlib
from pathlib import Path

import numpy as np
import pytest

torch = pytest.importorskip("torch")
pytestmark = pytest.mark.gpu

GOLDEN = Path(__file__).resolve().parent / "golden"
REL_F32 = 1e-5
REL_BF16 = 1e-2


@pytest.fixture(scope="module")
def cfgs(fvsr):
    if not torch.cuda.is_available():
        pytest.skip("no CUDA device")
    return importlib.import_module("fvsr_b200.configs")


def npf(t):
    return t.float().cpu().numpy()


def sample_items(heads, nq, n, seed):
    rng = np.random.default_rng(seed)
    return np.sort(rng.choice(heads * nq, size=min(n, heads * nq), replace=False)).astype(np.int32)


def rows_of(items, nq):
    sl = []
    for w in items:
        h, qb = divmod(int(w), nq)
        sl.append((slice(qb * 128, qb * 128 + 128), slice(h * 128, h * 128 + 128)))
    return sl


def gather_rows(x, items, nq):
    return np.concatenate([x[s] for s in rows_of(items, nq)], axis=0)


# ------------------------------------------------------------------------------------------------------------------
# pooling
# ------------------------------------------------------------------------------------------------------------------
@pytest.mark.parametrize("dtype,heads", [("bf16", 12), ("f32", 12), ("bf16", 2), ("bf16", 1), ("f32", 2), ("bf16", 5)])
def test_pool_bit_exact(fvsr, orc, cfgs, dtype, heads):
    """12 heads: 512-channel CTAs; 1, 2 heads: several blocks per CTA (a sharded rank's Q/K); 5: a partial CTA."""
    g = fvsr.Geometry(heads=heads, bh=1, bw=1, q_slices=1, kv_slices=1,
                      dtype=fvsr.FVSR_BF16 if dtype == "bf16" else fvsr.FVSR_F32)
    gen = torch.Generator(device="cuda").manual_seed(7)
    x = torch.randn((37 * 128, heads * 128), generator=gen, device="cuda")
    if dtype == "bf16":
        x = x.to(torch.bfloat16)
    got = fvsr.pool(x, g).cpu().numpy()
    want = orc.pool(npf(x))
    assert np.array_equal(got.view(np.uint32), want.view(np.uint32))


# ------------------------------------------------------------------------------------------------------------------
# selection (draftBlockMaskAndProbs) — bit-exact at every config's full size
# ------------------------------------------------------------------------------------------------------------------
SELECT_CASES = [(1, 0, None), (2, 0, None), (3, 0, None), (5, 0, None), (4, 0, 3)]


@pytest.mark.parametrize("cfg_id,layer,qs", SELECT_CASES, ids=[f"config{c}" + ("_chunk0" if q else "") for c, _, q in SELECT_CASES])
def test_select_bit_exact(fvsr, orc, cfgs, cfg_id, layer, qs):
    cfg = cfgs.CONFIGS[cfg_id]
    g = cfg.geometry(q_slices=qs)
    q, k, _ = cfgs.synth_qkv(cfg, g, cfgs.seed_of(cfg_id, 0, layer))
    r = fvsr.draft_block_mask_and_probs(q, k, g)
    torch.cuda.synchronize()
    loc = orc.local_block_mask(g.bh, g.bw, g.local_range)
    probs, mask, kidx, kcnt = orc.draft_block_mask_and_probs(npf(q), npf(k), g.heads, g.q_slices, g.s, loc, g.topk)
    gp = r["probs"].cpu().numpy()
    assert np.array_equal(gp.view(np.uint32), probs.view(np.uint32)), "block probabilities differ"
    assert np.array_equal(r["mask"].cpu().numpy().astype(bool), mask), "block mask differs"
    assert np.array_equal(r["kcnt"].cpu().numpy(), kcnt)
    assert np.array_equal(r["kidx"].cpu().numpy(), kidx)
    # size-independent properties: kept pairs are locality-allowed, counts add up to topk per (head, slice) row
    assert not (mask & ~np.tile(loc, (g.nq // g.s, g.nk // g.s))[None]).any()
    assert int(kcnt.sum()) == g.topk * g.heads * g.q_slices


def test_select_with_pooled_keys_matches(fvsr, orc, cfgs):
    cfg = cfgs.CONFIGS[2]
    g = cfg.geometry()
    q, k, _ = cfgs.synth_qkv(cfg, g, 77)
    pk = fvsr.pool(k, g)
    a = fvsr.draft_block_mask_and_probs(q, k, g)
    b = fvsr.draft_block_mask_and_probs(q, None, g, pooled_k=pk)
    for key in ("mask", "kidx", "kcnt"):
        assert torch.equal(a[key], b[key])


def test_select_topk_edge_cases(fvsr, orc, cfgs):
    """topk = 0 keeps only entries above the row maximum (none); topk ≥ n − 1 keeps all but the row minimum."""
    cfg = cfgs.CONFIGS[2]
    for topk in (0, 10 ** 7):
        g = cfg.geometry()
        g.topk = topk
        q, k, _ = cfgs.synth_qkv(cfg, g, 5)
        r = fvsr.draft_block_mask_and_probs(q, k, g)
        loc = orc.local_block_mask(g.bh, g.bw, g.local_range)
        _, mask, kidx, kcnt = orc.draft_block_mask_and_probs(npf(q), npf(k), g.heads, 1, g.s, loc, topk)
        assert np.array_equal(r["mask"].cpu().numpy().astype(bool), mask)
        assert np.array_equal(r["kcnt"].cpu().numpy(), kcnt)


@pytest.mark.parametrize("kv_slices", [12, 32], ids=["nk960", "nk2560_max"])
def test_long_key_rows_select_and_attend(fvsr, orc, cfgs, kv_slices):
    """Key rows longer than any config's: 960 key blocks (the softmax's four-chunk register path) and the supported
    maximum of 2560 (its streaming path) — selection bit-exact, bf16 attention on sampled items within the bf16 bar;
    one more slice is refused before any launch."""
    g = fvsr.Geometry(heads=2, bh=8, bw=10, q_slices=1, kv_slices=kv_slices, local_range=11, topk=0,
                      dtype=fvsr.FVSR_BF16)
    g.topk = int(0.25 * g.allowed_per_row())
    gen = torch.Generator(device="cuda").manual_seed(100 + kv_slices)
    q = torch.randn((g.nq * 128, g.channels), generator=gen, device="cuda").to(torch.bfloat16)
    k = torch.randn((g.nk * 128, g.channels), generator=gen, device="cuda").to(torch.bfloat16)
    v = torch.randn((g.nk * 128, g.channels), generator=gen, device="cuda").to(torch.bfloat16)
    r = fvsr.draft_block_mask_and_probs(q, k, g)
    out = fvsr.block_sparse_attention(q, k, v, r["kidx"], r["kcnt"], g)
    torch.cuda.synchronize()
    loc = orc.local_block_mask(g.bh, g.bw, g.local_range)
    probs, mask, kidx, kcnt = orc.draft_block_mask_and_probs(npf(q), npf(k), g.heads, 1, g.s, loc, g.topk)
    assert np.array_equal(r["probs"].cpu().numpy().view(np.uint32), probs.view(np.uint32))
    assert np.array_equal(r["kidx"].cpu().numpy(), kidx) and np.array_equal(r["kcnt"].cpu().numpy(), kcnt)
    items = sample_items(g.heads, g.nq, 8, kv_slices)
    ref = orc.attention(npf(q), npf(k), npf(v), kidx, kcnt, g.heads, items=items)
    cmp = orc.compare(gather_rows(npf(out), items, g.nq), gather_rows(ref, items, g.nq))
    assert cmp["rel"] <= REL_BF16, cmp
    import ctypes
    over = fvsr.Geometry(**{**g.__dict__, "kv_slices": 2560 // g.s + 1})
    n = ctypes.c_size_t(0)
    assert fvsr.lib().fvsr_lcsa_workspace_size(ctypes.byref(over.params()), ctypes.byref(n)) == fvsr.FVSR_EUNSUPPORTED
    fvsr.device_check()


# ------------------------------------------------------------------------------------------------------------------
# attention against the reference's own oracle outputs (golden fixtures, Diag.swift:86-98 recipe)
# ------------------------------------------------------------------------------------------------------------------
@pytest.mark.parametrize("case", ["attn_probe_a", "attn_probe_b"])
@pytest.mark.parametrize("dtype", ["f32", "bf16"])
def test_kernel_attention_matches_reference_golden(fvsr, orc, cfgs, case, dtype):
    from make_golden import ATTN_CASES, attn_inputs
    spec = [c for c in ATTN_CASES if c[0] == case][0]
    _, heads, nq, nk, density, seed, empty = spec
    gold = np.load(GOLDEN / f"{case}.npz")
    q, k, v, mask = attn_inputs(heads, nq, nk, density, seed, empty)
    dt = torch.float32 if dtype == "f32" else torch.bfloat16
    tq, tk, tv = (torch.from_numpy(a).to("cuda").to(dt)[None] for a in (q, k, v))
    out = fvsr.FlashVSRAttentionOps.kernel(tq, tk, tv, torch.from_numpy(mask).cuda(), heads)
    got = npf(out[0])
    cmp = orc.compare(got, gold["out"])
    assert cmp["rel"] <= (REL_F32 if dtype == "f32" else REL_BF16), cmp
    e = empty[1] * 128
    assert not got[e:e + 128, empty[0] * 128:(empty[0] + 1) * 128].any(), "empty query block must be zeros"


@pytest.mark.parametrize("dtype", ["f32", "bf16"])
def test_kernel_attention_random_masks_with_empty_rows(fvsr, orc, cfgs, dtype):
    """Diag.swift:111-121: random masks of several densities with forced empty query blocks."""
    heads, nq, nk = 2, 12, 36
    dt = torch.float32 if dtype == "f32" else torch.bfloat16
    gen = torch.Generator(device="cuda").manual_seed(3)
    for density in (0.3, 0.4, 0.6, 1.0):
        q = torch.randn((1, nq * 128, heads * 128), generator=gen, device="cuda").to(dt)
        k = torch.randn((1, nk * 128, heads * 128), generator=gen, device="cuda").to(dt)
        v = torch.randn((1, nk * 128, heads * 128), generator=gen, device="cuda").to(dt)
        m = (torch.rand((heads, nq, nk), generator=gen, device="cuda") < density).float()
        m[1, 3] = 0
        m[0, 0] = 0
        out = fvsr.kernel_block_attention(q, k, v, m, heads)
        kidx, kcnt = orc.mask_to_lists(m.cpu().numpy())
        ref = orc.attention(npf(q[0]), npf(k[0]), npf(v[0]), kidx, kcnt, heads)
        cmp = orc.compare(npf(out[0]), ref)
        assert cmp["rel"] <= (REL_F32 if dtype == "f32" else REL_BF16), (density, cmp)


# ------------------------------------------------------------------------------------------------------------------
# end to end (select → attention) at the configs' full sizes
# ------------------------------------------------------------------------------------------------------------------
def test_config1_fp32_end_to_end(fvsr, orc, cfgs):
    cfg = cfgs.CONFIGS[1]
    g = cfg.geometry()
    q, k, v = cfgs.synth_qkv(cfg, g, cfgs.seed_of(1, 0, 0))
    r = fvsr.draft_block_mask_and_probs(q, k, g)
    out = fvsr.block_sparse_attention(q, k, v, r["kidx"], r["kcnt"], g)
    loc = orc.local_block_mask(g.bh, g.bw, g.local_range)
    _, mask, kidx, kcnt = orc.draft_block_mask_and_probs(npf(q), npf(k), g.heads, 1, g.s, loc, g.topk)
    assert np.array_equal(r["kidx"].cpu().numpy(), kidx)
    ref = orc.attention(npf(q), npf(k), npf(v), kidx, kcnt, g.heads)
    cmp = orc.compare(npf(out), ref)
    assert cmp["rel"] <= REL_F32, cmp


def per_item_rel(got, ref, heads, nq):
    """max |Δ| / max |ref| of every (head, query block) item that kept a block: (H, Nq) array, 0 for empty items."""
    d = np.abs(got - ref).reshape(nq, 128, heads, 128).max(axis=(1, 3)).T
    m = np.abs(ref).reshape(nq, 128, heads, 128).max(axis=(1, 3)).T
    return np.where(m > 0, d / np.maximum(m, 1e-30), 0.0)


@pytest.mark.parametrize("cfg_id", [2, 3, 5])
def test_bf16_end_to_end_every_item(fvsr, orc, cfgs, cfg_id):
    """Configs 2, 3 and 5 at full size: the GPU selection equals the oracle's, and the attention of EVERY (head, query
    block) item is within the bf16 bar of the fp32 reference — globally (the reference's measure) and item by item.
    The checker is the oracle's fp32 attention (pinned to the reference's own oracle by the golden fixtures)."""
    cfg = cfgs.CONFIGS[cfg_id]
    g = cfg.geometry()
    q, k, v = cfgs.synth_qkv(cfg, g, cfgs.seed_of(cfg_id, 0, 1))
    r = fvsr.draft_block_mask_and_probs(q, k, g, want_probs=False, want_mask=False)
    out = fvsr.block_sparse_attention(q, k, v, r["kidx"], r["kcnt"], g)
    torch.cuda.synchronize()
    qn, kn, vn = npf(q), npf(k), npf(v)
    loc = orc.local_block_mask(g.bh, g.bw, g.local_range)
    _, _, kidx, kcnt = orc.draft_block_mask_and_probs(qn, kn, g.heads, g.q_slices, g.s, loc, g.topk)
    assert np.array_equal(r["kidx"].cpu().numpy(), kidx) and np.array_equal(r["kcnt"].cpu().numpy(), kcnt)
    ref = orc.attention(qn, kn, vn, kidx, kcnt, g.heads, fast=True)
    got = npf(out)
    cmp = orc.compare(got, ref)
    assert cmp["rel"] <= REL_BF16, cmp
    rel = per_item_rel(got, ref, g.heads, g.nq)
    assert rel.max() <= REL_BF16, (float(rel.max()), np.unravel_index(int(rel.argmax()), rel.shape))
    h_e, q_e = np.nonzero(kcnt == 0)              # empty query blocks are exactly zero
    for h, qb in zip(h_e, q_e):
        assert not got[qb * 128:(qb + 1) * 128, h * 128:(h + 1) * 128].any()


@pytest.mark.parametrize("cfg_id,qs", [(2, None), (3, None), (4, 3), (5, None)],
                         ids=["config2", "config3", "config4_chunk0", "config5"])
def test_select_flips_against_float64(fvsr, orc, cfgs, cfg_id, qs):
    """The GPU mask against an order-independent float64 evaluation of DiT.swift:158-174 (exact threshold) at full
    size: every flip must be a near-tie by the reference's own classifier (Sources/Smoke/Gates.swift:239-277: the
    probability within 1e-3 relative of its nearest sorted neighbour, or below 1e-30)."""
    cfg = cfgs.CONFIGS[cfg_id]
    g = cfg.geometry(q_slices=qs)
    q, k, _ = cfgs.synth_qkv(cfg, g, cfgs.seed_of(cfg_id, 0, 2))
    r = fvsr.draft_block_mask_and_probs(q, k, g)
    torch.cuda.synchronize()
    loc = orc.local_block_mask(g.bh, g.bw, g.local_range)
    m64, _ = orc.select_f64(npf(q), npf(k), g.heads, g.q_slices, g.s, loc, g.topk)
    rep = orc.mask_flip_report(r["mask"].cpu().numpy().astype(bool), m64, r["probs"].cpu().numpy(), g.q_slices)
    print(f"config {cfg_id}{' chunk 0' if qs else ''}: {rep}")
    assert rep["worst_gap"] <= 1e-3, rep


def test_bf16_constant_values_full_size(fvsr, cfgs):
    """Size-independent property at config 3: with V constant over keys, every non-empty query row returns that
    constant (softmax weights sum to one), whatever the selection."""
    cfg = cfgs.CONFIGS[3]
    g = cfg.geometry()
    q, k, _ = cfgs.synth_qkv(cfg, g, 99)
    gen = torch.Generator(device="cuda").manual_seed(1)
    vrow = torch.randn((1, g.channels), generator=gen, device="cuda").to(torch.bfloat16)
    v = vrow.expand(k.shape[0], -1).contiguous()
    r = fvsr.draft_block_mask_and_probs(q, k, g, want_probs=False, want_mask=False)
    out = fvsr.block_sparse_attention(q, k, v, r["kidx"], r["kcnt"], g).float()
    kc = r["kcnt"]
    live = (kc > 0).t().repeat_interleave(128, 0).repeat_interleave(128, 1)   # (Lq, H·128)
    want = vrow.float().expand_as(out)
    err = ((out - want).abs() * live).max().item()
    assert err <= REL_BF16 * vrow.float().abs().max().item(), err
    assert (out[~live] == 0).all()


# ------------------------------------------------------------------------------------------------------------------
# streaming: paged KV cache + per-layer forward (DiT.swift:504-538)
# ------------------------------------------------------------------------------------------------------------------
@pytest.mark.parametrize("kv_len,dtype", [(2, "bf16"), (3, "bf16"), (2, "f32")])
def test_streaming_forward_matches_reference_semantics(fvsr, orc, cfgs, kv_len, dtype):
    heads = 2
    base = cfgs.CONFIGS[4]
    g0 = fvsr.Geometry(heads=heads, bh=base.bh, bw=base.bw, q_slices=3, kv_slices=3, local_range=11,
                       dtype=fvsr.FVSR_BF16 if dtype == "bf16" else fvsr.FVSR_F32)
    cache = fvsr.KVCache(g0, kv_len=kv_len, max_new_slices=3)
    tdt = torch.bfloat16 if dtype == "bf16" else torch.float32
    ref_k = ref_v = None
    gen = torch.Generator(device="cuda").manual_seed(11)
    s = g0.s
    for chunk in range(4):
        qs = 3 if chunk == 0 else 1
        g = fvsr.Geometry(**{**g0.__dict__, "q_slices": qs})
        kv_total = (0 if ref_k is None else ref_k.shape[0] // (s * 128)) + qs
        gfull = fvsr.Geometry(**{**g.__dict__, "kv_slices": kv_total})
        g.topk = gfull.topk = int(round(0.6 * gfull.allowed_per_row()))
        lq = qs * s * 128
        q = (0.5 * torch.randn((lq, heads * 128), generator=gen, device="cuda")).to(tdt)
        kn = (0.5 * torch.randn((lq, heads * 128), generator=gen, device="cuda")).to(tdt)
        vn = (0.5 * torch.randn((lq, heads * 128), generator=gen, device="cuda")).to(tdt)
        kidx = torch.empty((heads, gfull.nq, gfull.nk), dtype=torch.int32, device="cuda")
        kcnt = torch.empty((heads, gfull.nq), dtype=torch.int32, device="cuda")
        out = fvsr.lcsa_forward(q, kn, vn, cache, g, kidx=kidx, kcnt=kcnt)
        # reference semantics: kW = concat(cache, new); select; attend; drop the oldest slice if slices > kvLen
        kw = npf(kn) if ref_k is None else np.concatenate([ref_k, npf(kn)])
        vw = npf(vn) if ref_v is None else np.concatenate([ref_v, npf(vn)])
        loc = orc.local_block_mask(g.bh, g.bw, g.local_range)
        _, mask, okidx, okcnt = orc.draft_block_mask_and_probs(npf(q), kw, heads, qs, s, loc, g.topk)
        assert np.array_equal(kidx.cpu().numpy(), okidx), f"chunk {chunk}: selection differs"
        ref = orc.attention(npf(q), kw, vw, okidx, okcnt, heads)
        cmp = orc.compare(npf(out), ref)
        assert cmp["rel"] <= (REL_BF16 if dtype == "bf16" else REL_F32), (chunk, cmp)
        slices = kw.shape[0] // (s * 128)
        if slices > kv_len:
            kw, vw = kw[s * 128:], vw[s * 128:]
        ref_k, ref_v = kw, vw
        assert cache.slices == ref_k.shape[0] // (s * 128)
        gk, gv = cache.gather()
        assert np.array_equal(npf(gk), ref_k) and np.array_equal(npf(gv), ref_v)
    cache.close()
    fvsr.device_check()


def test_config4_stream_full_size(fvsr, orc, cfgs):
    """Config 4 as a stream, at full size: 10 chunks of the 1280×768 output (12 heads, 6×10 spatial blocks; chunk 0 =
    3 slices, then 1 slice per chunk), kvLen 2, two DiT layers each with its own window cache, Q/K/V seeded per
    (chunk, layer). Every layer call of every chunk goes through fvsr_lcsa_forward (append, selection over
    cache ⊕ current, attention, trim) and is checked against the reference's semantics (DiT.swift:504-538) on the
    oracle: the concatenated K/V window, the selection (kidx bit-exact), the attention of every item (bf16 bar), and
    the cache contents after the trim."""
    cfg = cfgs.CONFIGS[4]
    kv_len, layers, chunks = 2, 2, 10
    g0 = cfg.geometry(q_slices=3)
    s = g0.s
    srows = s * 128
    loc = orc.local_block_mask(g0.bh, g0.bw, g0.local_range)
    caches = [fvsr.KVCache(g0, kv_len=kv_len, max_new_slices=3) for _ in range(layers)]
    ref_kv = [None] * layers            # the reference window (K, V) of each layer, on the device
    for chunk in range(chunks):
        qs = 3 if chunk == 0 else 1
        for layer in range(layers):
            have = 0 if ref_kv[layer] is None else ref_kv[layer][0].shape[0] // srows
            g = cfg.geometry(q_slices=qs, kv_slices=have + qs)      # topk = 60 % of the allowed pairs of this window
            q, kn, vn = cfgs.synth_qkv(cfg, g, cfgs.seed_of(4, chunk, layer), kv_rows=qs * srows)
            kidx = torch.empty((g.heads, g.nq, g.nk), dtype=torch.int32, device="cuda")
            kcnt = torch.empty((g.heads, g.nq), dtype=torch.int32, device="cuda")
            out = fvsr.lcsa_forward(q, kn, vn, caches[layer], g, kidx=kidx, kcnt=kcnt)
            torch.cuda.synchronize()
            kw = kn if ref_kv[layer] is None else torch.cat([ref_kv[layer][0], kn])     # DiT.swift:508-511
            vw = vn if ref_kv[layer] is None else torch.cat([ref_kv[layer][1], vn])
            qn, kwn, vwn = npf(q), npf(kw), npf(vw)
            _, _, okidx, okcnt = orc.draft_block_mask_and_probs(qn, kwn, g.heads, qs, s, loc, g.topk)
            tag = f"chunk {chunk} layer {layer}"
            assert np.array_equal(kidx.cpu().numpy(), okidx), f"{tag}: selection differs"
            ref = orc.attention(qn, kwn, vwn, okidx, okcnt, g.heads, fast=True)
            got = npf(out)
            cmp = orc.compare(got, ref)
            assert cmp["rel"] <= REL_BF16, (tag, cmp)
            rel = per_item_rel(got, ref, g.heads, g.nq)
            assert rel.max() <= REL_BF16, (tag, float(rel.max()))
            if kw.shape[0] // srows > kv_len:                                          # DiT.swift:532-538
                kw, vw = kw[srows:], vw[srows:]
            ref_kv[layer] = (kw, vw)
            gk, gv = caches[layer].gather()
            assert torch.equal(gk, kw) and torch.equal(gv, vw), f"{tag}: cache contents differ"
    for c in caches:
        c.close()
    fvsr.device_check()


@pytest.mark.parametrize("heads,dtype", [(12, "bf16"), (3, "f32"), (1, "bf16")])
def test_cache_append_pages(fvsr, heads, dtype):
    """The one-launch append writes every new slice into its own page: gather() returns the last kv_len slices in
    order after appends of 1 and 3 slices wrap the page ring, for channel counts of 1, 3 and 12 heads."""
    g = fvsr.Geometry(heads=heads, bh=3, bw=5, q_slices=3, kv_slices=5, local_range=11,
                      dtype=fvsr.FVSR_BF16 if dtype == "bf16" else fvsr.FVSR_F32)
    tdt = torch.bfloat16 if dtype == "bf16" else torch.float32
    rows = g.s * 128
    cache = fvsr.KVCache(g, kv_len=2, max_new_slices=3)
    gen = torch.Generator(device="cuda").manual_seed(5)
    ks, vs = [], []
    for n in (3, 1, 3, 1, 1, 3):
        k = torch.randn((n * rows, g.channels), generator=gen, device="cuda").to(tdt)
        v = torch.randn((n * rows, g.channels), generator=gen, device="cuda").to(tdt)
        cache.append(k, v, n)
        ks += list(k.split(rows))
        vs += list(v.split(rows))
        gk, gv = cache.gather()
        assert torch.equal(gk, torch.cat(ks[-cache.slices:])) and torch.equal(gv, torch.cat(vs[-cache.slices:]))
        while cache.slices > 2:
            cache.trim()
    cache.close()
    fvsr.device_check()


def test_device_check_clean(fvsr, cfgs):
    fvsr.device_check()


@pytest.mark.parametrize("cfg_id", [1, 2])
def test_layer_entry_equals_select_then_attention(fvsr, cfgs, cfg_id):
    """fvsr_lcsa_layer (pooling, the one-launch selection that also orders the items, attention) gives the selection
    and the output of fvsr_lcsa_select followed by fvsr_lcsa_attention, bit for bit."""
    cfg = cfgs.CONFIGS[cfg_id]
    g = cfg.geometry()
    q, k, v = cfgs.synth_qkv(cfg, g, cfgs.seed_of(cfg_id, 0, 5))
    kidx = torch.empty((g.heads, g.nq, g.nk), dtype=torch.int32, device="cuda")
    kcnt = torch.empty((g.heads, g.nq), dtype=torch.int32, device="cuda")
    out = fvsr.lcsa_layer(q, k, v, g, kidx=kidx, kcnt=kcnt)
    r = fvsr.draft_block_mask_and_probs(q, k, g, want_mask=False, want_probs=False)
    want = fvsr.block_sparse_attention(q, k, v, r["kidx"], r["kcnt"], g)
    torch.cuda.synchronize()
    assert torch.equal(kidx, r["kidx"]) and torch.equal(kcnt, r["kcnt"])
    assert torch.equal(out.view(torch.int16) if out.dtype == torch.bfloat16 else out.view(torch.int32),
                       want.view(torch.int16) if want.dtype == torch.bfloat16 else want.view(torch.int32))
    fvsr.device_check()

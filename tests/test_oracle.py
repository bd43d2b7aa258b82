"""CPU tests of the oracle: the reference's known-answer tests, its own attention oracle's outputs (golden fixtures),
and the fixed-order arithmetic the GPU kernels must reproduce. Citations are relative to the reference tree."""
from __future__ import annotations

from pathlib import Path

import numpy as np
import pytest

import detrand
from make_golden import ATTN_CASES, SELECT_CASES, attn_inputs, local_mask, select_inputs

GOLDEN = Path(__file__).resolve().parent / "golden"


# --- Tests/FlashVSRMLXTests/FlashVSRStructureTests.swift:34-44 -------------------------------------------------
def test_window_partition_round_trip_and_order(orc):
    f, h, w, c = 4, 16, 24, 3
    x = np.arange(f * h * w * c, dtype=np.float32).reshape(1, f, h, w, c)
    p = orc.window_partition(x)
    assert p.shape == ((f // 2) * (h // 8) * (w // 8), 128, c)
    win = (1 * (h // 8) + 1) * (w // 8) + 2
    tok = (1 * 8 + 3) * 8 + 5
    np.testing.assert_array_equal(p[win, tok], x[0, 3, 11, 21])
    r = orc.window_reverse(p, 1, f, h, w)
    np.testing.assert_array_equal(r.reshape(x.shape), x)


# --- FlashVSRStructureTests.swift:46-58 ------------------------------------------------------------------------
@pytest.mark.parametrize("bh,bw,r", [(3, 4, 11), (6, 10, 3), (5, 5, 4)])
def test_local_block_mask_matches_definition(orc, bh, bw, r):
    m = orc.local_block_mask(bh, bw, r)
    for q in range(bh * bw):
        for k in range(bh * bw):
            qr, qc, kr, kc = q // bw, q % bw, k // bw, k % bw
            lo = lambda v: v - r // 2  # noqa: E731
            want = lo(qr) <= kr <= lo(qr) + r - 1 and lo(qc) <= kc <= lo(qc) + r - 1
            assert m[q, k] == want
    np.testing.assert_array_equal(m, local_mask(bh, bw, r))


def test_local_block_mask_range_covering_grid_is_dense(orc):
    assert orc.local_block_mask(3, 4, 11).all()


# --- FlashVSRStructureTests.swift:60-75 ------------------------------------------------------------------------
def test_draft_mask_keeps_strictly_above_threshold(orc):
    q = np.ones((2 * 128, 128), np.float32)
    k = np.zeros((2 * 128, 128), np.float32)
    k[:128] = 2.0                                       # key block 0 scores higher than block 1
    local = np.ones((2, 2), bool)
    _, m, _, kcnt = orc.draft_block_mask_and_probs(q, k, heads=1, q_slices=1, s=2, local=local, topk=1)
    assert m.sum() == 0                                 # threshold = 2nd largest = p0 → nothing strictly above
    _, m0, kidx, kcnt = orc.draft_block_mask_and_probs(q, k, heads=1, q_slices=1, s=2, local=local, topk=2)
    np.testing.assert_array_equal(m0.reshape(-1).astype(np.float32), [1, 0, 1, 0])
    np.testing.assert_array_equal(kcnt, [[1, 1]])
    np.testing.assert_array_equal(kidx[0, :, 0], [0, 0])


def test_topk_larger_than_row_keeps_all_but_minimum(orc):
    """k = min(n − 1, topk) (DiT.swift:171): a huge topk thresholds at the smallest entry."""
    q = detrand.normal(5, (2 * 128, 128))
    k = detrand.normal(6, (4 * 128, 128))
    probs, m, _, _ = orc.draft_block_mask_and_probs(q, k, heads=1, q_slices=1, s=2, local=np.ones((2, 2), bool),
                                                    topk=10 ** 6)
    assert m.sum() == probs.size - (probs == probs.min()).sum()


# --- DiT.swift:478-485 -----------------------------------------------------------------------------------------
def test_geometry_topk(orc):
    assert orc.geometry_topk(60, 2.0) == 7199
    assert orc.geometry_topk(135, 2.0 * 768 * 1280 / (1152 * 1920)) == int(135 * 135 * (2.0 * 768 * 1280 / (1152 * 1920))) - 1
    assert orc.geometry_topk(8, 0.5) == 31


# --- the softmax exponential shared with the GPU ---------------------------------------------------------------
def test_exp_accuracy(orc):
    xs = np.concatenate([np.linspace(-103.9, 0.0, 20001), -np.logspace(-8, 1, 2001), [0.0, -1e-30, 88.0, 1.0]])
    xs = xs.astype(np.float32)
    got = np.array([orc.fvsr_exp(x) for x in xs], np.float32)
    want = np.exp(xs.astype(np.float64))
    normal = want >= np.finfo(np.float32).tiny
    ulp = np.spacing(want[normal].astype(np.float32)).astype(np.float64)
    err_ulp = np.abs(got[normal].astype(np.float64) - want[normal]) / ulp
    assert err_ulp.max() <= 1.0, err_ulp.max()
    sub = ~normal
    assert np.all(np.abs(got[sub].astype(np.float64) - want[sub]) <= 2 ** -149)
    assert orc.fvsr_exp(float("-inf")) == 0.0
    assert orc.fvsr_exp(-200.0) == 0.0


# --- pooling order ---------------------------------------------------------------------------------------------
def test_pool_fixed_order(orc):
    x = detrand.normal(7, (3 * 128, 40), bf16_exact=False)
    got = orc.pool(x)
    want = np.empty((3, 40), np.float32)
    for b in range(3):
        for c in range(40):
            parts = []
            for g in range(4):
                acc = np.float32(0)
                for t in range(32 * g, 32 * g + 32):
                    acc = np.float32(acc + x[b * 128 + t, c])
                parts.append(acc)
            want[b, c] = np.float32(np.float32(parts[0] + parts[1]) + np.float32(parts[2] + parts[3])) * np.float32(1 / 128)
    np.testing.assert_array_equal(got, want)
    xb = orc.f32_to_bf16_bits(x)
    np.testing.assert_allclose(orc.pool(xb), orc.bf16_bits_to_f32(xb).reshape(3, 128, 40).mean(1), rtol=0, atol=1e-6)


# --- attention against the reference's own oracle (golden fixtures) --------------------------------------------
@pytest.mark.parametrize("case", ATTN_CASES, ids=[c[0] for c in ATTN_CASES])
def test_attention_matches_reference_oracle(orc, case):
    name, heads, nq, nk, density, seed, empty = case
    g = np.load(GOLDEN / f"{name}.npz")
    q, k, v, mask = attn_inputs(heads, nq, nk, density, seed, empty)
    np.testing.assert_array_equal(g["mask"], mask.astype(np.uint8))
    kidx, kcnt = orc.mask_to_lists(mask)
    assert kcnt[empty[0], empty[1]] == 0
    out = orc.attention(q, k, v, kidx, kcnt, heads)
    cmp = orc.compare(out, g["out"])
    assert cmp["rel"] < 2e-6, cmp                      # reference oracle is fp32 SDPA; ours accumulates in fp64
    e = empty[1] * 128
    assert not out[e:e + 128, empty[0] * 128:(empty[0] + 1) * 128].any()
    fast = orc.attention(q, k, v, kidx, kcnt, heads, fast=True)
    assert orc.compare(fast, g["out"])["rel"] < 5e-6


def test_attention_items_subset(orc):
    name, heads, nq, nk, density, seed, empty = ATTN_CASES[0]
    q, k, v, mask = attn_inputs(heads, nq, nk, density, seed, empty)
    kidx, kcnt = orc.mask_to_lists(mask)
    full = orc.attention(q, k, v, kidx, kcnt, heads)
    items = [1 * nq + 2, 0 * nq + 0]
    part = orc.attention(q, k, v, kidx, kcnt, heads, items=items)
    for w in items:
        h, qb = divmod(w, nq)
        sl = (slice(qb * 128, qb * 128 + 128), slice(h * 128, h * 128 + 128))
        np.testing.assert_array_equal(part[sl], full[sl])


def test_attention_bf16_inputs_match_fp32_of_same_values(orc):
    name, heads, nq, nk, density, seed, empty = ATTN_CASES[1]
    q, k, v, mask = attn_inputs(heads, nq, nk, density, seed, empty)      # bf16-representable values
    kidx, kcnt = orc.mask_to_lists(mask)
    a = orc.attention(q, k, v, kidx, kcnt, heads)
    b = orc.attention(*(orc.f32_to_bf16_bits(t) for t in (q, k, v)), kidx, kcnt, heads)
    np.testing.assert_array_equal(a, b)


# --- selection against the float64 line-by-line evaluation -----------------------------------------------------
@pytest.mark.parametrize("case", SELECT_CASES, ids=[c[0] for c in SELECT_CASES])
def test_select_matches_f64_evaluation(orc, case):
    name, heads, bh, bw, qs, kvs, r, keep, seed = case
    g = np.load(GOLDEN / f"{name}.npz")
    topk = int(g["meta"][6])
    q, k = select_inputs(heads, bh, bw, qs, kvs, seed)
    probs, m, kidx, kcnt = orc.draft_block_mask_and_probs(q, k, heads, qs, bh * bw, local_mask(bh, bw, r), topk)
    rep = orc.mask_flip_report(m, g["mask"].astype(bool), probs, qs)
    assert rep["flips"] == 0, rep
    np.testing.assert_allclose(probs, g["probs"], rtol=2e-5, atol=1e-9)
    assert int(kcnt.sum()) == int(g["mask"].sum()) == topk * heads * qs
    for h in range(heads):
        for i in range(probs.shape[1]):
            sel = np.nonzero(m[h, i])[0]
            np.testing.assert_array_equal(kidx[h, i, :len(sel)], sel)
            assert (kidx[h, i, len(sel):] == -1).all()


def test_select_bad_shapes_rejected(orc):
    pq = np.zeros((6, 128), np.float32)
    with pytest.raises(ValueError):
        orc.select(pq, np.zeros((7, 128), np.float32), 1, 1, 6, np.ones((6, 6), bool), 3)   # Nk not a multiple of s
    with pytest.raises(ValueError):
        orc.select(pq, np.zeros((12, 128), np.float32), 1, 1, 6, np.ones((6, 6), bool), -1)  # negative topk


# ---------------------------------------------------------------------------------------------------------------
# q/k side of blockForward: WanRMSNorm (DiT.swift:34-47), ropeApply (DiT.swift:100-107), windowPartition (113-118)
# ---------------------------------------------------------------------------------------------------------------
def _torch_reference_prepare(x, weight, cos, sin, heads, eps, dtype):
    """DiT.swift:43-46 and 101-107 written with torch's fp32 elementwise ops, as the Swift code composes MLX ops:
    normalise in fp32, cast to T, times the weight (in T); rotate the (even, odd) pairs in fp32, cast to T."""
    import torch
    t = torch.bfloat16 if dtype == "bf16" else torch.float32
    xt = torch.from_numpy(x).view(torch.bfloat16) if dtype == "bf16" else torch.from_numpy(x)
    if weight is not None:
        wt = torch.from_numpy(weight).view(torch.bfloat16) if dtype == "bf16" else torch.from_numpy(weight)
        xf = xt.float()
        n = xf * torch.rsqrt((xf * xf).mean(dim=-1, keepdim=True) + eps)
        xt = n.to(t) * wt
    if cos is not None:
        L = xt.shape[0]
        xf = xt.float().reshape(L, heads, 64, 2)
        re, im = xf[..., 0], xf[..., 1]
        c = torch.from_numpy(cos).reshape(L, 1, 64)
        s = torch.from_numpy(sin).reshape(L, 1, 64)
        xt = torch.stack([re * c - im * s, re * s + im * c], dim=-1).reshape(L, heads * 128).to(t)
    out = xt.view(torch.int16).numpy().view(np.uint16) if dtype == "bf16" else xt.numpy()
    return out


def _bf16_ulps(a, b):
    ia = a.astype(np.int32)
    ib = b.astype(np.int32)
    # bf16 bit patterns of finite values: distance in units in the last place (same-sign values)
    return np.abs(ia - ib)


@pytest.mark.parametrize("dtype", ["f32", "bf16"])
def test_prepare_without_norm_and_rotation_is_the_window_partition(orc, dtype):
    f, h, w, heads = 4, 16, 24, 2
    rng = np.random.default_rng(3)
    x = rng.standard_normal((f * h * w, heads * 128), dtype=np.float32)
    if dtype == "bf16":
        x = orc.f32_to_bf16_bits(x)
    out = orc.prepare(x, f, h, w, heads)
    xs = x if dtype == "f32" else x.astype(np.float32)   # partition is a permutation: compare the bit patterns
    want = orc.window_partition(xs.reshape(1, f, h, w, heads * 128)).reshape(out.shape)
    assert np.array_equal(out.astype(np.float32) if dtype == "bf16" else out, want)


@pytest.mark.parametrize("dtype,heads", [("f32", 3), ("bf16", 2), ("bf16", 12)])
def test_prepare_matches_the_reference_formulas(orc, dtype, heads):
    """The rotation is bit-exact against torch's fp32 ops on the same normalised values; the norm agrees within one
    unit of the storage type's last place (only the sum of squares' order and the rsqrt rounding may differ)."""
    f, h, w = 2, 8, 16
    L, C = f * h * w, heads * 128
    rng = np.random.default_rng(7)
    x = (rng.standard_normal((L, C)) * 2.0).astype(np.float32)
    wgt = (1.0 + 0.1 * rng.standard_normal(C)).astype(np.float32)
    ang = rng.uniform(-np.pi, np.pi, (L, 64))
    cos, sin = np.cos(ang).astype(np.float32), np.sin(ang).astype(np.float32)
    if dtype == "bf16":
        x, wgt = orc.f32_to_bf16_bits(x), orc.f32_to_bf16_bits(wgt)
    # rotation alone: exact
    got = orc.prepare(x, f, h, w, heads, cos=cos, sin=sin)
    want = orc.window_partition(
        (_torch_reference_prepare(x, None, cos, sin, heads, 1e-6, dtype).astype(np.float32) if dtype == "bf16" else
         _torch_reference_prepare(x, None, cos, sin, heads, 1e-6, dtype)).reshape(1, f, h, w, C)).reshape(L, C)
    assert np.array_equal(got.astype(np.float32) if dtype == "bf16" else got, want)
    # norm (+ rotation): within one ulp of T
    got = orc.prepare(x, f, h, w, heads, weight=wgt, eps=1e-6, cos=cos, sin=sin)
    ref = _torch_reference_prepare(x, wgt, cos, sin, heads, 1e-6, dtype)
    ref = orc.window_partition((ref.astype(np.float32) if dtype == "bf16" else ref).reshape(1, f, h, w, C))
    ref = ref.reshape(L, C)
    if dtype == "bf16":
        d = _bf16_ulps(got, ref.astype(np.uint16))
        assert d.max() <= 1 and (d == 0).mean() > 0.99, (d.max(), (d == 0).mean())
    else:
        # a one-ulp difference of a normalised value, carried through the rotation's cancellations
        rel = np.abs(got - ref).max(axis=1) / np.abs(ref).max(axis=1)
        assert rel.max() <= 8 * np.finfo(np.float32).eps, rel.max()


# --- DiT.swift:163-173: invariants of the selection rule on random geometries -----------------------------------
def test_select_invariants_over_random_geometries(orc):
    """Seeded random geometries (grid, slices, locality range, top-k from 0 past the row length):
    - kept entries are locality-allowed;
    - each query block's probabilities sum to one over its allowed key blocks, and are zero elsewhere;
    - each (head, query slice) row keeps at most k = min(n − 1, topk) entries, every kept one strictly above every
      dropped one;
    - kcnt counts the mask, and kidx lists its kept key blocks ascending, then −1."""
    rng = np.random.default_rng(77)
    for case in range(24):
        heads, bh, bw = int(rng.integers(1, 4)), int(rng.integers(1, 5)), int(rng.integers(1, 5))
        qs = int(rng.integers(1, 3))
        ks = int(rng.integers(qs, qs + 3))
        r = int(rng.integers(1, 8))
        s = bh * bw
        nq, nk = qs * s, ks * s
        n = s * nk
        topk = int(rng.integers(0, n + 2))
        pq = rng.standard_normal((nq, heads * 128)).astype(np.float32)
        pk = rng.standard_normal((nk, heads * 128)).astype(np.float32)
        loc = orc.local_block_mask(bh, bw, r)
        probs, mask, kidx, kcnt = orc.select(pq, pk, heads, qs, s, loc, topk)
        m = mask.astype(bool)
        allowed = np.tile(loc, (qs, ks))                               # [i, j] = loc[i mod s, j mod s]
        tag = f"case {case}: H={heads} {bh}x{bw} qs={qs} ks={ks} R={r} topk={topk}"
        assert not (m & ~allowed[None]).any(), tag
        assert (probs[:, ~allowed] == 0).all(), tag
        np.testing.assert_allclose(probs.sum(axis=2), 1.0, rtol=0, atol=2e-6, err_msg=tag)
        k = min(n - 1, topk)
        for h in range(heads):
            for sl in range(qs):
                p = probs[h, sl * s:(sl + 1) * s].reshape(-1)
                kept = m[h, sl * s:(sl + 1) * s].reshape(-1)
                assert kept.sum() <= k, tag
                if kept.any() and (~kept).any():
                    assert p[kept].min() > p[~kept].max(), tag
        np.testing.assert_array_equal(kcnt, m.sum(axis=2), err_msg=tag)
        for h in range(heads):
            for i in range(nq):
                want = np.flatnonzero(m[h, i])
                np.testing.assert_array_equal(kidx[h, i, :len(want)], want, err_msg=tag)
                assert (kidx[h, i, len(want):] == -1).all(), tag


# --- DiT.swift:279-313 semantics: properties of attention over kept blocks --------------------------------------
def test_attention_properties(orc):
    """Size-independent properties of attention over kept blocks, checked on the oracle that judges every path:
    - linear in V;
    - a V constant over keys passes through every non-empty query row, and query blocks with no kept key block give
      zero rows;
    - scaling a head's V columns scales that head's output columns;
    - adding one vector u to every key of a head shifts each query row's scores by the constant q·u, which the
      softmax cancels: the output is unchanged."""
    rng = np.random.default_rng(11)
    heads, nq, nk = 2, 3, 5
    q = rng.standard_normal((nq * 128, heads * 128)).astype(np.float32)
    k = rng.standard_normal((nk * 128, heads * 128)).astype(np.float32)
    v1 = rng.standard_normal((nk * 128, heads * 128)).astype(np.float32)
    v2 = rng.standard_normal((nk * 128, heads * 128)).astype(np.float32)
    mask = rng.random((heads, nq, nk)) < 0.5
    mask[1, 2] = False                                           # one empty query block
    mask[0, 0] = True                                            # one full one
    kidx, kcnt = orc.mask_to_lists(mask)
    att = lambda v: orc.attention(q, k, v, kidx, kcnt, heads).astype(np.float64)  # noqa: E731
    a, b = 0.75, -1.25
    mix = (a * v1.astype(np.float64) + b * v2.astype(np.float64)).astype(np.float32)
    lin = a * att(v1) + b * att(v2)
    np.testing.assert_allclose(att(mix), lin, rtol=0, atol=1e-6 * np.abs(lin).max())
    row = rng.standard_normal((1, heads * 128)).astype(np.float32)
    const = att(np.repeat(row, nk * 128, axis=0))
    for h in range(heads):
        for i in range(nq):
            blk = const[i * 128:(i + 1) * 128, h * 128:(h + 1) * 128]
            if kcnt[h, i] == 0:
                assert not blk.any()
            else:
                np.testing.assert_allclose(blk, np.broadcast_to(row[:, h * 128:(h + 1) * 128], blk.shape),
                                           rtol=0, atol=1e-6 * np.abs(row).max())
    scale = np.repeat(rng.uniform(0.5, 2.0, heads), 128).astype(np.float32)
    np.testing.assert_allclose(att(v1 * scale), att(v1) * scale, rtol=0, atol=1e-6 * np.abs(att(v1)).max())
    u = np.tile(0.5 * rng.standard_normal((1, heads * 128)).astype(np.float32), (nk * 128, 1))
    shifted = orc.attention(q, k + u, v1, kidx, kcnt, heads).astype(np.float64)
    np.testing.assert_allclose(shifted, att(v1), rtol=0, atol=1e-6 * np.abs(att(v1)).max())


# --- mask flips against float64 at the configs' full spatial sizes ---------------------------------------------
FLIP_CASES = [  # (config, bh, bw, q_slices, kv_slices, keep, distribution)
    (3, 9, 15, 1, 3, 0.30, "normal"),
    (4, 6, 10, 3, 3, 0.60, "c2"),
    (5, 12, 20, 1, 3, 0.25, "c2"),
]


@pytest.mark.parametrize("case", FLIP_CASES, ids=[f"config{c[0]}" for c in FLIP_CASES])
def test_select_flips_against_f64_at_full_size(orc, case):
    """The fixed-order fp32 selection against the order-independent float64 evaluation (exact threshold) of
    DiT.swift:158-174 at a config's full spatial size, two heads (selection rows are per head, so two are as
    representative as twelve): every flip must be a near-tie by the reference's classifier (Gates.swift:239-277).
    Inputs are seeded PCG64 normals rounded to bf16 (a property check, so no fixed bit stream is needed)."""
    cfg_id, bh, bw, qs, kvs, keep, dist = case
    heads, s = 2, bh * bw
    nq, nk, c = qs * s, kvs * s, heads * 128
    rng = np.random.default_rng(7000 + cfg_id)
    std = 0.5 if dist == "c2" else 1.0
    q = rng.standard_normal((nq * 128, c), dtype=np.float32) * np.float32(std)
    k = rng.standard_normal((nk * 128, c), dtype=np.float32) * np.float32(std)
    if dist == "c2":
        off = rng.standard_normal((nk, 1, c), dtype=np.float32) * np.float32(0.3)
        k = (k.reshape(nk, 128, c) + off).reshape(-1, c)
    loc = local_mask(bh, bw, 11)
    topk = int(round(keep * int(loc.sum()) * kvs))
    qb, kb = orc.f32_to_bf16_bits(q), orc.f32_to_bf16_bits(k)
    probs, m, _, kcnt = orc.draft_block_mask_and_probs(qb, kb, heads, qs, s, loc, topk)
    m64, _ = orc.select_f64(qb, kb, heads, qs, s, loc, topk)
    rep = orc.mask_flip_report(m, m64, probs, qs)
    assert rep["worst_gap"] <= 1e-3, rep
    assert int(kcnt.sum()) == topk * heads * qs

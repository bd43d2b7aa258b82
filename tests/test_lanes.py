"""The reference's study lanes of FlashVSRAttentionOps (dense, gathered; SparseAttention.swift:190-201) as restated in
``tests/lanes.py``, checked on the CPU against the oracle with the reference's probe recipe
(Sources/Smoke/Diag.swift:86-121: random block masks of density 0.3-0.6 with forced empty query blocks, fp32 and
bf16 against fp32), and their grouping rules (score and gather budgets) against one group."""
from __future__ import annotations

import importlib

import numpy as np
import pytest

torch = pytest.importorskip("torch")

REL_F32 = 1e-5
REL_BF16 = 1e-2


@pytest.fixture(scope="module")
def lanes():
    return importlib.import_module("lanes")


def probe_inputs(seed, heads=2, nq=4, nk=6, density=0.45):
    rng = np.random.default_rng(seed)
    q = rng.standard_normal((nq * 128, heads * 128)).astype(np.float32)
    k = rng.standard_normal((nk * 128, heads * 128)).astype(np.float32)
    v = rng.standard_normal((nk * 128, heads * 128)).astype(np.float32)
    mask = rng.random((heads, nq, nk)) < density
    mask[0, 1] = False                              # forced empty query blocks
    mask[heads - 1, nq - 1] = False
    return q, k, v, mask


@pytest.mark.parametrize("seed,density", [(1, 0.3), (2, 0.45), (3, 0.6)])
@pytest.mark.parametrize("lane", ["dense", "gathered"])
def test_lane_matches_oracle(fvsr, orc, lanes, lane, seed, density):
    heads = 2
    q, k, v, mask = probe_inputs(seed, heads=heads, density=density)
    kidx, kcnt = orc.mask_to_lists(mask)
    ref = orc.attention(q, k, v, kidx, kcnt, heads)
    fn = getattr(lanes, f"{lane}_block_attention")
    bm = torch.from_numpy(mask.astype(np.float32))
    got = fn(torch.from_numpy(q)[None], torch.from_numpy(k)[None], torch.from_numpy(v)[None], bm, heads)
    assert got.shape == (1, q.shape[0], q.shape[1])
    cmp = orc.compare(got[0].numpy(), ref)
    assert cmp["rel"] <= REL_F32, cmp
    # bf16 inputs against the fp32 reference of the same (rounded) values
    qb, kb, vb = (torch.from_numpy(t).to(torch.bfloat16) for t in (q, k, v))
    ref_b = orc.attention(*(t.float().numpy() for t in (qb, kb, vb)), kidx, kcnt, heads)
    got_b = fn(qb, kb, vb, bm, heads)
    assert got_b.dtype == torch.bfloat16
    cmp_b = orc.compare(got_b.float().numpy(), ref_b)
    assert cmp_b["rel"] <= REL_BF16, cmp_b
    for h, qbk in zip(*np.nonzero(kcnt == 0)):
        assert not got[0, qbk * 128:(qbk + 1) * 128, h * 128:(h + 1) * 128].any()


def test_lane_budgets_split_into_groups_without_changing_results(fvsr, lanes):
    """A score budget of one query block's scores and a gather budget of one padded block pair force a group per query
    block (DiT.swift:284, 240-246); every row is computed alone either way."""
    heads = 2
    q, k, v, mask = probe_inputs(7, heads=heads, nq=5, nk=4)
    tq, tk, tv, bm = (torch.from_numpy(t) for t in (q, k, v, mask.astype(np.float32)))
    one = lanes.dense_block_attention(tq, tk, tv, bm, heads)
    split = lanes.dense_block_attention(tq, tk, tv, bm, heads, score_budget_bytes=128 * k.shape[0] * 4)
    torch.testing.assert_close(split, one, rtol=0, atol=1e-6)
    g_one = lanes.gathered_block_attention(tq, tk, tv, bm, heads)
    g_split = lanes.gathered_block_attention(tq, tk, tv, bm, heads, gather_budget_bytes=1)
    torch.testing.assert_close(g_split, g_one, rtol=0, atol=1e-6)
    torch.testing.assert_close(g_one, one, rtol=0, atol=1e-5)


def test_lanes_reject_bad_shapes(fvsr, lanes):
    q = torch.zeros((256, 256))
    k = torch.zeros((384, 256))
    with pytest.raises(ValueError):
        lanes.dense_block_attention(q, k, k, torch.ones((2, 2, 2)), 2)        # Nk = 3 blocks, mask says 2
    with pytest.raises(ValueError):
        lanes.gathered_block_attention(q, k, k, torch.ones((2, 2, 3)), 3)     # 3 heads of 128 ≠ 256 columns
    with pytest.raises(fvsr.FVSRError):
        fvsr.FlashVSRAttentionOps.kernel(q, k, k, torch.ones((2, 2, 3)), 2, simdgroups=0)

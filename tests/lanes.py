"""The reference's two study lanes of block-masked attention, restated with torch for tests that compare lanes.

TEST INFRASTRUCTURE ONLY: the product package does not import this module.

``FlashVSRAttentionOps`` (Sources/FlashVSRMLX/SparseAttention.swift:190-201) offers three lanes with one meaning: per
head, softmax(q·kᵀ/√128) over the key tokens of the kept key blocks, times v; query blocks with no kept key block
give zero rows. The reference's probes check the kernel lane against the dense one (Sources/Smoke/Diag.swift:86-121).

- ``kernel`` is the product: the sm_100a kernels behind the C ABI (``FlashVSRAttentionOps.kernel`` in the package).
- ``dense`` (blockMaskedAttention, DiT.swift:279-313) and ``gathered`` (gatheredBlockAttention, DiT.swift:219-273)
  are the reference's other two algorithms. They are restated here with torch's scaled-dot-product attention (library
  arithmetic, on whatever device the tensors are on), keeping the reference's grouping rules and budgets, so a test
  can hold the kernel lane against them as the reference's probes do.
"""
from __future__ import annotations

import math
import os


def _prep(q, k, v, block_mask, heads: int):
    import torch

    def rows(t):
        if t.dim() == 3:
            if t.shape[0] != 1:
                raise ValueError("batch must be 1")
            t = t[0]
        return t

    q2, k2, v2 = rows(q), rows(k), rows(v)
    lq, d = q2.shape
    lk = k2.shape[0]
    if d % heads or d // heads != 128 or k2.shape[1] != d or v2.shape != k2.shape:
        raise ValueError("q, k, v must be (L, H·128) with head dim 128")
    nq, nk = int(block_mask.shape[1]), int(block_mask.shape[2])
    if block_mask.shape[0] != heads or lq != nq * 128 or lk != nk * 128:
        raise ValueError("block_mask must be (H, Lq/128, Lk/128)")
    sel = torch.as_tensor(block_mask, device=q2.device) > 0.5
    return q2, k2, v2, sel, nq, nk


def dense_block_attention(q, k, v, block_mask, heads: int, score_budget_bytes: int | None = None):
    """blockMaskedAttention (DiT.swift:279-313): per head, attention under the token-expanded block mask, in groups of
    query blocks whose fp32 scores fit `score_budget_bytes` (FLASHVSR_ATTN_BUDGET_MB, default 512 MB, DiT.swift:275-277);
    a query block that kept nothing gives zeros (DiT.swift:300-304)."""
    import torch
    import torch.nn.functional as F

    shape = q.shape
    q2, k2, v2, sel, nq, nk = _prep(q, k, v, block_mask, heads)
    if score_budget_bytes is None:
        score_budget_bytes = int(os.environ.get("FLASHVSR_ATTN_BUDGET_MB", "512")) << 20
    lk = k2.shape[0]
    group = max(1, min(nq, score_budget_bytes // (128 * lk * 4)))
    out = torch.empty_like(q2)
    scale = 1.0 / math.sqrt(128)
    for h in range(heads):
        cols = slice(h * 128, (h + 1) * 128)
        kh, vh = k2[:, cols][None, None], v2[:, cols][None, None]
        for g0 in range(0, nq, group):
            g1 = min(nq, g0 + group)
            bm = sel[h, g0:g1]
            tok = bm.repeat_interleave(128, 0).repeat_interleave(128, 1)            # (n·128, Lk)
            o = F.scaled_dot_product_attention(q2[g0 * 128:g1 * 128, cols][None, None], kh, vh,
                                               attn_mask=tok[None, None], scale=scale)[0, 0]
            live = bm.any(dim=1).repeat_interleave(128)[:, None]
            out[g0 * 128:g1 * 128, cols] = torch.where(live, o, torch.zeros((), dtype=o.dtype, device=o.device))
    return out.reshape(shape)


def gathered_block_attention(q, k, v, block_mask, heads: int, gather_budget_bytes: int = 1 << 30):
    """gatheredBlockAttention (DiT.swift:219-273): per head, each query block attends to its kept key blocks only,
    gathered (kept first, ascending) and padded to the group's largest count; a group of query blocks grows while the
    padded K and V gathers fit `gather_budget_bytes`; a query block that kept nothing gives zeros."""
    import torch
    import torch.nn.functional as F

    shape = q.shape
    q2, k2, v2, sel, nq, nk = _prep(q, k, v, block_mask, heads)
    counts = sel.sum(dim=-1).to(torch.int64)                                         # (H, Nq)
    order = torch.argsort((~sel).to(torch.int8), dim=-1, stable=True)               # kept blocks first, ascending
    counts_host = counts.cpu().tolist()
    item = k2.element_size()
    out = torch.zeros_like(q2)
    scale = 1.0 / math.sqrt(128)
    for h in range(heads):
        cols = slice(h * 128, (h + 1) * 128)
        qb = q2[:, cols].reshape(nq, 1, 128, 128)
        kb = k2[:, cols].reshape(nk, 128, 128)
        vb = v2[:, cols].reshape(nk, 128, 128)
        ch = counts_host[h]
        g0 = 0
        while g0 < nq:
            g1, max_c = g0, 0
            while g1 < nq:
                m = max(max_c, ch[g1])
                if g1 > g0 and (g1 + 1 - g0) * max(m, 1) * 128 * 128 * item * 2 > gather_budget_bytes:
                    break
                max_c, g1 = m, g1 + 1
            n = g1 - g0
            if max_c > 0:
                idx = order[h, g0:g1, :max_c].reshape(-1)
                kg = kb[idx].reshape(n, 1, max_c * 128, 128)
                vg = vb[idx].reshape(n, 1, max_c * 128, 128)
                valid = torch.arange(max_c, device=q2.device)[None, :] < counts[h, g0:g1, None]   # (n, maxC)
                key_mask = valid.repeat_interleave(128, 1)[:, None, None, :]               # (n, 1, 1, maxC·128)
                o = F.scaled_dot_product_attention(qb[g0:g1], kg, vg, attn_mask=key_mask, scale=scale)
                live = (counts[h, g0:g1] > 0).repeat_interleave(128)[:, None]
                rows = o.reshape(n * 128, 128)
                out[g0 * 128:g1 * 128, cols] = torch.where(live, rows,
                                                           torch.zeros((), dtype=rows.dtype, device=rows.device))
            g0 = g1
    return out.reshape(shape)

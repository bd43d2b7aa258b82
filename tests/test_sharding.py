"""Query-block sharding of the (head, query block) item space across ranks (config 5, strong scaling).

CPU: the partition covers every item exactly once, is balanced, and every rank derives the same plan (two gloo
ranks). GPU: a rank's range attention on its local heads reproduces the one-GPU result for the same items."""
from __future__ import annotations

import importlib
import os

import numpy as np
import pytest
import torch
import torch.distributed as dist
import torch.multiprocessing as mp


@pytest.mark.parametrize("heads,nq,world", [(12, 240, 1), (12, 240, 2), (12, 240, 8), (12, 135, 3), (1, 5, 8)])
def test_shard_items_partition(fvsr, heads, nq, world):
    seen = np.zeros(heads * nq, np.int32)
    sizes = []
    for r in range(world):
        sh = fvsr.shard_items(heads, nq, world, r)
        seen[sh.begin:sh.end] += 1
        sizes.append(sh.end - sh.begin)
        if sh.end > sh.begin:
            assert sh.head_lo == sh.begin // nq and sh.head_hi == (sh.end - 1) // nq
            lb, lc = sh.local_range(nq)
            assert 0 <= lb and lb + lc <= sh.heads * nq and lc == sh.end - sh.begin
    assert (seen == 1).all()
    assert max(sizes) - min(sizes) <= 1


def _gloo_rank(rank, world, port, results):
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
    dist.init_process_group("gloo", rank=rank, world_size=world)
    import sys
    sys.path.insert(0, os.environ["FVSR_ROOT"])
    from __graft_entry__ import _load_package
    fvsr = _load_package()
    sh = fvsr.shard_items(12, 240, world, rank)
    t = torch.tensor([sh.end - sh.begin, sh.begin, sh.end], dtype=torch.int64)
    gathered = [torch.zeros_like(t) for _ in range(world)]
    dist.all_gather(gathered, t)
    if rank == 0:
        results.put([g.tolist() for g in gathered])
    dist.destroy_process_group()


def test_shard_plan_agrees_across_gloo_ranks(fvsr):
    world = 2
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    os.environ["FVSR_ROOT"] = str(__import__("pathlib").Path(__file__).resolve().parent.parent)
    port = 29500 + os.getpid() % 1000
    procs = [ctx.Process(target=_gloo_rank, args=(r, world, port, q)) for r in range(world)]
    for p in procs:
        p.start()
    res = q.get(timeout=120)
    for p in procs:
        p.join(timeout=60)
        assert p.exitcode == 0
    counts = [r[0] for r in res]
    assert sum(counts) == 12 * 240
    assert res[0][2] == res[1][1]          # rank 0 ends where rank 1 starts


@pytest.mark.gpu
def test_range_attention_reproduces_one_gpu_items(fvsr):
    if not torch.cuda.is_available():
        pytest.skip("no CUDA device")
    cfgs = importlib.import_module("fvsr_b200.configs")
    cfg = cfgs.CONFIGS[2]
    g = cfg.geometry()
    heads = 4
    g = fvsr.Geometry(**{**g.__dict__, "heads": heads})
    one = fvsr.Geometry(**{**g.__dict__, "heads": 1})
    per_head = [cfgs.synth_qkv(cfg, one, 500 + h) for h in range(heads)]
    q, k, v = (torch.cat([ph[i] for ph in per_head], dim=1).contiguous() for i in range(3))
    sel = fvsr.draft_block_mask_and_probs(q, k, g, want_mask=False, want_probs=False)
    full = fvsr.block_sparse_attention(q, k, v, sel["kidx"], sel["kcnt"], g)
    world = 3
    for r in range(world):
        sh = fvsr.shard_items(heads, g.nq, world, r)
        gl = fvsr.Geometry(**{**g.__dict__, "heads": sh.heads})
        ql, kl, vl = (torch.cat([per_head[h][i] for h in range(sh.head_lo, sh.head_hi + 1)], dim=1).contiguous()
                      for i in range(3))
        sl = fvsr.draft_block_mask_and_probs(ql, kl, gl, want_mask=False, want_probs=False)
        out = torch.zeros_like(ql)
        lb, lc = sh.local_range(g.nq)
        order = fvsr.item_order(sl["kcnt"], gl, lb, lc) if r % 2 == 0 else None   # the schedule changes no result
        if order is not None:
            o = order.cpu().numpy()
            assert sorted(o.tolist()) == list(range(lb, lb + lc))
            kc = sl["kcnt"].view(-1).cpu().numpy()
            for hseg in range(sh.heads):   # longest first within each head segment, heads in order
                seg = [x for x in o if x // g.nq == hseg]
                assert all(kc[a] >= kc[b] for a, b in zip(seg, seg[1:]))
            nz = [kc[x] > 0 for x in o]     # every empty item after every non-empty one, empties by id
            assert nz == sorted(nz, reverse=True)
            empties = [x for x in o if kc[x] <= 0]
            assert empties == sorted(empties)
            heads_nz = [x // g.nq for x in o if kc[x] > 0]
            assert heads_nz == sorted(heads_nz)
        fvsr.block_sparse_attention_range(ql, kl, vl, sl["kidx"], sl["kcnt"], gl, lb, lc, out, order=order)
        torch.cuda.synchronize()
        for it in range(sh.begin, sh.end):
            h, qb = divmod(it, g.nq)
            hl = h - sh.head_lo
            a = out[qb * 128:(qb + 1) * 128, hl * 128:(hl + 1) * 128]
            b = full[qb * 128:(qb + 1) * 128, h * 128:(h + 1) * 128]
            assert torch.equal(a, b), (r, it)
        # items of the touched heads outside the rank's range are left unwritten
        outside = [it for it in range(sh.head_lo * g.nq, (sh.head_hi + 1) * g.nq) if not sh.begin <= it < sh.end]
        for it in outside[:4]:
            h, qb = divmod(it, g.nq)
            hl = h - sh.head_lo
            assert not out[qb * 128:(qb + 1) * 128, hl * 128:(hl + 1) * 128].any()
    fvsr.device_check()


def _config5_rank(fvsr, world, rank, dtype=None):
    """Config 5 as rank `rank` of `world` holds it: the heads its items touch, and its range in local items."""
    cfgs = importlib.import_module("fvsr_b200.configs")
    cfg = cfgs.CONFIGS[5]
    g = cfg.geometry()
    sh = fvsr.shard_items(g.heads, g.nq, world, rank)
    one = fvsr.Geometry(**{**g.__dict__, "heads": 1})
    per_head = [cfgs.synth_qkv(cfg, one, 900 + h) for h in range(sh.head_lo, sh.head_hi + 1)]
    q, k, v = (torch.cat([ph[i] for ph in per_head], dim=1).contiguous() for i in range(3))
    gl = fvsr.Geometry(**{**g.__dict__, "heads": sh.heads})
    sel = fvsr.draft_block_mask_and_probs(q, k, gl, want_mask=False, want_probs=False)
    if dtype == "f32":
        q, k, v = q.float(), k.float(), v.float()
        gl = fvsr.Geometry(**{**gl.__dict__, "dtype": 0})
    lb, lc = sh.local_range(g.nq)
    return gl, q, k, v, sel, lb, lc


@pytest.mark.gpu
@pytest.mark.parametrize("world,rank", [(12, 0), (24, 1)])
def test_schedule_gives_every_sm_an_equal_share(fvsr, world, rank):
    """A range inside one head: the persistent partition (equal key-block shares, cut items merged)."""
    if not torch.cuda.is_available():
        pytest.skip("no CUDA device")
    gl, q, k, v, sel, lb, lc = _config5_rank(fvsr, world, rank)
    assert lb // gl.nq == (lb + lc - 1) // gl.nq
    buf = fvsr.make_schedule(sel["kcnt"], gl, lb, lc)
    hdr, seg_begin, segs, comb, empties = fvsr.schedule_view(buf, gl, lc)
    kc = sel["kcnt"].view(-1).cpu().numpy()[lb:lb + lc].astype(np.int64)
    G = torch.cuda.get_device_properties(0).multi_processor_count
    assert hdr["heads"] == 1
    assert sorted(empties.tolist()) == [lb + i for i in range(lc) if kc[i] == 0] and hdr["empty_items"] == len(empties)
    assert seg_begin[0] == 0 and seg_begin[G] == hdr["segments"] and (np.diff(seg_begin) >= 0).all()
    S = int(kc.sum())
    Q = max(-(-S // G), 1)
    per_sm = [int(segs[seg_begin[c]:seg_begin[c + 1], 2].sum()) for c in range(G)]
    assert per_sm == [min(Q, max(0, S - c * Q)) for c in range(G)]
    # every non-empty item's key list [0, cnt) is covered once; cut items have consecutive piece slots
    by_item = {}
    for it, b, n, slot in segs.tolist():
        by_item.setdefault(it, []).append((b, n, slot))
    assert sorted(by_item) == [lb + i for i in range(lc) if kc[i] > 0]
    cut = {}
    for it, parts in by_item.items():
        parts.sort()
        assert parts[0][0] == 0 and sum(n for _, n, _ in parts) == kc[it - lb]
        assert all(parts[i][0] + parts[i][1] == parts[i + 1][0] for i in range(len(parts) - 1))
        if len(parts) == 1:
            assert parts[0][2] == -1
        else:
            slots = [sl for _, _, sl in parts]
            assert slots == list(range(slots[0], slots[0] + len(parts)))
            cut[it] = (slots[0], len(parts))
    assert cut and {int(c[0]): (int(c[1]), int(c[2])) for c in comb} == cut
    assert hdr["cut_items"] == len(cut) <= G - 1 and hdr["pieces"] == sum(n for _, n in cut.values())
    fvsr.device_check()


@pytest.mark.gpu
@pytest.mark.parametrize("world,rank,dtype", [(12, 0, "bf16"), (24, 1, "bf16"), (8, 0, "bf16"), (12, 0, "f32")])
def test_scheduled_attention_matches_range_attention(fvsr, orc, world, rank, dtype):
    if not torch.cuda.is_available():
        pytest.skip("no CUDA device")
    gl, q, k, v, sel, lb, lc = _config5_rank(fvsr, world, rank, dtype)
    ref_out = torch.zeros_like(q)
    fvsr.block_sparse_attention_range(q, k, v, sel["kidx"], sel["kcnt"], gl, lb, lc, ref_out,
                                      order=fvsr.item_order(sel["kcnt"], gl, lb, lc))
    buf = fvsr.make_schedule(sel["kcnt"], gl, lb, lc)
    out = torch.full_like(q, 7.0)                         # empty items must be overwritten with zeros
    fvsr.block_sparse_attention_scheduled(q, k, v, sel["kidx"], sel["kcnt"], gl, lb, lc, out, buf)
    torch.cuda.synchronize()
    nq = gl.nq

    def block(t, it):
        h, qb = divmod(it, nq)
        return t[qb * 128:(qb + 1) * 128, h * 128:(h + 1) * 128]

    G = torch.cuda.get_device_properties(0).multi_processor_count
    persistent = fvsr.schedule_is_persistent(gl, lb, lc, G)
    assert persistent == (dtype == "bf16" and lb // nq == (lb + lc - 1) // nq)
    cut = set()
    if persistent:
        _, _, _, comb, _ = fvsr.schedule_view(buf, gl, lc)
        cut = {int(c[0]) for c in comb}
        assert cut
    for it in range(lb, lb + lc):                         # whole items: the per-item kernel's exact arithmetic
        if it not in cut:
            assert torch.equal(block(out, it), block(ref_out, it)), it
    if cut:                                               # cut items: merged pieces vs the fp32 oracle (bf16 bar)
        items = np.array(sorted(cut)[:6], np.int32)
        ref = orc.attention(q.float().cpu().numpy(), k.float().cpu().numpy(), v.float().cpu().numpy(),
                            sel["kidx"].cpu().numpy(), sel["kcnt"].cpu().numpy(), gl.heads, items=items)
        for it in items:
            h, qb = divmod(int(it), nq)
            r = ref[qb * 128:(qb + 1) * 128, h * 128:(h + 1) * 128]
            cmp = orc.compare(block(out, int(it)).float().cpu().numpy(), r)
            assert cmp["rel"] <= 1e-2, (int(it), cmp)
            cmp2 = orc.compare(block(out, int(it)).float().cpu().numpy(),
                               block(ref_out, int(it)).float().cpu().numpy())
            assert cmp2["rel"] <= 1e-2, (int(it), cmp2)
    fvsr.device_check()


def test_schedule_entry_points_validate(fvsr):
    import ctypes
    L = fvsr.lib()
    g = fvsr.Geometry(heads=2, bh=4, bw=4, q_slices=1, kv_slices=3, local_range=5, topk=10, dtype=1)
    p = g.params()
    n = ctypes.c_size_t(0)
    assert L.fvsr_lcsa_schedule_size(ctypes.byref(p), -1, ctypes.byref(n)) == fvsr.FVSR_EINVAL
    assert L.fvsr_lcsa_schedule_size(ctypes.byref(p), 2 * g.nq + 1, ctypes.byref(n)) == fvsr.FVSR_EINVAL
    assert L.fvsr_lcsa_schedule(ctypes.byref(p), None, 0, 4, None, 0, None) != fvsr.FVSR_OK
    assert L.fvsr_lcsa_attention_scheduled(ctypes.byref(p), None, None, None, None, None, None, 5, -2, None, 0,
                                           None) == fvsr.FVSR_EINVAL


@pytest.mark.gpu
def test_scheduled_attention_with_every_item_empty(fvsr):
    """topk = 0 keeps nothing: the persistent partition has no work, and every item of the range is written as
    zeros by the combine step (SparseAttention.swift:47-53)."""
    if not torch.cuda.is_available():
        pytest.skip("no CUDA device")
    gl, q, k, v, _, lb, lc = _config5_rank(fvsr, 12, 0)
    g0 = fvsr.Geometry(**{**gl.__dict__, "topk": 0})
    sel = fvsr.draft_block_mask_and_probs(q, k, g0, want_mask=False, want_probs=False)
    assert int(sel["kcnt"].sum()) == 0
    G = torch.cuda.get_device_properties(0).multi_processor_count
    assert fvsr.schedule_is_persistent(g0, lb, lc, G)
    buf = fvsr.make_schedule(sel["kcnt"], g0, lb, lc)
    out = torch.full_like(q, 7.0)
    fvsr.block_sparse_attention_scheduled(q, k, v, sel["kidx"], sel["kcnt"], g0, lb, lc, out, buf)
    torch.cuda.synchronize()
    hdr, seg_begin, segs, comb, empties = fvsr.schedule_view(buf, g0, lc)
    assert hdr["segments"] == 0 and hdr["cut_items"] == 0 and hdr["empty_items"] == lc
    for it in range(lb, lb + lc):
        h, qb = divmod(it, g0.nq)
        assert not out[qb * 128:(qb + 1) * 128, h * 128:(h + 1) * 128].any(), it
    fvsr.device_check()

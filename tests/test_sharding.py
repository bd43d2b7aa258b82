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

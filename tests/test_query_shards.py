"""The query-block partition of one streamed chunk across ranks (fvsr_kv_cache_reserve / commit and
fvsr_lcsa_forward_shard; the host side in shard.py).

On one GPU the ranks are emulated in turn, with copies in place of the all-gathers: each rank's output rows, and the
selection every rank computes, must equal fvsr_lcsa_forward on the whole chunk bit for bit (the per-item arithmetic is
the same). With two or more GPUs, two processes run the real NCCL path of ShardedChunk and compare with one GPU.
CPU: the shard plan covers the chunk exactly once and its padded shards reassemble it."""
from __future__ import annotations

import importlib
import os

import numpy as np
import pytest

torch = pytest.importorskip("torch")


@pytest.mark.parametrize("nq,world", [(135, 1), (135, 2), (135, 8), (240, 8), (60, 7), (3, 8)])
def test_query_shard_plan(fvsr, nq, world):
    seen = np.zeros(nq, np.int32)
    for r in range(world):
        sh = fvsr.query_shard(nq, world, r)
        assert sh.width == -(-nq // world) and 0 <= sh.blocks <= sh.width
        assert sh.begin == min(nq, r * sh.width)                   # rank r's padded shard sits at r·width
        seen[sh.begin:sh.end] += 1
    assert (seen == 1).all()
    with pytest.raises(fvsr.FVSRError):
        fvsr.query_shard(nq, world, world)


def _slices(cfgs, cfg, g, seed, n):
    rows = g.s * 128
    gen = torch.Generator(device="cuda").manual_seed(seed)
    return [(0.5 * torch.randn((rows, g.channels), generator=gen, device="cuda")).to(torch.bfloat16) for _ in range(n)]


def _rank_cache(fvsr, g, sh, world, k0, v0, k1, v1, kn, vn):
    """A rank's cache after the gathers: two cached slices, and the current slice's padded shards (what the
    all-gathers of every rank's shard write) committed as the newest page."""
    w = sh.width
    cache = fvsr.KVCache(g, 2, 1, page_blocks=w * world)
    for k, v in ((k0, v0), (k1, v1)):
        cache.append(k, v, 1)
    kp, vp, pkp = cache.reserve()
    assert kp.shape == (w * world * 128, g.channels) and pkp.shape == (w * world, g.channels)
    for r2 in range(world):
        s2 = fvsr.query_shard(g.nq, world, r2)
        if s2.blocks:
            kp[r2 * w * 128:r2 * w * 128 + s2.blocks * 128] = kn[s2.begin * 128:s2.end * 128]
            vp[r2 * w * 128:r2 * w * 128 + s2.blocks * 128] = vn[s2.begin * 128:s2.end * 128]
            pkp[r2 * w:r2 * w + s2.blocks] = fvsr.pool(kn[s2.begin * 128:s2.end * 128], g)
    cache.commit()
    return cache


@pytest.mark.gpu
@pytest.mark.parametrize("cfg_id,world", [(2, 2), (2, 7), (3, 8)])
def test_emulated_ranks_reassemble_the_one_gpu_layer(fvsr, orc, cfg_id, world):
    """Every rank in turn on one GPU. One-launch form (fvsr_lcsa_forward_shard): the selection and the rank's output
    rows equal fvsr_lcsa_forward's bit for bit. Split form (select, then the cached slices' blocks into fp32
    partials, then the current slice's merged): the selection is the same and the rows are within the bf16 bar of
    the fp32 oracle, as the one-launch rows are."""
    if not torch.cuda.is_available():
        pytest.skip("no CUDA device")
    cfgs = importlib.import_module("fvsr_b200.configs")
    cfg = cfgs.CONFIGS[cfg_id]
    g = cfg.geometry(q_slices=1, kv_slices=3)
    k0, v0, k1, v1, q, kn, vn = _slices(cfgs, cfg, g, 40 + world, 7)
    ref_cache = fvsr.KVCache(g, 2, 1)
    for k, v in ((k0, v0), (k1, v1)):
        ref_cache.append(k, v, 1)
    kidx = torch.empty((g.heads, g.nq, g.nk), dtype=torch.int32, device="cuda")
    kcnt = torch.empty((g.heads, g.nq), dtype=torch.int32, device="cuda")
    ref = fvsr.lcsa_forward(q, kn, vn, ref_cache, g, kidx=kidx, kcnt=kcnt)
    ref_k, ref_v = ref_cache.gather()
    pq_full = fvsr.pool(q, g)
    oracle = orc.attention(q.float().cpu().numpy(), torch.cat([k0, k1, kn]).float().cpu().numpy(),
                           torch.cat([v0, v1, vn]).float().cpu().numpy(), kidx.cpu().numpy(), kcnt.cpu().numpy(),
                           g.heads, fast=True)
    full = fvsr.Geometry(**{**g.__dict__, "kv_slices": 3})
    for r in range(world):
        sh = fvsr.query_shard(g.nq, world, r)
        rows = slice(sh.begin * 128, sh.end * 128)
        cache = _rank_cache(fvsr, g, sh, world, k0, v0, k1, v1, kn, vn)
        rk = torch.full_like(kidx, -7)
        rc = torch.full_like(kcnt, -7)
        out = torch.empty((sh.blocks * 128, g.channels), dtype=torch.bfloat16, device="cuda")
        if sh.blocks:
            fvsr.lcsa_forward_shard(q[rows], sh, pq_full, cache, g, out=out, kidx=rk, kcnt=rc)
            torch.cuda.synchronize()
            assert torch.equal(rk, kidx) and torch.equal(rc, kcnt), f"rank {r}: selection differs"
            assert torch.equal(out.view(torch.int16), ref[rows].view(torch.int16)), r
        assert cache.slices == 2
        ck, cv = cache.gather()
        assert torch.equal(ck, ref_k) and torch.equal(cv, ref_v)
        cache.close()
        if not sh.blocks:
            continue
        # the split form, on a fresh copy of the rank's cache
        cache = _rank_cache(fvsr, g, sh, world, k0, v0, k1, v1, kn, vn)
        ws = fvsr.make_workspace(full)
        part = torch.empty(fvsr.partial_size(g, sh), dtype=torch.uint8, device="cuda")
        rc2 = torch.full_like(kcnt, -7)
        out2 = torch.empty_like(out)
        fvsr.lcsa_select_shard(pq_full, sh, cache, g, ws, kcnt=rc2)
        fvsr.lcsa_attend_shard(q[rows], sh, cache, g, ws, out2, partial=part, kcnt=rc2)
        torch.cuda.synchronize()
        assert torch.equal(rc2, kcnt)
        got = out2.float().cpu().numpy()
        cmp = orc.compare(got, oracle[rows])
        assert cmp["rel"] <= 1e-2, (r, cmp)
        assert orc.compare(got, out.float().cpu().numpy())["rel"] <= 1e-2
        assert cache.slices == 2
        cache.close()
    ref_cache.close()
    fvsr.device_check()


def _nccl_rank(rank, world, port, root, q_out):
    import sys
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port), NCCL_NVLS_ENABLE="0")
    torch.cuda.set_device(rank)
    import torch.distributed as dist
    import datetime
    dist.init_process_group("nccl", rank=rank, world_size=world, timeout=datetime.timedelta(seconds=60),
                            device_id=torch.device("cuda", rank))
    sys.path.insert(0, root)
    from __graft_entry__ import _load_package
    fvsr = _load_package()
    cfgs = importlib.import_module("fvsr_b200.configs")
    nccl = importlib.import_module("fvsr_b200.nccl")
    shard_mod = importlib.import_module("fvsr_b200.shard")
    cfg = cfgs.CONFIGS[2]
    g = cfg.geometry(q_slices=1, kv_slices=3)
    k0, v0, k1, v1, q, kn, vn = _slices(cfgs, cfg, g, 77, 7)          # same seeds on every rank
    comm = nccl.Comm(rank, world, torch.device("cuda", rank))
    ref_cache = fvsr.KVCache(g, 2, 1)
    ref_cache.append(k0, v0, 1)
    ref_cache.append(k1, v1, 1)
    ref = fvsr.lcsa_forward(q, kn, vn, ref_cache, g)
    results = []
    # the one-call form (gather after the selection, no split): bit for bit; the default form (gather beside the
    # selection and the cached slices' attention, merged partials): within the bf16 bar of the one-GPU rows
    for split, spare in ((False, 0), (True, 32)):
        sc = shard_mod.ShardedChunk(fvsr, g, 2, 1, rank, world, comm, split=split, spare_sms=spare)
        sc.prefill(0, [k0, k1], [v0, v1])
        sh = sc.shard
        kpad = torch.zeros((sc.shard_rows(), g.channels), dtype=torch.bfloat16, device="cuda")
        vpad = torch.zeros_like(kpad)
        kpad[:sh.blocks * 128] = kn[sh.begin * 128:sh.end * 128]
        vpad[:sh.blocks * 128] = vn[sh.begin * 128:sh.end * 128]
        out = torch.empty((sh.blocks * 128, g.channels), dtype=torch.bfloat16, device="cuda")
        sc.layer(0, q[sh.begin * 128:sh.end * 128].contiguous(), kpad, vpad, out)
        torch.cuda.synchronize()
        comm.check()
        want = ref[sh.begin * 128:sh.end * 128]
        if split:
            rel = ((out.float() - want.float()).abs().max() / want.float().abs().max()).item()
            results.append(rel <= 1e-2)
        else:
            results.append(torch.equal(out.view(torch.int16), want.view(torch.int16)))
        sc.close()
    same = all(results)
    q_out.put((rank, bool(same)))
    comm.destroy()
    dist.destroy_process_group()


@pytest.mark.gpu
def test_nccl_ranks_reassemble_the_one_gpu_layer(fvsr):
    if not torch.cuda.is_available() or torch.cuda.device_count() < 2:
        pytest.skip("needs two GPUs")
    import torch.multiprocessing as mp
    world = 2
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    root = str(__import__("pathlib").Path(__file__).resolve().parent.parent)
    port = 29600 + os.getpid() % 1000
    procs = [ctx.Process(target=_nccl_rank, args=(r, world, port, root, q)) for r in range(world)]
    for p in procs:
        p.start()
    res = dict(q.get(timeout=300) for _ in range(world))
    for p in procs:
        p.join(timeout=120)
    assert res == {0: True, 1: True}, res

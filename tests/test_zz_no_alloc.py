"""fvsr_lcsa_select_noalloc — selection for callers that cannot allocate device memory (an engine that owns every
buffer under a fixed budget, or a real-time thread that must not take an allocation's device-wide synchronisation).

Called through the C ABI and checked against the workspace-based fvsr_lcsa_select on the same inputs. Selection is
bit-exact by design, so the bar is equality. Two calls in a row of different sizes check that the shared scratch
array, which keeps the previous call's contents, does not leak into the next result. This file is collected last so
that a run stopping at the first failure has already run every other test; it also passes alone in a fresh process.
"""
from __future__ import annotations

import ctypes
import importlib

import pytest

torch = pytest.importorskip("torch")
pytestmark = pytest.mark.gpu


@pytest.fixture(scope="module")
def cfgs(fvsr):
    if not torch.cuda.is_available():
        pytest.skip("no CUDA device")
    return importlib.import_module("fvsr_b200.configs")


def _noalloc(fvsr, g, q, k, pooled_k=None):
    dev = q.device
    kidx = torch.full((g.heads, g.nq, g.nk), 7, dtype=torch.int32, device=dev)
    kcnt = torch.full((g.heads, g.nq), 7, dtype=torch.int32, device=dev)
    mask = torch.full((g.heads, g.nq, g.nk), 7, dtype=torch.uint8, device=dev)
    probs = torch.full((g.heads, g.nq, g.nk), 7.0, dtype=torch.float32, device=dev)
    p = g.params()
    st = fvsr.lib().fvsr_lcsa_select_noalloc(ctypes.byref(p), fvsr._ptr(q), fvsr._ptr(k), fvsr._ptr(pooled_k),
                                             fvsr._ptr(kidx), fvsr._ptr(kcnt), fvsr._ptr(mask), fvsr._ptr(probs),
                                             fvsr._stream())
    assert st == fvsr.FVSR_OK, fvsr.lib().fvsr_last_error()
    return {"kidx": kidx, "kcnt": kcnt, "mask": mask, "probs": probs}


def test_noalloc_matches_workspace_entry_point_two_calls_in_a_row(fvsr, cfgs):
    for cfg_id, seed in ((3, 31), (2, 32)):  # the larger call first, so the second one finds stale scratch
        cfg = cfgs.CONFIGS[cfg_id]
        g = cfg.geometry()
        q, k, _ = cfgs.synth_qkv(cfg, g, seed)
        got = _noalloc(fvsr, g, q, k)
        want = fvsr.draft_block_mask_and_probs(q, k, g)
        torch.cuda.synchronize()
        for key in ("kidx", "kcnt", "mask"):
            assert torch.equal(got[key], want[key]), (cfg_id, key)
        assert torch.equal(got["probs"].view(torch.int32), want["probs"].view(torch.int32)), cfg_id
    fvsr.device_check()


def _same(got, want, tag):
    for key in ("kidx", "kcnt", "mask"):
        assert torch.equal(got[key], want[key]), (tag, key)
    assert torch.equal(got["probs"].view(torch.int32), want["probs"].view(torch.int32)), tag


def test_noalloc_with_pooled_keys_matches(fvsr, cfgs):
    """The streaming caller's form: pooled keys passed in (the cache keeps them), so no key scratch is reserved and
    the histograms sit at another offset of the array. Bit-exact against fvsr_lcsa_select given the same keys."""
    cfg = cfgs.CONFIGS[2]
    g = cfg.geometry()
    q, k, _ = cfgs.synth_qkv(cfg, g, 33)
    pk = fvsr.pool(k, g)
    got = _noalloc(fvsr, g, q, None, pooled_k=pk)
    want = fvsr.draft_block_mask_and_probs(q, None, g, pooled_k=pk)
    torch.cuda.synchronize()
    _same(got, want, "pooled keys")
    fvsr.device_check()


def test_noalloc_call_recorded_in_a_graph(fvsr, cfgs):
    """A call made inside a stream capture uses the address found by the context's uncaptured calls; the replayed
    graph gives the same result as the direct entry point on new inputs copied into the captured buffers."""
    cfg = cfgs.CONFIGS[2]
    g = cfg.geometry()
    q, k, _ = cfgs.synth_qkv(cfg, g, 34)
    _noalloc(fvsr, g, q, k)                       # an uncaptured call in this context first
    torch.cuda.synchronize()
    s = torch.cuda.Stream()
    s.wait_stream(torch.cuda.current_stream())
    graph = torch.cuda.CUDAGraph()
    with torch.cuda.graph(graph, stream=s):
        got = _noalloc(fvsr, g, q, k)
    q2, k2, _ = cfgs.synth_qkv(cfg, g, 35)
    q.copy_(q2)
    k.copy_(k2)
    graph.replay()
    want = fvsr.draft_block_mask_and_probs(q2, k2, g)
    torch.cuda.synchronize()
    _same(got, want, "graph replay")
    del graph
    fvsr.device_check()


def test_noalloc_rejects_calls_beyond_its_scratch(fvsr, cfgs):
    g = fvsr.Geometry(heads=12, bh=12, bw=20, q_slices=1, kv_slices=8, local_range=11, topk=100)  # pooled keys > 8 MiB
    t = torch.zeros((128, g.channels), dtype=torch.bfloat16, device="cuda")
    p = g.params()
    st = fvsr.lib().fvsr_lcsa_select_noalloc(ctypes.byref(p), fvsr._ptr(t), fvsr._ptr(t), None, fvsr._ptr(t),
                                             fvsr._ptr(t), None, fvsr._ptr(t), fvsr._stream())
    assert st == fvsr.FVSR_EUNSUPPORTED
    assert b"scratch" in fvsr.lib().fvsr_last_error()

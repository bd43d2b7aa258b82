"""Properties the C ABI states for its layer calls (include/fvsr_lcsa.h, "Conventions"), checked directly:

- the last error message is per calling thread (CPU: host validation only);
- select → item order → attention can be captured into a CUDA graph and replayed: no allocation and no host
  synchronisation inside a call, and a replay reads its input buffers afresh (GPU);
- calls on distinct streams from distinct host threads, each with its own workspace, run side by side and give
  results identical to the same calls run one after another (GPU).

The reference is single-threaded on one stream (Pipeline.swift:178-179); these are properties of the replacement."""
from __future__ import annotations

import ctypes
import importlib
import threading

import pytest

torch = pytest.importorskip("torch")


def test_last_error_is_per_thread(fvsr):
    """Two threads fail with different messages; each still reads its own after the other failed."""
    L = fvsr.lib()
    n = ctypes.c_size_t(0)
    barrier = threading.Barrier(2, timeout=30)
    seen: dict[str, bytes] = {}
    errors: list[BaseException] = []

    def worker(name: str, field: str, value: int, first: bool):
        try:
            g = fvsr.Geometry(heads=12, bh=6, bw=10, q_slices=1, kv_slices=3, local_range=11, topk=10)
            p = g.params()
            setattr(p, field, value)
            if not first:
                barrier.wait()                      # the other thread has failed first
            assert L.fvsr_lcsa_workspace_size(ctypes.byref(p), ctypes.byref(n)) != fvsr.FVSR_OK
            if first:
                barrier.wait()
            barrier.wait()                          # both have failed
            seen[name] = L.fvsr_last_error()
        except BaseException as e:                  # re-raised in the main thread
            errors.append(e)
            barrier.abort()

    ts = [threading.Thread(target=worker, args=("a", "heads", 0, True)),
          threading.Thread(target=worker, args=("b", "head_dim", 64, False))]
    for t in ts:
        t.start()
    for t in ts:
        t.join(60)
    assert not errors, errors
    assert seen["a"] and seen["b"] and seen["a"] != seen["b"], seen


@pytest.fixture(scope="module")
def cfgs(fvsr):
    if not torch.cuda.is_available():
        pytest.skip("no CUDA device")
    return importlib.import_module("fvsr_b200.configs")


def _layer(fvsr, g, q, k, v, ws, stream=None, mask=False):
    """pool + selection into `ws`, longest-first item order, attention over every item; returns the results."""
    r = fvsr.draft_block_mask_and_probs(q, k, g, want_mask=mask, want_probs=mask, workspace=ws, stream=stream)
    items = g.heads * g.nq
    order = fvsr.item_order(r["kcnt"], g, 0, items, stream=stream)
    out = torch.empty_like(q)
    fvsr.block_sparse_attention_range(q, k, v, r["kidx"], r["kcnt"], g, 0, items, out, order=order, stream=stream)
    return r, out


@pytest.mark.gpu
def test_layer_replays_from_a_cuda_graph(fvsr, cfgs):
    cfg = cfgs.CONFIGS[2]
    g = cfg.geometry()
    q, k, v = cfgs.synth_qkv(cfg, g, cfgs.seed_of(2, 0, 3))
    ws = fvsr.make_workspace(g)
    side = torch.cuda.Stream()
    side.wait_stream(torch.cuda.current_stream())
    with torch.cuda.stream(side):
        _layer(fvsr, g, q, k, v, ws)                # warm-up outside the capture
    torch.cuda.current_stream().wait_stream(side)
    torch.cuda.synchronize()
    graph = torch.cuda.CUDAGraph()
    with torch.cuda.graph(graph):
        r_g, out_g = _layer(fvsr, g, q, k, v, ws)
    prev = None
    for seed in (11, 12):
        q2, k2, v2 = cfgs.synth_qkv(cfg, g, seed)
        q.copy_(q2)
        k.copy_(k2)
        v.copy_(v2)
        graph.replay()
        r_e, out_e = _layer(fvsr, g, q, k, v, ws)   # eager, same buffers, after the replay on the same stream
        torch.cuda.synchronize()
        assert torch.equal(r_g["kidx"], r_e["kidx"]) and torch.equal(r_g["kcnt"], r_e["kcnt"]), f"seed {seed}"
        assert torch.equal(out_g, out_e), f"seed {seed}"
        if prev is not None:
            assert not torch.equal(out_g, prev)     # the replay saw the new inputs
        prev = out_g.clone()
    del graph
    fvsr.device_check()


@pytest.mark.gpu
def test_calls_on_distinct_streams_from_distinct_threads(fvsr, cfgs):
    cfg = cfgs.CONFIGS[2]
    g = cfg.geometry()
    n, reps = 4, 3
    inputs = [cfgs.synth_qkv(cfg, g, cfgs.seed_of(2, 1, i)) for i in range(n)]
    want = [_layer(fvsr, g, *inputs[i], fvsr.make_workspace(g), mask=True) for i in range(n)]
    torch.cuda.synchronize()

    got: list = [None] * n
    errors: list[BaseException] = []
    barrier = threading.Barrier(n, timeout=60)

    def worker(i: int):
        try:
            s = torch.cuda.Stream()
            with torch.cuda.stream(s):
                ws = fvsr.make_workspace(g)
                barrier.wait()
                for _ in range(reps):
                    res = _layer(fvsr, g, *inputs[i], ws, stream=s, mask=True)
                s.synchronize()
                got[i] = res
        except BaseException as e:                  # re-raised in the main thread
            errors.append(e)
            barrier.abort()

    ts = [threading.Thread(target=worker, args=(i,)) for i in range(n)]
    for t in ts:
        t.start()
    for t in ts:
        t.join(120)
    assert not errors, errors
    for i in range(n):
        (rw, ow), (rg, og) = want[i], got[i]
        for key in ("mask", "probs", "kidx", "kcnt"):
            assert torch.equal(rw[key], rg[key]), f"thread {i}: {key}"
        assert torch.equal(ow, og), f"thread {i}: attention output"
    fvsr.device_check()

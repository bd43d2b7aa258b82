"""CPU tests of the C ABI: the library loads, exports every entry point include/fvsr_lcsa.h declares, and rejects bad
arguments on the host before touching a device. No compute call needs a GPU here."""
from __future__ import annotations

import ctypes
import re
from pathlib import Path

import pytest

ROOT = Path(__file__).resolve().parent.parent


def declared_symbols() -> list[str]:
    text = (ROOT / "include" / "fvsr_lcsa.h").read_text()
    text = re.sub(r"/\*.*?\*/", "", text, flags=re.S)
    return sorted(set(re.findall(r"\b(fvsr_[a-z0-9_]+)\s*\(", text)))


def test_header_declares_the_boundary():
    syms = declared_symbols()
    for must in ("fvsr_lcsa_select", "fvsr_lcsa_attention", "fvsr_lcsa_forward", "fvsr_kv_cache_append",
                 "fvsr_lcsa_workspace_size"):
        assert must in syms


def test_library_exports_every_declared_symbol(fvsr):
    L = fvsr.lib()
    missing = [s for s in declared_symbols() if not hasattr(L, s)]
    assert not missing, missing
    assert sorted(fvsr.EXPORTED) == declared_symbols()


def test_version_and_status_strings(fvsr):
    L = fvsr.lib()
    assert L.fvsr_version() >= 100
    assert L.fvsr_status_string(fvsr.FVSR_OK) == b"ok"
    assert b"timed out" in L.fvsr_status_string(fvsr.FVSR_ETIMEOUT)


def test_workspace_size_matches_layout(fvsr):
    g = fvsr.Geometry(heads=12, bh=9, bw=15, q_slices=1, kv_slices=3, local_range=11, topk=8384)
    n = fvsr.workspace_size(g)
    a = lambda x: (x + 255) // 256 * 256  # noqa: E731
    c = 12 * 128
    want = a(g.nq * c * 4) + a(g.nk * c * 4) + a(12 * g.nq * g.nk * 4) * 2 + a(12 * g.nq * 4) + a(12 * 1 * 5136 * 4) + a(12 * g.nq * 4)
    assert n == want


@pytest.mark.parametrize("field,value,status", [
    ("heads", 0, 1), ("head_dim", 64, 1), ("bh", 0, 1), ("q_slices", 0, 1), ("kv_slices", 0, 1),
    ("local_range", 0, 1), ("topk", -1, 1), ("dtype", 7, 1), ("kv_slices", 100, 5),
])
def test_bad_params_rejected_on_host(fvsr, field, value, status):
    g = fvsr.Geometry(heads=12, bh=6, bw=10, q_slices=1, kv_slices=3, local_range=11, topk=10)
    p = g.params()
    setattr(p, field, value)
    n = ctypes.c_size_t(0)
    assert fvsr.lib().fvsr_lcsa_workspace_size(ctypes.byref(p), ctypes.byref(n)) == status
    assert fvsr.lib().fvsr_last_error()


def test_null_pointers_rejected_before_any_launch(fvsr):
    L = fvsr.lib()
    g = fvsr.Geometry(heads=2, bh=2, bw=2, q_slices=1, kv_slices=2, local_range=3, topk=3)
    p = g.params()
    assert L.fvsr_lcsa_select(ctypes.byref(p), None, None, None, None, None, None, None, None, 0, None) == fvsr.FVSR_EINVAL
    assert L.fvsr_lcsa_attention(ctypes.byref(p), None, None, None, None, None, None, None) == fvsr.FVSR_EINVAL
    assert L.fvsr_lcsa_pool(None, None, 0, None, None) == fvsr.FVSR_EINVAL
    assert L.fvsr_kv_cache_trim(None) == fvsr.FVSR_EINVAL
    h = ctypes.c_void_p()
    assert L.fvsr_kv_cache_create(ctypes.byref(p), 0, 1, ctypes.byref(h)) == fvsr.FVSR_EINVAL
    assert L.fvsr_kv_cache_create(ctypes.byref(p), 30, 5, ctypes.byref(h)) == fvsr.FVSR_EINVAL
    assert L.fvsr_kv_cache_destroy(None) == fvsr.FVSR_OK


def test_misaligned_pointer_rejected(fvsr):
    L = fvsr.lib()
    g = fvsr.Geometry(heads=2, bh=2, bw=2, q_slices=1, kv_slices=2, local_range=3, topk=3)
    p = g.params()
    bad = ctypes.c_void_p(0x1000 + 4)
    ok = ctypes.c_void_p(0x1000)
    assert L.fvsr_lcsa_attention(ctypes.byref(p), bad, ok, ok, ok, ok, ok, None) == fvsr.FVSR_EINVAL
    assert b"aligned" in L.fvsr_last_error()


@pytest.mark.parametrize("bh,bw,q_slices", [(65536, 65536, 1), (1 << 16, 1 << 15, 1), (2, 2, 2**31 - 1),
                                             (1, 1, 65535), (1, 1, 6000)])
def test_huge_geometry_rejected_without_overflow(fvsr, bh, bw, q_slices):
    """Block counts are formed in 64 bits: grids whose 32-bit product wraps (to zero or a negative count) are
    rejected as unsupported, not accepted as tiny problems."""
    g = fvsr.Geometry(heads=12, bh=bh, bw=bw, q_slices=q_slices, kv_slices=1, local_range=11, topk=10)
    p = g.params()
    n = ctypes.c_size_t(0)
    assert fvsr.lib().fvsr_lcsa_workspace_size(ctypes.byref(p), ctypes.byref(n)) == 5   # FVSR_EUNSUPPORTED
    assert b"too large" in fvsr.lib().fvsr_last_error() or b"exceeds" in fvsr.lib().fvsr_last_error()
    if q_slices == 65535:   # Nq + Nk = 65536: too many for one selection; Nq alone is allowed where no key blocks are
        g.kv_slices = 0     # involved (pooling, cache, prepare)
        assert fvsr.lib().fvsr_lcsa_pool(ctypes.byref(g.params()), None, 0, None, None) == fvsr.FVSR_OK


def test_misaligned_buffers_rejected_by_every_entry_point(fvsr):
    """Every pointer a kernel dereferences is checked for its access width on the host: 16 bytes for rows, the
    workspace and schedules; 4 bytes for index lists, counts, orders, probabilities, masks, pooled rows and norm weights.
    The addresses are never dereferenced: each call fails its host check before any device call."""
    L = fvsr.lib()
    g = fvsr.Geometry(heads=2, bh=2, bw=2, q_slices=1, kv_slices=2, local_range=3, topk=3, dtype=fvsr.FVSR_BF16)
    p = ctypes.byref(g.params())
    ok = ctypes.c_void_p(1 << 20)
    odd2 = ctypes.c_void_p((1 << 20) + 2)    # not 4-byte aligned
    odd4 = ctypes.c_void_p((1 << 20) + 4)    # 4- but not 16-byte aligned
    big = 1 << 30
    n = g.heads * g.nq
    eps = ctypes.c_float(1e-6)
    calls = {
        "select kidx": lambda: L.fvsr_lcsa_select(p, ok, ok, None, odd2, ok, None, None, ok, big, None),
        "select probs": lambda: L.fvsr_lcsa_select(p, ok, ok, None, ok, ok, None, odd2, ok, big, None),
        "select workspace": lambda: L.fvsr_lcsa_select(p, ok, ok, None, ok, ok, None, None, odd4, big, None),
        "attention kcnt": lambda: L.fvsr_lcsa_attention(p, ok, ok, ok, ok, odd2, ok, None),
        "range order": lambda: L.fvsr_lcsa_attention_range(p, ok, ok, ok, ok, ok, ok, 0, n, odd2, None),
        "item order kcnt": lambda: L.fvsr_lcsa_item_order(p, odd2, 0, n, ok, None),
        "schedule kcnt": lambda: L.fvsr_lcsa_schedule(p, odd2, 0, n, ok, big, None),
        "scheduled kidx": lambda: L.fvsr_lcsa_attention_scheduled(p, ok, ok, ok, odd2, ok, ok, 0, n, ok, big, None),
        "mask form mask": lambda: L.fvsr_lcsa_attention_mask(p, ok, ok, ok, odd2, ok, ok, big, None),
        "mask form workspace": lambda: L.fvsr_lcsa_attention_mask(p, ok, ok, ok, ok, ok, odd4, big, None),
        "noalloc kcnt": lambda: L.fvsr_lcsa_select_noalloc(p, ok, ok, None, ok, odd2, None, ok, None),
        "noalloc q": lambda: L.fvsr_lcsa_select_noalloc(p, odd4, ok, None, ok, ok, None, ok, None),
        "prepare norm": lambda: L.fvsr_lcsa_prepare(p, ok, ok, ok, odd2, None, eps, None, None, ok, ok, ok, None, None,
                                                    None),
        "prepare pooled": lambda: L.fvsr_lcsa_prepare(p, ok, ok, ok, None, None, eps, None, None, ok, ok, ok, odd2,
                                                      None, None),
    }
    for name, call in calls.items():
        assert call() == fvsr.FVSR_EINVAL, name
        assert b"aligned" in L.fvsr_last_error(), (name, L.fvsr_last_error())


def test_topk_formula_and_allowed_counts(fvsr):
    """DiT.swift:482 and the per-row allowed counts the configs translate their keep fractions with."""
    assert fvsr.Geometry.topk_from_ratio(60, 2.0) == 7199
    counts = {2: 8640, 3: 27945, 5: 58140}
    import importlib
    cfgs = importlib.import_module("fvsr_b200.configs").CONFIGS
    for c, want in counts.items():
        assert cfgs[c].geometry().allowed_per_row() == want
    assert cfgs[3].geometry().topk == 8384
    assert cfgs[5].geometry().topk == 14535
    assert cfgs[1].geometry().topk == 96


def test_token_order_entry_points_check_arguments_on_host(fvsr):
    """fvsr_lcsa_prepare / fvsr_lcsa_forward_tokens reject bad arguments before any launch (the addresses below are
    never dereferenced: every case fails a host check first)."""
    L = fvsr.lib()
    fake = ctypes.c_void_p(1 << 20)  # 16-byte aligned, never touched
    g = fvsr.Geometry(heads=17, bh=2, bw=2, q_slices=1, kv_slices=1, local_range=3, topk=3)
    p = g.params()
    args = [fake, fake, fake, None, None, ctypes.c_float(1e-6), None, None, fake, fake, fake, None, None, None]
    assert L.fvsr_lcsa_prepare(ctypes.byref(p), *args) == fvsr.FVSR_EUNSUPPORTED
    p.heads = 2
    bad = list(args)
    bad[6] = fake  # cos without sin
    assert L.fvsr_lcsa_prepare(ctypes.byref(p), *bad) == fvsr.FVSR_EINVAL
    assert b"together" in L.fvsr_last_error()
    bad = list(args)
    bad[0] = ctypes.c_void_p((1 << 20) + 8)  # misaligned q_lin
    assert L.fvsr_lcsa_prepare(ctypes.byref(p), *bad) == fvsr.FVSR_EINVAL
    bad = list(args)
    bad[9] = None  # no k_win
    assert L.fvsr_lcsa_prepare(ctypes.byref(p), *bad) == fvsr.FVSR_EINVAL
    bad = list(args)
    bad[3], bad[5] = fake, ctypes.c_float(-1.0)  # a norm with a negative eps
    assert L.fvsr_lcsa_prepare(ctypes.byref(p), *bad) == fvsr.FVSR_EINVAL
    assert L.fvsr_lcsa_forward_tokens(ctypes.byref(p), fake, fake, fake, None, None, ctypes.c_float(1e-6), None, None,
                                      None, fake, fake, None, None, fake, 1 << 20, None) == fvsr.FVSR_EINVAL


def test_wait_probe_limit_checked_on_host(fvsr):
    L = fvsr.lib()
    assert L.fvsr_wait_probe(0, None) == fvsr.FVSR_EINVAL
    assert L.fvsr_wait_probe(4_000_001, None) == fvsr.FVSR_EINVAL


def test_linear_rejects_bad_shapes_before_any_launch(fvsr):
    """fvsr_linear / fvsr_linear_qkv check the tile multiples and the pointers on the host (no device needed)."""
    L = fvsr.lib()
    p = 16  # any non-NULL, aligned address: nothing is launched
    for m, n, k in ((100, 256, 64), (128, 200, 64), (128, 256, 60), (0, 256, 64)):
        assert L.fvsr_linear(m, n, k, p, p, None, 0, None, None, p, None) == fvsr.FVSR_EINVAL
        assert b"multiple" in L.fvsr_last_error()
    assert L.fvsr_linear(128, 256, 64, None, p, None, 0, None, None, p, None) == fvsr.FVSR_EINVAL
    assert L.fvsr_linear(128, 256, 64, p, p, None, 2, None, None, p, None) == fvsr.FVSR_EINVAL   # gate, resid
    assert L.fvsr_linear(128, 256, 64, p, p, None, 7, None, None, p, None) == fvsr.FVSR_EINVAL   # epilogue
    assert L.fvsr_linear_qkv(128, 100, 64, p, p, None, p, p, p, None) == fvsr.FVSR_EINVAL


def test_block_ops_reject_bad_arguments_before_any_launch(fvsr):
    L = fvsr.lib()
    p = 16
    assert L.fvsr_layernorm(8, 100, p, None, None, None, None, 1e-6, p, None) == fvsr.FVSR_EINVAL
    assert L.fvsr_layernorm(8, 4096, p, None, None, None, None, 1e-6, p, None) == fvsr.FVSR_EINVAL
    assert L.fvsr_layernorm(8, 256, p, None, None, p, None, 1e-6, p, None) == fvsr.FVSR_EINVAL     # shift w/o scale
    assert L.fvsr_layernorm(8, 256, p, None, p, None, None, 1e-6, p, None) == fvsr.FVSR_EINVAL     # bias w/o weight
    assert L.fvsr_rmsnorm(8, 256, p, None, 1e-6, p, None) == fvsr.FVSR_EINVAL                      # no weight
    assert L.fvsr_cross_attention(12, 100, 512, p, p, p, p, None) == fvsr.FVSR_EINVAL
    assert L.fvsr_cross_attention(0, 128, 128, p, p, p, p, None) == fvsr.FVSR_EINVAL
